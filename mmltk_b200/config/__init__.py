from .presets import PRESETS, PresetSpec, WEIGHT_CATALOG, find_preset, infer_preset_from_path, preset_names
from .model_config import RfDetrConfig, config_from_preset
from .train_options import AugmentationConfig, AugGroup, TrainOptions, apply_recipe, lr_scale, warmup_momentum
