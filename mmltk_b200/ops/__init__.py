"""Hot ops of the RF-DETR stack.  CUDA tensors run the in-tree sm_100a kernels;
CPU tensors run the plain-PyTorch fp32 definitions that serve as test oracles."""
from ._ext import has_kernels, has_native, kernels, native
from .attention import (attention, attention_reference, qk_split_attention, qkv_attention, qkv_attention_reference,
                        short_attention,
                        short_attention_ok)
from .conv import conv3x3, conv3x3_ok
from .linear import ffn_add_norm, gather_rows, linear, linear_pair, linear_scale_residual, mlp_relu, mlp_scale_residual
from .msda import msda, msda_reference
from .norm import (add_layer_norm, concat_channels, grouped_layer_norm, layer_norm, layer_norm_with_residual,
                   scaled_residual_layer_norm, taps_layer_norm)
from .posembed import sine_embed, sine_embed_reference
from .losses import dense_focal_neg
