from .losses import SetCriterion
from .matcher import hungarian_match, matcher_cost_reference
from .targets import Targets, pad_targets
