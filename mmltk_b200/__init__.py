"""mmltk_b200: a Blackwell-native (sm_100a) RF-DETR training and inference framework.

PyTorch is the framework layer; the hot ops are in-tree CUDA kernels for
sm_100a and the DDP gradient path is an in-kernel NVSwitch collective.
"""
__version__ = "0.1.0"
