"""B200-native (sm_100a) Flow2Surf reverse-flow denoising.

Drop-in for the reference's hot path: the operators of flow2surf/models/ops,
the Flow2SurfNet model and patch_denoise, all computed by hand-written CUDA
kernels in libflow2surf_sm100.so behind a C-ABI (include/flow2surf_b200.h);
with the operators' backward passes and the training losses
(flow2surf/training/losses.py) on the same library.
"""

from .losses import dcd_loss, velocity_loss
from .network import Flow2SurfNet, build_model
from .ops import knn_indices, offset_attention_aggregate, reduce_neighbor_messages

__all__ = [
    "Flow2SurfNet",
    "build_model",
    "dcd_loss",
    "knn_indices",
    "offset_attention_aggregate",
    "reduce_neighbor_messages",
    "velocity_loss",
]
