"""B200-native batch-invariant operators (drop-in for ``batch_invariant_ops`` 0.2.0).

The public names mirror yiannisha/robotics-batch-invariant-ops
``batch_invariant_ops/__init__.py``; the kernels behind them are hand-written
sm_100a CUDA in ``libbio_sm100.so``.
"""

from .batch_invariant_ops import (
    AttentionBlockSize,
    bmm_persistent,
    conv1d_batch_invariant,
    conv2d_batch_invariant,
    conv3d_batch_invariant,
    conv_transpose2d_batch_invariant,
    conv_transpose3d_batch_invariant,
    disable_batch_invariant_mode,
    enable_batch_invariant_mode,
    gated_linear_batch_invariant,
    get_batch_invariant_attention_block_size,
    is_batch_invariant_mode_enabled,
    layer_norm_batch_invariant,
    linalg_vector_norm_batch_invariant,
    linear_batch_invariant,
    linear_residual_batch_invariant,
    log_softmax,
    matmul_persistent,
    mean_dim,
    rms_norm_batch_invariant,
    scaled_dot_product_attention_batch_invariant,
    set_batch_invariant_mode,
    softmax,
    varlen_scaled_dot_product_attention_batch_invariant,
)
from .moe import deterministic_token_choice_moe

__version__ = "0.2.0"

__all__ = [
    "set_batch_invariant_mode",
    "is_batch_invariant_mode_enabled",
    "disable_batch_invariant_mode",
    "enable_batch_invariant_mode",
    "matmul_persistent",
    "linear_batch_invariant",
    "bmm_persistent",
    "conv1d_batch_invariant",
    "conv2d_batch_invariant",
    "conv3d_batch_invariant",
    "conv_transpose2d_batch_invariant",
    "conv_transpose3d_batch_invariant",
    "scaled_dot_product_attention_batch_invariant",
    "varlen_scaled_dot_product_attention_batch_invariant",
    "linalg_vector_norm_batch_invariant",
    "softmax",
    "log_softmax",
    "mean_dim",
    "get_batch_invariant_attention_block_size",
    "AttentionBlockSize",
    "deterministic_token_choice_moe",
    # additions (no counterpart in the reference): fused normalisations and
    # the fused gated MLP input projection
    "layer_norm_batch_invariant",
    "rms_norm_batch_invariant",
    "gated_linear_batch_invariant",
    "linear_residual_batch_invariant",
]
