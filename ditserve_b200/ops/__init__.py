"""Hot DiT ops.  CUDA tensors run the hand-written sm_100a kernels of
``ditserve_b200._C``; CPU tensors run the fp32 PyTorch statement of the same op."""
from ._ext import KernelTimeout, KernelTimer, available, check_status, ext, kernel, launch_counts, status_word
from .attention import (SPARSE_K_BLOCK, SPARSE_Q_BLOCK, attention, attention_reference, attention_segments,
                        block_sparse_table, segment_table, segments_reference, sliding_window_block_mask,
                        tile_window_block_mask, token_mask)
from .conv import conv_bias, conv_cl, conv_cl_reference, conv_weight_2d
from .gemm import linear, linear_reference
from .norm import (layernorm_modulate, layernorm_modulate_reference, rms_norm_reference, rmsnorm_rope_, rmsnorm_rope_qk_,
                   rope_reference)
from .sched import sched_step, sched_step_reference

__all__ = [
    "KernelTimeout", "KernelTimer", "available", "check_status", "ext", "kernel", "launch_counts", "status_word",
    "SPARSE_K_BLOCK", "SPARSE_Q_BLOCK", "block_sparse_table", "sliding_window_block_mask", "tile_window_block_mask",
    "token_mask", "attention", "attention_reference", "conv_bias", "conv_cl", "conv_cl_reference", "conv_weight_2d", "attention_segments", "segment_table", "segments_reference", "linear", "linear_reference",
    "layernorm_modulate", "layernorm_modulate_reference", "rms_norm_reference", "rmsnorm_rope_", "rmsnorm_rope_qk_",
    "rope_reference", "sched_step", "sched_step_reference",
]
