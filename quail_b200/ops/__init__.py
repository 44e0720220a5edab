"""Python entry points of the sm_100a kernels in `quail_b200._C`.

Every op here runs the hand-written CUDA kernel; there is no PyTorch
fallback on a GPU. If the extension is missing on a machine with a GPU,
importing an op raises, so a test or a bench can never pass on eager
PyTorch by accident. `quail_b200.ops.reference` holds the plain fp32
PyTorch statement of each op, used by the CPU model and by the kernel
tests.
"""

from quail_b200.ops.kernels import (  # noqa: F401
    EPI_BF16,
    EPI_RESIDUAL,
    EPI_SWIGLU_BF16,
    EPI_GEGLU_BF16,
    EPI_GEGLU_FP8,
    EPI_SWIGLU_FP8,
    chunk_attention,
    decode_attention,
    embed_gather,
    final_norm_readout,
    gemm,
    gemm_mx,
    gemm_nvfp4,
    head_readout,
    READOUT_TOPK,
    quant_rows_nvfp4,
    sf_bytes,
    rmsnorm_quant_mx,
    quant_rows_mx,
    count_launch,
    kernels_available,
    launch_count,
    native,
    prefill_attention,
    prefill_attention_tc,
    prefill_attention_tc2,
    gemm_mx_qkv_rope,
    quant_mx_ss,
    row_rinv,
    EPI_RESIDUAL_MX,
    qk_norm_rope_kv,
    quant_rows,
    read_and_clear_error,
    set_wait_budget,
    rmsnorm_quant,
    sae_features,
    row_argmax_lse,
    small_attention,
    SMALL_ATTENTION_SHAPES,
    post_norm_add_norm,
    kv_copy_rows,
    attention_merge,
)
from quail_b200.ops.quant import (  # noqa: F401
    FP8_MAX,
    dequantize_act,
    dequantize_mx,
    interleave_gate_up_mx,
    quantize_act_mx,
    quantize_weight_mx,
    requantize_weight_mx,
    pack_sf_atoms,
    unpack_sf_atoms,
    dequantize_weight,
    interleave_gate_up,
    quantize_act,
    quantize_weight,
)
