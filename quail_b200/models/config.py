"""Decoder configurations of the model families the engine runs.

The numbers of the named architectures follow the Hugging Face configs of
Qwen/Qwen3-4B, -8B, -32B and -30B-A3B (the reference's model specs:
quail/specs/data/models/qwen3-4b-fp8.toml, qwen3-32b-fp8.toml).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    layers: int
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int          # dense SwiGLU width (per expert for MoE: moe_intermediate)
    vocab: int = 151_936
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    tied_head: bool = False
    weight_dtype: str = "fp8"  # "fp8" (e4m3 + 128x128 block scales) or "bf16"
    num_experts: int = 0
    top_k: int = 0
    moe_intermediate: int = 0
    max_position: int = 40_960
    init_std: float = 0.02
    # sparse autoencoder on the residual stream after the last loaded layer
    # (a model with one serves AI.SAE_FEATURES only); 0 = none
    sae_features: int = 0
    sae_keep: int = 0

    @property
    def q_dim(self) -> int:
        return self.num_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def has_sae(self) -> bool:
        return self.sae_features > 0

    @property
    def fp8(self) -> bool:
        return self.weight_dtype == "fp8"

    def dense_params_per_token(self) -> int:
        """Projection parameters each token multiplies (active experts only)."""
        attn = self.hidden * self.qkv_dim + self.q_dim * self.hidden
        if self.is_moe:
            mlp = self.top_k * 3 * self.hidden * self.moe_intermediate + self.hidden * self.num_experts
        else:
            mlp = 3 * self.hidden * self.intermediate
        return self.layers * (attn + mlp)

    def kv_bytes_per_token(self) -> int:
        return self.layers * 2 * self.kv_dim * 2

    def with_(self, **kw) -> "DecoderConfig":
        return replace(self, **kw)

    def to_dict(self) -> dict:
        return asdict(self)


QWEN3_4B = DecoderConfig(name="qwen3-4b", layers=36, hidden=2560, num_q_heads=32, num_kv_heads=8,
                         head_dim=128, intermediate=9728, tied_head=True)
QWEN3_8B = DecoderConfig(name="qwen3-8b", layers=36, hidden=4096, num_q_heads=32, num_kv_heads=8,
                         head_dim=128, intermediate=12288, weight_dtype="bf16")
QWEN3_32B = DecoderConfig(name="qwen3-32b", layers=64, hidden=5120, num_q_heads=64, num_kv_heads=8,
                          head_dim=128, intermediate=25600)
QWEN3_30B_A3B = DecoderConfig(name="qwen3-30b-a3b", layers=48, hidden=2048, num_q_heads=32,
                              num_kv_heads=4, head_dim=128, intermediate=6144, num_experts=128,
                              top_k=8, moe_intermediate=768)
# the CPU plumbing model (fp32, tiny)
QWEN3_TINY = DecoderConfig(name="qwen3-tiny", layers=2, hidden=256, num_q_heads=4, num_kv_heads=2,
                           head_dim=64, intermediate=768, weight_dtype="bf16")
# the smallest model the GPU kernels take (head_dim 128, hidden multiple of 256)
QWEN3_GPU_TINY = DecoderConfig(name="qwen3-gpu-tiny", layers=2, hidden=1024, num_q_heads=8,
                               num_kv_heads=4, head_dim=128, intermediate=1024)
# the smallest MoE the GPU kernels take: 16 experts, top-4, expert width 256
QWEN3_MOE_GPU_TINY = DecoderConfig(name="qwen3-moe-gpu-tiny", layers=2, hidden=1024, num_q_heads=8,
                                   num_kv_heads=2, head_dim=128, intermediate=1024, num_experts=16, top_k=4,
                                   moe_intermediate=256)
# AI.SAE_FEATURES models: a Qwen3 decoder truncated after the SAE's layer with a
# 32K-feature, keep-100 SAE (the shape of the reference's
# qwen3.5-2b-sae-bf16 spec: layers 0-11 of 24, W32K, L0 100), random init
QWEN3_4B_SAE = QWEN3_4B.with_(name="qwen3-4b-sae-bf16", layers=12, weight_dtype="bf16", sae_features=32768,
                              sae_keep=100)
QWEN3_SAE_TINY = QWEN3_TINY.with_(name="qwen3-sae-tiny", sae_features=512, sae_keep=16)
QWEN3_GPU_SAE_TINY = QWEN3_GPU_TINY.with_(name="qwen3-gpu-sae-tiny", weight_dtype="bf16", sae_features=2048,
                                          sae_keep=32)

CONFIGS = {c.name: c for c in (QWEN3_4B, QWEN3_8B, QWEN3_32B, QWEN3_30B_A3B, QWEN3_TINY, QWEN3_GPU_TINY,
                               QWEN3_MOE_GPU_TINY, QWEN3_4B_SAE, QWEN3_SAE_TINY, QWEN3_GPU_SAE_TINY)}

# model spec names (as in EngineConfig.model) -> decoder config
MODEL_CONFIGS = {
    "qwen3-4b-fp8": QWEN3_4B,
    "qwen3-4b-bf16": QWEN3_4B.with_(weight_dtype="bf16", name="qwen3-4b-bf16"),
    "qwen3-8b-bf16": QWEN3_8B,
    "qwen3-32b-fp8": QWEN3_32B,
    "qwen3-30b-a3b-fp8": QWEN3_30B_A3B,
    "qwen3-tiny": QWEN3_TINY,
    "qwen3-gpu-tiny": QWEN3_GPU_TINY,
    "qwen3-moe-gpu-tiny": QWEN3_MOE_GPU_TINY,
    "qwen3-4b-sae-bf16": QWEN3_4B_SAE,
    "qwen3-sae-tiny": QWEN3_SAE_TINY,
    "qwen3-gpu-sae-tiny": QWEN3_GPU_SAE_TINY,
}
