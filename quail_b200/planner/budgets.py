"""Memory budgets and the roofline cost model of a model on a device.

Same quantities as the reference's planner (crates/quail-planner/src/cost/
budgets.rs: POOL_FRACTION, ACT_RESERVE_CHUNKS, chunk_budget, arena_pages,
compute_knee, kernel_index_cap), computed for this engine's kernels:

- chunk_tokens: new tokens per forward pass. The tcgen05 GEMMs reach their
  throughput plateau near 16k rows (M) for the Qwen3 shapes, and a chunk's
  activations must fit beside the arena; capped so every int32 offset the
  kernels form stays in range.
- arena_pages: KV pages that fit in POOL_FRACTION of the device memory after
  the weights and ACT_RESERVE_CHUNKS chunks of activations.
- compute_knee: rows per pass where a projection turns from weight-bandwidth
  bound to tensor-core bound (peak FLOP/s x weight bytes / (2 x HBM B/s)).
"""

from __future__ import annotations

from dataclasses import dataclass

from quail_b200.planner.specs import DEVICES, DeviceSpec

POOL_FRACTION = 0.95
ACT_RESERVE_CHUNKS = 2
INT32_MAX = (1 << 31) - 1
DEFAULT_CHUNK_TOKENS = 16_384


def weight_bytes(cfg) -> float:
    wb = 1.0 if cfg.fp8 else 2.0
    proj = cfg.dense_params_per_token() * wb
    if cfg.is_moe:
        # every expert is resident, only top_k are read per token
        proj += cfg.layers * (cfg.num_experts - cfg.top_k) * 3 * cfg.hidden * cfg.moe_intermediate * wb
    embed = cfg.vocab * cfg.hidden * 2 * (1 if cfg.tied_head else 2)
    return proj + embed


def activation_bytes_per_token(cfg) -> int:
    """Peak live activation bytes per token of one layer's forward (bf16/e4m3 buffers)."""
    H = cfg.hidden
    inter = cfg.moe_intermediate * cfg.top_k if cfg.is_moe else cfg.intermediate
    return (2 * H            # residual
            + 2 * cfg.qkv_dim  # qkv bf16
            + 2 * cfg.q_dim    # q
            + cfg.q_dim + 64   # attention output e4m3 + scales
            + H + 64           # normed e4m3 + scales
            + inter + 64)      # SwiGLU output e4m3 + scales


def kernel_index_cap(cfg) -> int:
    """Largest chunk whose element offsets fit int32 in every kernel."""
    widest = max(cfg.qkv_dim, 2 * (cfg.moe_intermediate if cfg.is_moe else cfg.intermediate), cfg.hidden)
    return INT32_MAX // widest


KV_POOL_TOKENS_ENV = "QUAIL_KV_POOL_TOKENS"


def kv_pool_cap_tokens():
    """The KV pool cap QUAIL_KV_POOL_TOKENS sets, in tokens, or None."""
    import os
    v = os.environ.get(KV_POOL_TOKENS_ENV, "").strip()
    try:
        return int(v) if v else None
    except ValueError:
        raise ValueError(f"{KV_POOL_TOKENS_ENV}={v!r} is not a token count") from None


@dataclass
class Budgets:
    cfg: object
    device: DeviceSpec
    chunk_tokens: int
    gpus: int = 1

    @classmethod
    def for_model(cls, cfg, device_name: str, gpus: int = 1, chunk_tokens: int | None = None,
                  registry=None) -> "Budgets":
        dev = (registry.device(device_name) if registry is not None else None) or DEVICES[device_name]
        chunk = chunk_tokens or DEFAULT_CHUNK_TOKENS
        chunk = min(chunk, kernel_index_cap(cfg))
        free = dev.mem_bytes * POOL_FRACTION - weight_bytes(cfg)
        while chunk > 256 and ACT_RESERVE_CHUNKS * chunk * activation_bytes_per_token(cfg) > 0.25 * free:
            chunk //= 2
        return cls(cfg, dev, chunk, gpus)

    def state_slots(self, cfg) -> int:
        """Recurrent-state slots of a hybrid model: one per resident key (prefix, documents,
        questions in flight), bounded by a tenth of device memory (fp32 conv window + delta-rule
        state of every Gated DeltaNet layer per slot)."""
        if not cfg.is_hybrid:
            return 0
        per = len(cfg.gdn_layers) * 4 * ((cfg.conv_width - 1) * cfg.gdn_conv_dim
                                         + cfg.gdn_value_heads * cfg.gdn_key_dim * cfg.gdn_value_dim)
        per += len(cfg.conv_layers) * 4 * (cfg.conv_width - 1) * cfg.hidden
        cap = int(self.device.mem_bytes * 0.1 // per)
        if self.device.name == "cpu":
            cap = min(cap, 256)
        return max(16, min(cap, 4096))

    def arena_pages(self, page_tokens: int) -> int:
        cfg = self.cfg
        free = (self.device.mem_bytes * POOL_FRACTION - weight_bytes(cfg)
                - ACT_RESERVE_CHUNKS * self.chunk_tokens * activation_bytes_per_token(cfg))
        page_bytes = 2 * page_tokens * sum(cfg.kv_dims) * 2
        if self.device.name == "cpu":
            free = min(free, 2 << 30)
        pages = int(free // page_bytes)
        # room for at least two chunks of new KV
        need = 2 * (self.chunk_tokens // page_tokens + 64)
        if pages < need:
            raise MemoryError(f"the arena holds {pages} pages; a chunk of {self.chunk_tokens} tokens needs {need}")
        # enough for eight chunks in flight and retained documents; more
        # only costs start-up time zeroing memory nothing reads
        pages = min(pages, 8 * (self.chunk_tokens // page_tokens) + 256)
        cap = kv_pool_cap_tokens()
        if cap is not None:
            # an experiment's cap on the KV pool (the reference's QUAIL_KV_POOL_TOKENS,
            # crates/quail-planner/src/cost/budgets.rs:287-320)
            pages = min(pages, max(cap // page_tokens, 1))
        return pages

    def compute_knee(self) -> int:
        wb = 1.0 if self.cfg.fp8 else 2.0
        peak = self.device.gemm_flops(self.cfg.fp8)
        return int(peak * wb / (2 * self.device.hbm_bw))

    def pass_seconds(self, tokens: int, context_tokens: float = 0.0) -> float:
        """Roofline time of one pass of `tokens` new tokens (max of compute and weight reads)."""
        cfg, dev = self.cfg, self.device
        peak = dev.gemm_flops(cfg.fp8)
        flops = 2.0 * cfg.dense_params_per_token() * tokens
        flops += 4.0 * cfg.layers * cfg.q_dim * context_tokens * tokens
        bytes_ = weight_bytes(cfg) + tokens * activation_bytes_per_token(cfg) * cfg.layers * 2
        return max(flops / peak, bytes_ / dev.hbm_bw)
