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
    # a shared expert beside the routed ones, scaled per token by sigmoid(x . w_gate) (Qwen3.5 MoE); 0 = none
    shared_intermediate: int = 0
    max_position: int = 40_960
    init_std: float = 0.02
    # sparse autoencoder on the residual stream after the last loaded layer
    # (a model with one serves AI.SAE_FEATURES only); 0 = none
    sae_features: int = 0
    sae_keep: int = 0
    # hybrid decoders: per-layer kinds ("gdn" = Gated DeltaNet (Qwen3.5),
    # "conv" = gated short convolution (LFM2), "attn" = full attention);
    # empty = every layer is attention
    layer_kinds: tuple = ()
    arch: str = "qwen3"              # checkpoint naming: "qwen3", "qwen3_5" or "lfm2"
    attn_output_gate: bool = False   # attention output * sigmoid(gate), gate from q_proj
    partial_rotary: float = 1.0      # fraction of head_dim that RoPE rotates
    norm_offset: bool = False        # RMSNorm scales by (1 + w) (zero-centered weights)
    gdn_key_heads: int = 0
    gdn_value_heads: int = 0
    gdn_key_dim: int = 0
    gdn_value_dim: int = 0
    conv_width: int = 0
    # what the model answers with: "generative" (LM head), "reranker" (yes / no
    # logits of a Qwen3 reranker prompt, AI.SCORE only) or "decision" (an
    # option-scoring head over the backbone's rows, no text output)
    mlp_fp4: bool = False            # MLP projections in NVFP4 (E2M1 + UE4M3 16-value blocks)
    role: str = "generative"
    prompt_layout: str = "ai-if"     # "ai-if", "decision2-noul" or "mammoth"
    decision_head_dim: int = 0
    # how a decision model answers: "" = its own option-scoring head; "slot_lm" = the LM
    # head's logits of the option letters at the prompt's last row
    readout: str = ""
    # "causal"; or "document_isolated": the full-attention layers read the system turn and the
    # document as one block, both ways, and each question reads that block and itself, whole
    # (recurrent layers stay causal), so a document's KV serves its own questions only
    attention_mask: str = "causal"
    turn_prefix: str | None = None   # the chat text before every prompt (None: the role's default)
    turn_suffix: str | None = None   # the chat text after every question (None: the role's default)
    # set attention (LFM3 / d1, attention_mask="set"): a pass is a document and up to
    # `set_size` questions, recomputed per pass with no KV kept
    set_size: int = 0
    sliding_window: int = 0          # "swa" layers: each token reads the last `sliding_window` tokens
    rotary_pairs: float = 1.0        # full-attention layers rotate this share of the frequency pairs
    answer_temperature: float = 1.0  # divides an option / yes-no margin before the softmax / sigmoid
    read_span_tokens: int = 0        # the longest span a pointer read returns
    read_found: tuple = ()           # a pointer read's (raw, calibrated) P(found) knots
    answer_spellings: tuple = ()     # (true spellings, false spellings) read at a yes / no slot
    # vision tower (Qwen3.5): a ViT over 16-pixel patches (2 frames per patch for a still image),
    # 2x2 patches merged into one LM token; 0 layers = text only. The LM reads image tokens with
    # interleaved multimodal RoPE over (time, height, width) position streams.
    vision_depth: int = 0
    vision_hidden: int = 0
    vision_heads: int = 0
    vision_intermediate: int = 0
    vision_patch: int = 16
    vision_merge: int = 2
    vision_temporal: int = 2
    vision_pos_embeddings: int = 2304
    mrope_sections: tuple = (11, 11, 10)   # rotary frequency pairs per (t, h, w) stream, interleaved
    vision_start_id: int = 248_053
    vision_end_id: int = 248_054
    # Gemma 4 layers (DiffusionGemma): "attn" layers are the global ones, with their own head
    # geometry, rotary base and rotated share; "swa" layers slide over `sliding_window` tokens
    full_kv_heads: int = 0
    full_head_dim: int = 0
    full_rope_theta: float = 0.0
    full_rotary_pairs: float = 1.0
    k_eq_v: bool = False             # global layers: the values are the key projection (before k_norm)
    attn_scale: float = 0.0          # softmax scale (0: 1 / sqrt(head_dim))
    hidden_act: str = "silu"         # "silu" (SwiGLU) or "gelu_tanh" (GeGLU)
    embed_scale: float = 1.0         # embeddings are multiplied by this (Gemma: sqrt(hidden))
    final_softcap: float = 0.0       # logits -> c * tanh(logits / c) when > 0
    canvas_tokens: int = 0           # diffusion canvas rows after each question (0: none)
    canvas_seed: int = 0
    # a classification's answer canvas: rows read each other both ways; row 0 a random id per
    # document and draw, row 1 the turn close, the rest padding; row 0 holds the answer
    canvas_answer_rows: int = 0
    canvas_turn_close: int = 106
    canvas_pad: int = 0

    @property
    def bidirectional(self) -> bool:
        return self.attention_mask == "document_isolated"

    @property
    def decision_head(self) -> bool:
        """A separate option-scoring head (Decision 2.0), not the LM head's letter logits."""
        return self.role == "decision" and self.readout != "slot_lm"

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
    def is_hybrid(self) -> bool:
        """Layers besides plain attention (Gated DeltaNet, short convolutions; Gemma 4's sliding
        layers are attention with a window and do not count)."""
        return not self.gemma4 and any(k != "attn" for k in self.layer_kinds)

    @property
    def conv_layers(self) -> list:
        return [i for i in range(self.layers) if self.kind(i) == "conv"]

    def kind(self, i: int) -> str:
        return self.layer_kinds[i] if self.layer_kinds else "attn"

    @property
    def attn_layers(self) -> list:
        """Indices of the layers with a KV cache."""
        return [i for i in range(self.layers) if self.kind(i) in ("attn", "swa")]

    @property
    def gemma4(self) -> bool:
        return self.arch == "gemma4"

    def attn_geometry(self, i: int) -> tuple:
        """(KV heads, head_dim) of layer i's KV cache: Gemma 4's global layers have their own."""
        if self.gemma4 and self.kind(i) == "attn":
            return self.full_kv_heads, self.full_head_dim
        return self.num_kv_heads, self.head_dim

    @property
    def kv_dims(self) -> list:
        """KV elements per token of each attention layer (K or V alone)."""
        return [h * d for h, d in (self.attn_geometry(i) for i in self.attn_layers)]

    @property
    def has_vision(self) -> bool:
        return self.vision_depth > 0

    @property
    def set_attention(self) -> bool:
        return self.attention_mask == "set"

    @property
    def gdn_layers(self) -> list:
        return [i for i in range(self.layers) if self.kind(i) == "gdn"]

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_heads * self.gdn_key_dim + self.gdn_value_heads * self.gdn_value_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

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
        if self.gemma4:
            return 2 * sum(self.kv_dims) * 2
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
# the flagship layer sequence at the smallest size: fp8 MX GEMMs, the fused QKV epilogue and
# the tcgen05 attention (4 q heads per KV head, as Qwen3-4B / 8B / 32B)
QWEN3_GPU_TINY_GQA4 = DecoderConfig(name="qwen3-gpu-tiny-gqa4", layers=2, hidden=1024, num_q_heads=8,
                                    num_kv_heads=2, head_dim=128, intermediate=1024)
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

# Qwen3.5 hybrid: three Gated DeltaNet layers per gated full-attention layer
# (the reference spec quail/specs/data/models/qwen3.5-4b-bf16.toml)
_Q35_KINDS = ("gdn", "gdn", "gdn", "attn")
QWEN35_4B = DecoderConfig(name="qwen3.5-4b", layers=32, hidden=2560, num_q_heads=16, num_kv_heads=4,
                          head_dim=256, intermediate=9216, vocab=248_320, rope_theta=10_000_000.0,
                          tied_head=True, weight_dtype="bf16", layer_kinds=_Q35_KINDS * 8,
                          attn_output_gate=True, partial_rotary=0.25, norm_offset=True, arch="qwen3_5",
                          gdn_key_heads=16,
                          gdn_value_heads=32, gdn_key_dim=128, gdn_value_dim=128, conv_width=4,
                          max_position=262_144)
# Qwen3.5's vision tower (Hugging Face Qwen3_5VisionConfig defaults: 27 layers, width 1152, 16 heads)
_Q35_VISION = dict(vision_depth=27, vision_hidden=1152, vision_heads=16, vision_intermediate=4304)
QWEN35_VL_4B = QWEN35_4B.with_(name="qwen3.5-4b-vl", **_Q35_VISION)
QWEN35_TINY = QWEN35_4B.with_(name="qwen3.5-tiny", layers=4, hidden=256, num_q_heads=4, num_kv_heads=2,
                              head_dim=64, intermediate=512, vocab=151_936, gdn_key_heads=2, gdn_value_heads=4,
                              gdn_key_dim=32, gdn_value_dim=32, layer_kinds=_Q35_KINDS, max_position=40_960)
# the smallest hybrid the GPU kernels take: head_dim 256 attention (2 q heads per KV
# head), 128-dim Gated DeltaNet heads (2 key, 4 value heads)
QWEN35_GPU_TINY = QWEN35_4B.with_(name="qwen3.5-gpu-tiny", layers=4, hidden=1024, num_q_heads=4, num_kv_heads=2,
                                  intermediate=1024, vocab=4096, gdn_key_heads=2, gdn_value_heads=4,
                                  layer_kinds=_Q35_KINDS, max_position=8192)
# LFM2: gated short convolutions (width 3) and GQA attention (head_dim 64)
# (the reference spec quail/specs/data/models/lfm2-2.6b-bf16.toml)
_LFM2_KINDS = tuple("conv conv attn conv conv attn conv conv conv attn conv conv conv attn conv conv conv attn "
                    "conv conv conv attn conv conv attn conv conv attn conv conv".split())
LFM2_2_6B = DecoderConfig(name="lfm2-2.6b", layers=30, hidden=2048, num_q_heads=32, num_kv_heads=8, head_dim=64,
                          intermediate=10752, vocab=65_536, tied_head=True, weight_dtype="bf16", arch="lfm2",
                          layer_kinds=_LFM2_KINDS, conv_width=3, rms_eps=1e-5, max_position=128_000)
LFM2_TINY = LFM2_2_6B.with_(name="lfm2-tiny", layers=3, hidden=256, num_q_heads=4, num_kv_heads=2,
                            intermediate=512, vocab=151_936, layer_kinds=("conv", "conv", "attn"),
                            max_position=40_960)
LFM2_GPU_TINY = LFM2_2_6B.with_(name="lfm2-gpu-tiny", layers=3, hidden=1024, num_q_heads=16, num_kv_heads=4,
                                intermediate=1024, vocab=4096, layer_kinds=("conv", "attn", "conv"),
                                max_position=8192)
# further reference specs on the architectures above (quail/specs/data/models/*.toml)
QWEN3_06B = DecoderConfig(name="qwen3-0.6b", layers=28, hidden=1024, num_q_heads=16, num_kv_heads=8, head_dim=128,
                          intermediate=3072, tied_head=True, weight_dtype="bf16")
QWEN3_RERANKER_06B = QWEN3_06B.with_(name="qwen3-reranker-0.6b", vocab=151_669, role="reranker")
QWEN3_RERANKER_4B = QWEN3_4B.with_(name="qwen3-reranker-4b", vocab=151_669, weight_dtype="bf16", role="reranker")
DECISION2_06B = QWEN3_06B.with_(name="decision-2.0-kai-0.6b", role="decision", prompt_layout="decision2-noul",
                                decision_head_dim=256)
# small stand-ins of the two roles for the tests (CPU and GPU kernel shapes)
DECISION_TINY = QWEN3_TINY.with_(name="decision-tiny", role="decision", prompt_layout="decision2-noul",
                                 decision_head_dim=32, weight_dtype="bf16")
DECISION_GPU_TINY = QWEN3_GPU_TINY.with_(name="decision-gpu-tiny", role="decision", prompt_layout="decision2-noul",
                                         decision_head_dim=128, weight_dtype="bf16")
RERANKER_TINY = QWEN3_TINY.with_(name="reranker-tiny", role="reranker", weight_dtype="bf16")
RERANKER_GPU_TINY = QWEN3_GPU_TINY.with_(name="reranker-gpu-tiny", role="reranker", weight_dtype="bf16")
QWEN35_9B = QWEN35_4B.with_(name="qwen3.5-9b", hidden=4096, intermediate=12288, tied_head=False)
QWEN35_4B_FP8 = QWEN35_4B.with_(name="qwen3.5-4b-fp8", weight_dtype="fp8")
QWEN35_GPU_TINY_FP8 = QWEN35_GPU_TINY.with_(name="qwen3.5-gpu-tiny-fp8", weight_dtype="fp8")
QWEN35_27B = QWEN35_4B.with_(name="qwen3.5-27b", layers=64, hidden=5120, num_q_heads=24, num_kv_heads=4,
                             intermediate=17408, tied_head=False, gdn_value_heads=48, layer_kinds=_Q35_KINDS * 16)
QWEN35_27B_FP8 = QWEN35_27B.with_(name="qwen3.5-27b-fp8", weight_dtype="fp8")
QWEN38_27B_FP8 = QWEN35_27B_FP8.with_(name="qwen3.8-27b-fp8")
# the NVFP4 checkpoint: attention in fp8, MLP in NVFP4 (the reference spec's mlp_weight_precision = "fp4")
QWEN38_27B_NVFP4 = QWEN38_27B_FP8.with_(name="qwen3.8-27b-nvfp4", mlp_fp4=True)
QWEN35_GPU_TINY_NVFP4 = QWEN35_GPU_TINY.with_(name="qwen3.5-gpu-tiny-nvfp4", weight_dtype="fp8", mlp_fp4=True)
# Qwen3.6-35B-A3B: the Qwen3.5 hybrid with 256 routed experts (top 8) and a shared expert
# (the reference spec quail/specs/data/models/qwen3.6-35b-a3b-fp8.toml; HF Qwen3_5MoeSparseMoeBlock)
QWEN36_35B_A3B = QWEN35_4B.with_(name="qwen3.6-35b-a3b-fp8", layers=40, hidden=2048, num_q_heads=16,
                                 num_kv_heads=2, intermediate=512, tied_head=False, weight_dtype="fp8",
                                 num_experts=256, top_k=8, moe_intermediate=512, shared_intermediate=512,
                                 layer_kinds=_Q35_KINDS * 10)
QWEN36_MOE_GPU_TINY = QWEN36_35B_A3B.with_(name="qwen3.6-moe-gpu-tiny", layers=4, hidden=1024, num_q_heads=4,
                                           num_kv_heads=2, vocab=4096, num_experts=16, top_k=4,
                                           gdn_key_heads=2, gdn_value_heads=4, layer_kinds=_Q35_KINDS,
                                           max_position=8192, moe_intermediate=256, shared_intermediate=256)
QWEN36_MOE_TINY = QWEN36_MOE_GPU_TINY.with_(name="qwen3.6-moe-tiny", hidden=256, head_dim=64, num_experts=8,
                                            top_k=2, moe_intermediate=128, shared_intermediate=128,
                                            gdn_key_dim=32, gdn_value_dim=32, weight_dtype="bf16")
QWEN35_2B_SAE = QWEN35_4B.with_(name="qwen3.5-2b-sae", layers=12, hidden=2048, num_q_heads=8, num_kv_heads=2,
                                intermediate=6144, gdn_value_heads=16, layer_kinds=_Q35_KINDS * 3,
                                sae_features=32768, sae_keep=100)
QWEN35_SAE_TINY = QWEN35_TINY.with_(name="qwen3.5-sae-tiny", sae_features=256, sae_keep=8)

# Base Labs' mammoth-1 and elephant-1: full fine-tunes of Qwen3.5 27B / 9B (bf16, own output
# head) that read the document block both ways and answer with the LM head's option-letter
# logits (the reference specs quail/specs/data/models/mammoth-1-bf16.toml, elephant-1-bf16.toml)
MAMMOTH_SYSTEM_TURN = ("<|im_start|>system\nApply the question to the state. Choose exactly one of the listed "
                       "options. Respond with only its uppercase letter, with no explanation or reasoning."
                       "<|im_end|>\n<|im_start|>user\n")
_ISOLATED = dict(role="decision", prompt_layout="mammoth", readout="slot_lm", attention_mask="document_isolated",
                 turn_prefix=MAMMOTH_SYSTEM_TURN)
MAMMOTH_1 = QWEN35_27B.with_(name="mammoth-1-bf16", **_ISOLATED)
ELEPHANT_1 = QWEN35_9B.with_(name="elephant-1-bf16", **_ISOLATED)
# stand-ins for the tests: the hybrid at the CPU and GPU kernel sizes, and a dense decoder with
# the same mask (whose answers a plain full-sequence forward can check)
MAMMOTH_TINY = QWEN35_TINY.with_(name="mammoth-tiny", **_ISOLATED)
MAMMOTH_GPU_TINY = QWEN35_GPU_TINY.with_(name="mammoth-gpu-tiny", **_ISOLATED)
ISOLATED_DENSE_TINY = QWEN3_TINY.with_(name="isolated-dense-tiny", **_ISOLATED)

# LiquidAI d1-2B (LFM3): short convolutions (7 taps) between attention layers that alternate
# full attention (half the frequency pairs rotated) and a 256-token sliding window; sandwich
# norms; a sigmoid gate per attention head; set attention (the reference spec
# quail/specs/data/models/d1-2b-bf16.toml)
_D1_KINDS = ("conv", "conv") + ("attn", "conv", "swa", "conv") * 5 + ("attn", "conv")
D1_TURN_PREFIX = "<|startoftext|><|im_start|>user\n"
D1_TURN_SUFFIX = "<|im_end|>\n<|im_start|>assistant\n<think></think>"
D1_2B = DecoderConfig(name="d1-2b", layers=24, hidden=2048, num_q_heads=16, num_kv_heads=4, head_dim=128,
                      intermediate=7680, vocab=128_000, tied_head=True, weight_dtype="bf16", arch="lfm3",
                      layer_kinds=_D1_KINDS, conv_width=7, rms_eps=1e-5, max_position=128_000,
                      attention_mask="set", set_size=16, sliding_window=256, rotary_pairs=0.5,
                      answer_temperature=1.337398453966105, read_span_tokens=512, prompt_layout="d1",
                      turn_prefix=D1_TURN_PREFIX, turn_suffix=D1_TURN_SUFFIX,
                      answer_spellings=(("yes", "Yes", "YES"), ("no", "No", "NO")))
D1_TINY = D1_2B.with_(name="d1-tiny", layers=4, hidden=256, num_q_heads=4, num_kv_heads=2, head_dim=64,
                      intermediate=512, vocab=151_936, layer_kinds=("conv", "attn", "conv", "swa"), set_size=4,
                      sliding_window=16, read_span_tokens=32, max_position=40_960)
D1_GPU_TINY = D1_2B.with_(name="d1-gpu-tiny", layers=4, hidden=1024, num_q_heads=8, num_kv_heads=2, head_dim=128,
                          intermediate=1024, vocab=4096, layer_kinds=("conv", "attn", "conv", "swa"), set_size=4,
                          sliding_window=64, read_span_tokens=64, max_position=8192)

# the smallest hybrids with a vision tower (the CPU model, the GPU kernels' shapes)
QWEN35_VL_TINY = QWEN35_TINY.with_(name="qwen3.5-vl-tiny", vision_depth=2, vision_hidden=96, vision_heads=4,
                                   vision_intermediate=192, vision_pos_embeddings=64, mrope_sections=(3, 3, 2),
                                   vision_start_id=151_933, vision_end_id=151_934)
QWEN35_VL_GPU_TINY = QWEN35_GPU_TINY.with_(name="qwen3.5-vl-gpu-tiny", vision_depth=2, vision_hidden=256,
                                           vision_heads=4, vision_intermediate=512, vision_pos_embeddings=256,
                                           vision_start_id=4093, vision_end_id=4094)

CONFIGS = {c.name: c for c in (QWEN3_4B, QWEN3_8B, QWEN3_32B, QWEN3_30B_A3B, QWEN3_TINY, QWEN3_GPU_TINY,
                               QWEN3_GPU_TINY_GQA4,
                               QWEN3_MOE_GPU_TINY, QWEN3_4B_SAE, QWEN3_SAE_TINY, QWEN3_GPU_SAE_TINY,
                               QWEN35_4B, QWEN35_TINY, QWEN35_GPU_TINY, LFM2_2_6B, LFM2_TINY, LFM2_GPU_TINY,
                               QWEN3_06B, QWEN3_RERANKER_06B, QWEN3_RERANKER_4B, DECISION2_06B, QWEN35_9B, QWEN35_27B,
                               QWEN35_2B_SAE, QWEN35_SAE_TINY, DECISION_TINY, DECISION_GPU_TINY, RERANKER_TINY,
                               QWEN35_4B_FP8, QWEN35_GPU_TINY_FP8, RERANKER_GPU_TINY, QWEN35_27B_FP8, QWEN38_27B_FP8,
                               QWEN36_35B_A3B, QWEN36_MOE_GPU_TINY, QWEN36_MOE_TINY, QWEN38_27B_NVFP4,
                               QWEN35_GPU_TINY_NVFP4, MAMMOTH_1, ELEPHANT_1, MAMMOTH_TINY, MAMMOTH_GPU_TINY,
                               ISOLATED_DENSE_TINY, D1_2B, D1_TINY, D1_GPU_TINY, QWEN35_VL_4B, QWEN35_VL_TINY,
                               QWEN35_VL_GPU_TINY)}

# DiffusionGemma (Gemma 4 MoE backbone, one-step canvas readout): 25 sliding-window layers over
# 1024 tokens with 256-wide heads, every sixth layer global with 512-wide heads and two KV heads
# whose values are the keys' projection; a dense GeGLU MLP beside 128 experts (top 8)
_DG_KINDS = tuple("attn" if (i + 1) % 6 == 0 else "swa" for i in range(30))
DIFFUSION_GEMMA_26B = DecoderConfig(
    name="diffusion-gemma-26b-a4b-fp8", layers=30, hidden=2816, num_q_heads=16, num_kv_heads=8, head_dim=256,
    intermediate=2112, vocab=262_144, rope_theta=10_000.0, rms_eps=1e-6, tied_head=True, weight_dtype="fp8",
    num_experts=128, top_k=8, moe_intermediate=704, max_position=131_072, layer_kinds=_DG_KINDS, arch="gemma4",
    sliding_window=1024, full_kv_heads=2, full_head_dim=512, full_rope_theta=1_000_000.0, full_rotary_pairs=0.25,
    k_eq_v=True, attn_scale=1.0, hidden_act="gelu_tanh", embed_scale=2816 ** 0.5, final_softcap=30.0,
    canvas_tokens=1, canvas_seed=20_260_514, prompt_layout="letters", canvas_answer_rows=16,
    turn_prefix="<bos><|turn>system\nYou are an expert at text analysis<turn|>\n<|turn>user\n",
    turn_suffix="<turn|>\n<|turn>model\n<|channel>thought\n<channel|>")
# the CPU model (fp32; checked against Hugging Face's Gemma4TextModel) and the GPU kernels' shapes
DIFFUSION_GEMMA_TINY = DIFFUSION_GEMMA_26B.with_(
    name="diffusion-gemma-tiny", layers=4, hidden=256, num_q_heads=4, num_kv_heads=2, head_dim=64,
    intermediate=256, vocab=151_936, num_experts=8, top_k=2, moe_intermediate=64, max_position=40_960,
    layer_kinds=("swa", "attn", "swa", "attn"), sliding_window=16, full_kv_heads=1, full_head_dim=128,
    embed_scale=256 ** 0.5, weight_dtype="bf16")
DIFFUSION_GEMMA_GPU_TINY = DIFFUSION_GEMMA_26B.with_(
    name="diffusion-gemma-gpu-tiny", layers=4, hidden=1024, num_q_heads=8, num_kv_heads=4, head_dim=256,
    intermediate=512, vocab=4096, num_experts=16, top_k=4, moe_intermediate=256, max_position=8192,
    layer_kinds=("swa", "attn", "swa", "attn"), sliding_window=64, full_kv_heads=1, full_head_dim=512,
    embed_scale=1024 ** 0.5, weight_dtype="bf16")
CONFIGS.update({c.name: c for c in (DIFFUSION_GEMMA_26B, DIFFUSION_GEMMA_TINY, DIFFUSION_GEMMA_GPU_TINY)})

# model spec names (as in EngineConfig.model) -> decoder config
MODEL_CONFIGS = {
    "qwen3-4b-fp8": QWEN3_4B,
    "qwen3-4b-bf16": QWEN3_4B.with_(weight_dtype="bf16", name="qwen3-4b-bf16"),
    "qwen3-8b-bf16": QWEN3_8B,
    "qwen3-32b-fp8": QWEN3_32B,
    "qwen3-30b-a3b-fp8": QWEN3_30B_A3B,
    "qwen3-tiny": QWEN3_TINY,
    "qwen3-gpu-tiny": QWEN3_GPU_TINY,
    "qwen3-gpu-tiny-gqa4": QWEN3_GPU_TINY_GQA4,
    "qwen3-moe-gpu-tiny": QWEN3_MOE_GPU_TINY,
    "qwen3-4b-sae-bf16": QWEN3_4B_SAE,
    "qwen3-sae-tiny": QWEN3_SAE_TINY,
    "qwen3-gpu-sae-tiny": QWEN3_GPU_SAE_TINY,
    "qwen3.5-4b-bf16": QWEN35_4B,
    "qwen3.5-tiny": QWEN35_TINY,
    "qwen3.5-gpu-tiny": QWEN35_GPU_TINY,
    "lfm2-2.6b-bf16": LFM2_2_6B,
    "lfm2-tiny": LFM2_TINY,
    "lfm2-gpu-tiny": LFM2_GPU_TINY,
    "qwen3-reranker-0.6b-bf16": QWEN3_RERANKER_06B,
    "qwen3-reranker-4b-bf16": QWEN3_RERANKER_4B,
    "decision-2.0-kai-0.6b-bf16": DECISION2_06B,
    "qwen3.5-9b-bf16": QWEN35_9B,
    "qwen3.5-27b-bf16": QWEN35_27B,
    "qwen3.5-2b-sae-bf16": QWEN35_2B_SAE,
    "qwen3.5-sae-tiny": QWEN35_SAE_TINY,
    "decision-tiny": DECISION_TINY,
    "decision-gpu-tiny": DECISION_GPU_TINY,
    "reranker-tiny": RERANKER_TINY,
    "reranker-gpu-tiny": RERANKER_GPU_TINY,
    "qwen3.5-4b-fp8": QWEN35_4B_FP8,
    "qwen3.5-gpu-tiny-fp8": QWEN35_GPU_TINY_FP8,
    "qwen3.5-27b-fp8": QWEN35_27B_FP8,
    "qwen3.8-27b-fp8": QWEN38_27B_FP8,
    "qwen3.8-27b-nvfp4": QWEN38_27B_NVFP4,
    "qwen3.5-gpu-tiny-nvfp4": QWEN35_GPU_TINY_NVFP4,
    "qwen3.6-35b-a3b-fp8": QWEN36_35B_A3B,
    "qwen3.6-moe-gpu-tiny": QWEN36_MOE_GPU_TINY,
    "qwen3.6-moe-tiny": QWEN36_MOE_TINY,
    "mammoth-1-bf16": MAMMOTH_1,
    "elephant-1-bf16": ELEPHANT_1,
    "mammoth-tiny": MAMMOTH_TINY,
    "mammoth-gpu-tiny": MAMMOTH_GPU_TINY,
    "isolated-dense-tiny": ISOLATED_DENSE_TINY,
    "d1-2b-bf16": D1_2B,
    "d1-tiny": D1_TINY,
    "qwen3.5-4b-vl-bf16": QWEN35_VL_4B,
    "qwen3.5-vl-tiny": QWEN35_VL_TINY,
    "qwen3.5-vl-gpu-tiny": QWEN35_VL_GPU_TINY,
    "d1-gpu-tiny": D1_GPU_TINY,
    "diffusion-gemma-26b-a4b-fp8": DIFFUSION_GEMMA_26B,
    "diffusion-gemma-tiny": DIFFUSION_GEMMA_TINY,
    "diffusion-gemma-gpu-tiny": DIFFUSION_GEMMA_GPU_TINY,
}
