"""Tensor-parallel Qwen3 (dense) on the fused AG->GEMM / GEMM->RS kernels.

Reference: the reference never splits weights (a model larger than one GPU
is refused, crates/quail-planner/src/validation.rs:408-420); this is the
engine's own TP for models like Qwen3-32B, one process per GPU.

Sharding (tp ranks): q heads and kv heads by head, gate/up by intermediate
column (interleaved per shard for the SwiGLU epilogue), o_proj and down by
input column. The residual stream is sharded by tokens: a chunk of T tokens
is padded to M = tp x rpr (rpr a multiple of 128) and rank r owns rows
[r*rpr, (r+1)*rpr). Per layer:

  rs_reduce_norm  (own rows)  -> e4m3 shard in the symmetric A buffer, flag up
  tp_ag_gemm      QKV         -> all M rows, local heads (gathers peers' rows)
  qk-norm/RoPE/KV write, tcgen05 attention on local heads (all M rows)
  tp_gemm_rs      o_proj      -> each owner's receive slot
  rs_reduce_norm  sum + residual + post-attention norm -> A buffer, flag up
  tp_ag_gemm      gate_up + SwiGLU -> e4m3 (all M rows, local columns)
  tp_gemm_rs      down        -> receive slots
  (next layer's rs_reduce_norm sums them)

Symmetric buffers (peer-addressable) come from torch.distributed's
symmetric memory (allocation + handle exchange only); every byte that moves
between GPUs is moved by the kernels above. Readout rows are summed across
ranks with one small NCCL all-reduce of logits.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from quail_b200.models.config import DecoderConfig
from quail_b200.ops import reference as ref


class TPState:
    """Per-rank symmetric buffers, peer pointers and monotonic epochs."""

    def __init__(self, cfg: DecoderConfig, group, max_tokens: int, device):
        import torch.distributed._symmetric_memory as symm
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        H = cfg.hidden
        inter_local = cfg.intermediate // self.tp
        self.rpr_max = -(-max_tokens // (self.tp * 128)) * 128
        self.M_max = self.rpr_max * self.tp
        K_max = max(H, inter_local, cfg.q_dim // self.tp)
        a_bytes = self.M_max * K_max
        sf_bytes = (self.M_max // 128) * (K_max // 128) * 512
        slot_bytes = self.tp * self.rpr_max * H * 2
        # one symmetric uint8 arena: [A | SF | slots | flags(64 ints) | counters(64 ints)]
        self.off_a, self.off_sf = 0, a_bytes
        self.off_slot = self.off_sf + sf_bytes
        self.off_flag = self.off_slot + slot_bytes
        self.off_ctr = self.off_flag + 256
        total = self.off_ctr + 256
        self.buf = symm.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, group.group_name if hasattr(group, "group_name") else
                                      dist.group.WORLD.group_name)
        self.peers = [int(p) for p in self.handle.buffer_ptrs]
        self.tile_ready = torch.zeros(self.M_max // 128, dtype=torch.int32, device=device)
        self.done_ctr = torch.zeros(1, dtype=torch.int32, device=device)
        self.ag_epoch = 0      # AG operations so far (flags / tile-ready words carry it)
        self.rs_tiles = 0      # tiles each source has pushed here so far (the receive counters' target)
        self.done_total = 0    # CTAs of every reduce-norm launch so far (the done counter's target)
        torch.cuda.synchronize(device)
        dist.barrier(group)

    # views of this rank's arena
    def a_sym(self, M, K):
        return self.buf[self.off_a:self.off_a + M * K].view(torch.float8_e4m3fn).view(M, K)

    def sf_sym(self, M, K):
        return self.buf[self.off_sf:self.off_sf + (M // 128) * (K // 128) * 512]

    def slots(self, rpr, H):
        return self.buf[self.off_slot:self.off_slot + self.tp * rpr * H * 2].view(torch.bfloat16).view(self.tp, rpr, H)

    def flag(self):
        return self.buf[self.off_flag:self.off_flag + 4].view(torch.int32)

    def counters(self):
        return self.buf[self.off_ctr:self.off_ctr + 4 * self.tp].view(torch.int32)

    def peer(self, off: int) -> list[int]:
        return [p + off for p in self.peers]


def _rng(seed, *key):
    g = torch.Generator(device="cuda")
    g.manual_seed(hash((seed,) + key) & ((1 << 62) - 1))
    return g


class TPQwen3:
    """One rank's shard of a Qwen3 dense model and its forward over a packed chunk."""

    def __init__(self, cfg: DecoderConfig, group, *, seed: int = 0, max_tokens: int = 16384, answer_ids=(0, 1),
                 full_weights: dict | None = None, comm: str = "fused"):
        from quail_b200.ops.quant import interleave_gate_up_mx, quantize_weight_mx
        assert cfg.fp8 and cfg.head_dim == 128
        assert comm in ("fused", "nccl")
        # "nccl": the baseline the fused kernels are measured against: NCCL
        # all-gather / reduce-scatter around the same MX GEMMs
        self.comm = comm
        from quail_b200.utils.op_timer import OpTimer
        self.timer = OpTimer()
        self.cfg = cfg
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.st = TPState(cfg, group, max_tokens, self.device)
        tp, r = self.st.tp, self.st.rank
        assert cfg.num_q_heads % tp == 0 and cfg.num_kv_heads % tp == 0 and cfg.intermediate % (tp * 128) == 0
        self.qh, self.kh, self.inter = cfg.num_q_heads // tp, cfg.num_kv_heads // tp, cfg.intermediate // tp
        H, D = cfg.hidden, 128
        dev = self.device
        bf = torch.bfloat16

        def full(name, shape, layer):
            if full_weights is not None:
                from quail_b200.models.weights import dequantized
                return dequantized(full_weights, f"model.layers.{layer}.{name}").to(dev, torch.float32)
            g = _rng(seed, layer, name)
            return torch.randn(*shape, generator=g, device=dev) * cfg.init_std

        self.layers = []
        for i in range(cfg.layers):
            q = full("self_attn.q_proj", (cfg.q_dim, H), i)
            k = full("self_attn.k_proj", (cfg.kv_dim, H), i)
            v = full("self_attn.v_proj", (cfg.kv_dim, H), i)
            o = full("self_attn.o_proj", (H, cfg.q_dim), i)
            gp = full("mlp.gate_proj", (cfg.intermediate, H), i)
            up = full("mlp.up_proj", (cfg.intermediate, H), i)
            dn = full("mlp.down_proj", (H, cfg.intermediate), i)
            qs = slice(r * self.qh * D, (r + 1) * self.qh * D)
            ks = slice(r * self.kh * D, (r + 1) * self.kh * D)
            js = slice(r * self.inter, (r + 1) * self.inter)
            L = {}
            L["wqkv"], L["sqkv"] = quantize_weight_mx(torch.cat([q[qs], k[ks], v[ks]]))
            L["wo"], L["so"] = quantize_weight_mx(o[:, qs].contiguous())
            L["wgu"], L["sgu"] = interleave_gate_up_mx(torch.cat([gp[js], up[js]]))
            L["wd"], L["sd"] = quantize_weight_mx(dn[:, js].contiguous())
            one = torch.ones(H, device=dev, dtype=bf)
            L["ln1"], L["ln2"] = one.clone(), one.clone()
            L["qn"] = torch.ones(D, device=dev, dtype=bf)
            L["kn"] = torch.ones(D, device=dev, dtype=bf)
            if full_weights is not None:
                p = f"model.layers.{i}."
                for key, name in (("ln1", "input_layernorm"), ("ln2", "post_attention_layernorm"),
                                  ("qn", "self_attn.q_norm"), ("kn", "self_attn.k_norm")):
                    L[key] = full_weights[p + name + ".weight"].to(dev, bf)
            self.layers.append(L)
            del q, k, v, o, gp, up, dn
        if full_weights is not None:
            self.embed = full_weights["model.embed_tokens.weight"].to(dev, bf).contiguous()
            self.final_norm = full_weights["model.norm.weight"].to(dev, bf)
            head = full_weights["model.embed_tokens.weight" if cfg.tied_head else "lm_head.weight"]
        else:
            g = _rng(seed, "embed")
            self.embed = (torch.randn(cfg.vocab, H, generator=g, device=dev) * cfg.init_std).to(bf)
            self.final_norm = torch.ones(H, device=dev, dtype=bf)
            head = self.embed
        self.head = head.to(dev, bf)
        self.set_answer_rows(answer_ids)
        self.cos_sin = ref.rope_cos_sin(cfg.max_position, 128, cfg.rope_theta, device=dev)
        self.scale = ref.softmax_scale(128)

    def set_answer_rows(self, ids):
        self.answer_rows = self.head[torch.as_tensor(list(ids), device=self.device).long()].contiguous()

    # ------------------------------------------------------------ collectives
    def _norm(self, h_local, w, M, rpr, tp_slots: int):
        """Sum receive slots (if any) into the residual, RMSNorm, MX-quantize into this rank's A rows."""
        from quail_b200 import ops
        st = self.st
        H = self.cfg.hidden
        if tp_slots:
            st.rs_tiles += (rpr // 128) * (-(-H // 256))
        st.ag_epoch += 1
        want = st.rs_tiles
        ops.count_launch()
        ops.native().tp_reduce_norm(st.slots(rpr, H), tp_slots, st.counters(), want, h_local, w, self.cfg.rms_eps,
                                    st.a_sym(M, H), st.sf_sym(M, H), st.rank * rpr, st.done_ctr, st.done_total,
                                    st.flag(), st.ag_epoch)
        st.done_total += -(-rpr // 8)

    def _ag(self, M, K, rpr, w, sfw, mode):
        from quail_b200 import ops
        st = self.st
        N = w.shape[0]
        if mode == 0:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
            osf = None
        else:
            out = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=self.device)
            osf = torch.empty(ops.sf_bytes(M, N // 2), dtype=torch.uint8, device=self.device)
        ops.count_launch()
        ops.native().tp_ag_gemm(st.a_sym(M, K), st.sf_sym(M, K), st.peer(st.off_a), st.peer(st.off_sf),
                                st.peer(st.off_flag), st.tile_ready, st.ag_epoch, st.rank, rpr, w, sfw, mode, out, osf)
        return out if mode == 0 else (out, osf)

    def _rs(self, a, sfa, w, sfw, rpr):
        from quail_b200 import ops
        st = self.st
        H = self.cfg.hidden
        slot_off = st.off_slot + st.rank * rpr * H * 2   # this source's slot on every rank
        ops.count_launch()
        ops.native().tp_gemm_rs(a, sfa, w, sfw, st.peer(slot_off), H,
                                [p + st.off_ctr + 4 * st.rank for p in st.peers], st.rank, rpr)

    # ------------------------------------------------------------ NCCL baseline pieces
    def _nccl_ag(self, h_local, w_norm, M, rpr):
        from quail_b200 import ops
        H = self.cfg.hidden
        x8, sf = ops.rmsnorm_quant_mx(h_local, w_norm, self.cfg.rms_eps)
        full = torch.empty(M, H, dtype=torch.uint8, device=self.device)
        sff = torch.empty(sf.numel() * self.st.tp, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(full, x8.view(torch.uint8), group=self.st.group)
        dist.all_gather_into_tensor(sff, sf, group=self.st.group)
        return full.view(torch.float8_e4m3fn), sff

    def _nccl_rs_add(self, part, h_local):
        out = torch.empty_like(h_local)
        dist.reduce_scatter_tensor(out, part, group=self.st.group)
        h_local += out

    # ------------------------------------------------------------ forward
    @torch.no_grad()
    def forward_chunk(self, chunk, arena) -> torch.Tensor:
        from quail_b200 import ops
        cfg, st = self.cfg, self.st
        T = chunk.num_tokens
        tp, r = st.tp, st.rank
        rpr = -(-T // (tp * 128)) * 128
        M = rpr * tp
        assert M <= st.M_max, "chunk larger than the TP buffers"
        H = cfg.hidden
        dev = self.device
        ids = torch.zeros(M, dtype=torch.int32, device=dev)
        ids[:T] = chunk.ids
        pos = torch.zeros(M, dtype=torch.int32, device=dev)
        pos[:T] = chunk.positions
        slots = torch.full((M,), -1, dtype=torch.int32, device=dev)
        slots[:T] = chunk.slots
        h = ops.embed_gather(ids[r * rpr:(r + 1) * rpr].contiguous(), self.embed)  # own residual rows
        fused = self.comm == "fused"
        tm = self.timer
        for li, L in enumerate(self.layers):
            kc, vc = arena.layer(li)
            if fused:
                with tm("norm_ln1"):
                    self._norm(h, L["ln1"], M, rpr, tp_slots=tp if li > 0 else 0)
                with tm("ag_gemm_qkv"):
                    qkv = self._ag(M, H, rpr, L["wqkv"], L["sqkv"], mode=0)
            else:
                with tm("nccl_ag_ln1"):
                    xa, sa = self._nccl_ag(h, L["ln1"], M, rpr)
                with tm("gemm_qkv"):
                    qkv = ops.gemm_mx(xa, sa, L["wqkv"], L["sqkv"])
            with tm("rope_kv"):
                q = ops.qk_norm_rope_kv(qkv, pos, L["qn"], L["kn"], self.cos_sin, slots, kc, vc, self.qh, self.kh,
                                        cfg.rms_eps)
            with tm("attention"):
                o8 = torch.zeros(M, self.qh * 128, dtype=torch.float8_e4m3fn, device=dev)  # padding rows stay 0
                os_ = torch.zeros(ops.sf_bytes(M, self.qh * 128), dtype=torch.uint8, device=dev)
                ops.chunk_attention(q, kc, vc, chunk, self.scale, mx=True, tc=True, out=o8, out_scale=os_)
            if fused:
                with tm("gemm_rs_o"):
                    self._rs(o8, os_, L["wo"], L["so"], rpr)
                with tm("norm_ln2"):
                    self._norm(h, L["ln2"], M, rpr, tp_slots=tp)
                with tm("ag_gemm_gate_up"):
                    a8, as_ = self._ag(M, H, rpr, L["wgu"], L["sgu"], mode=1)
                with tm("gemm_rs_down"):
                    self._rs(a8, as_, L["wd"], L["sd"], rpr)
            else:
                with tm("gemm_o"):
                    part = ops.gemm_mx(o8, os_, L["wo"], L["so"])
                with tm("nccl_rs_o"):
                    self._nccl_rs_add(part, h)
                with tm("nccl_ag_ln2"):
                    xa, sa = self._nccl_ag(h, L["ln2"], M, rpr)
                with tm("gemm_gate_up"):
                    a8, as_ = ops.gemm_mx(xa, sa, L["wgu"], L["sgu"], epi=ops.EPI_SWIGLU_FP8)
                with tm("gemm_down"):
                    part = ops.gemm_mx(a8, as_, L["wd"], L["sd"])
                with tm("nccl_rs_down"):
                    self._nccl_rs_add(part, h)
        if fused:
            # last down-projection: sum it into the residual (the final norm runs in the readout)
            self._norm(h, self.final_norm, M, rpr, tp_slots=tp)
        rows = chunk.final_rows.long()
        mine = (rows >= r * rpr) & (rows < (r + 1) * rpr)
        local = torch.where(mine, rows - r * rpr, torch.zeros_like(rows)).int()
        if getattr(chunk, "full_readout", False):
            # AI.CLASSIFY / MAP rows: answer rows plus the full-vocabulary argmax and log-sum-exp
            # of this rank's rows (the head is replicated); the other ranks' rows are zero
            normed = torch.empty(rows.numel(), H, dtype=torch.bfloat16, device=dev)
            ans = ops.final_norm_readout(h, local, self.final_norm, cfg.rms_eps, self.answer_rows, normed=normed)
            logits = ops.head_readout(normed, self.head, ans, getattr(chunk, "topk", False))
        else:
            logits = ops.final_norm_readout(h, local, self.final_norm, cfg.rms_eps, self.answer_rows)
        logits = logits * mine[:, None].float()
        # each row is owned by one rank: the sum hands every rank every row's readout
        dist.all_reduce(logits, group=st.group)
        return logits

    def check_errors(self) -> int:
        from quail_b200 import ops
        return ops.read_and_clear_error(self.device.index)
