"""Expert-parallel MoE layer on the fused dispatch/combine kernels.

W ranks (one process per GPU) each own E / W experts and run attention on
their own tokens (data-parallel attention). Per MoE layer, every rank runs,
in stream order (kernels in `quail_b200/csrc/moe.cu`):

  router GEMM (bf16 tcgen05) -> moe_route -> moe_plan (count exchange with
  every peer) -> moe_sort -> moe_gate_up (dispatch warps push token rows to
  the experts' owners while the grouped GEMM consumes arrived experts) ->
  moe_down (epilogue pushes weighted rows back to each token's home) ->
  moe_combine (sum of the K rows + residual, next layer's RMSNorm as MX).

With W = 1 the same kernels run on local buffers: the dispatch is the
permutation into expert-contiguous rows, the combine the weighted un-permute.
For W > 1 the receive buffers, combine buffers, counters and flags live in
one symmetric arena (torch.distributed symmetric memory gives the peer
pointers; every byte between GPUs is moved by the kernels).

Reference: MoE runs on one GPU only, through vLLM's fused Triton experts
(quail/backends/quail/executor/moe.py:12-87; FP8Experts asserts
tp == ep == dp == 1); expert parallelism is this engine's own.
"""

from __future__ import annotations

import torch

from quail_b200.models.config import DecoderConfig


def _align(n: int, a: int) -> int:
    return -(-n // a) * a


class EPState:
    """Buffers, peer pointers and monotonic counters of the MoE layers of one rank."""

    def __init__(self, cfg: DecoderConfig, max_tokens: int, device, group=None):
        import torch.distributed as dist
        from quail_b200 import ops
        assert cfg.is_moe and cfg.fp8
        if cfg.hidden not in (1024, 2048, 2816, 4096):
            # the combine kernel is instantiated per hidden size; refuse others here, in Python
            raise ValueError(f"the expert combine is not built for hidden size {cfg.hidden}")
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        from quail_b200.utils.op_timer import OpTimer
        self.timer = OpTimer()       # QB_OP_TIMING=1: device ms per MoE step (route, plan, dispatch + gate_up, ...)
        self.W = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        E, K, H, I = cfg.num_experts, cfg.top_k, cfg.hidden, cfg.moe_intermediate
        assert E % self.W == 0 and H % 256 == 0 and I % 128 == 0 and (2 * I) % 256 == 0
        self.E, self.K, self.H, self.I = E, K, H, I
        self.Epr = E // self.W
        self.M_max = _align(max_tokens, 128)
        # rows one rank can receive: every token of every rank sends at most
        # min(K, Epr) rows here; each local expert pads to 128
        self.R_cap = self.W * self.M_max * min(K, self.Epr) + self.Epr * 128
        self.t_cap = self.R_cap // 128
        dev = self.device
        i32 = torch.int32
        n_items = self.M_max * K
        self.ids = torch.zeros(n_items, dtype=i32, device=dev)
        self.wts = torch.zeros(n_items, dtype=torch.float32, device=dev)
        self.pos = torch.zeros(n_items, dtype=i32, device=dev)
        self.src_list = torch.zeros(n_items, dtype=i32, device=dev)
        self.counts = torch.zeros(E, dtype=i32, device=dev)
        self.plan = torch.zeros(ops.native().moe_plan_ints(E, self.Epr, self.t_cap), dtype=i32, device=dev)
        self.cum = torch.zeros(self.Epr, dtype=i32, device=dev)
        self.y = torch.empty(self.R_cap, I, dtype=torch.float8_e4m3fn, device=dev)
        self.ysf = torch.empty(ops.sf_bytes(self.R_cap, I), dtype=torch.uint8, device=dev)
        # the arena: [recv A | recv SF | recv meta | comb | recv counts | comb counter | counts_all | cflags]
        sizes = [
            ("recv_a", self.R_cap * H),
            ("recv_sf", ops.sf_bytes(self.R_cap, H)),
            ("recv_meta", self.R_cap * 8),
            ("comb", n_items * H * 2),
            ("recv_count", 4 * self.Epr),
            ("comb_counter", 4),
            ("counts_all", 4 * 2 * self.W * E),
            ("cflag", 4 * 2 * self.W),
        ]
        self.off = {}
        total = 0
        for name, nbytes in sizes:
            self.off[name] = total
            total += _align(nbytes, 256)
        if self.W > 1:
            import torch.distributed._symmetric_memory as symm
            self.buf = symm.empty(total, dtype=torch.uint8, device=dev)
            self.buf.zero_()
            name = group.group_name if hasattr(group, "group_name") else dist.group.WORLD.group_name
            self.handle = symm.rendezvous(self.buf, name)
            self.peers = [int(p) for p in self.handle.buffer_ptrs]
        else:
            self.buf = torch.zeros(total, dtype=torch.uint8, device=dev)
            self.peers = [self.buf.data_ptr()]
        self.comm = "fused"     # "nccl": the NCCL all-to-all baseline (forward_nccl)
        self.act = 1 if getattr(cfg, "hidden_act", "silu") == "gelu_tanh" else 0   # experts' gate activation
        self.epoch = 0          # MoE layers run so far (count-exchange flags carry it)
        self.comb_units = 0     # cumulative (row, 128-column) units this rank expects in its combine buffer
        if self.W > 1:
            torch.cuda.synchronize(dev)
            dist.barrier(group)

    # ------------------------------------------------------------ views
    def _view(self, name, nbytes):
        o = self.off[name]
        return self.buf[o:o + nbytes]

    def recv_a(self):
        return self._view("recv_a", self.R_cap * self.H).view(torch.float8_e4m3fn).view(self.R_cap, self.H)

    def recv_sf(self):
        from quail_b200 import ops
        return self._view("recv_sf", ops.sf_bytes(self.R_cap, self.H))

    def recv_meta(self):
        return self._view("recv_meta", self.R_cap * 8).view(torch.int32).view(self.R_cap, 2)

    def comb(self, M):
        return self._view("comb", M * self.K * self.H * 2).view(torch.bfloat16).view(M * self.K, self.H)

    def recv_count(self):
        return self._view("recv_count", 4 * self.Epr).view(torch.int32)

    def comb_counter(self):
        return self._view("comb_counter", 4).view(torch.int32)

    def counts_all(self):
        return self._view("counts_all", 4 * 2 * self.W * self.E).view(torch.int32)

    def cflag(self):
        return self._view("cflag", 4 * 2 * self.W).view(torch.int32)

    def peer(self, name) -> list[int]:
        return [p + self.off[name] for p in self.peers]

    def plan_header(self) -> tuple[int, int]:
        """(m-tiles, dispatch units) of the last plan (synchronizes; for tests)."""
        h = self.plan[:2].tolist()
        return h[0], h[1]

    # ------------------------------------------------------------ one MoE layer
    def forward(self, x8, xsf, xb, h, L, next_norm=None, eps: float = 1e-6):
        """MoE MLP of one layer for this rank's M tokens.

        x8/xsf: the post-attention RMSNorm of `h` as e4m3 + MX atoms, xb the
        same in bf16 (router input). h [M, H] bf16 is updated in place
        (residual + expert outputs). With `next_norm`, returns the next
        layer's input RMSNorm of the new h as (e4m3, atoms); else None.
        """
        if self.comm == "nccl":
            return self.forward_nccl(x8, xsf, xb, h, L, next_norm, eps)
        from quail_b200 import ops
        C = ops.native()
        M = h.shape[0]
        assert M <= self.M_max, f"{M} tokens > the MoE buffers' {self.M_max}"
        E, K = self.E, self.K
        self.epoch += 1
        ops.count_launch(5)
        tm = self.timer
        with tm("route"):
            if M > 0:
                logits = ops.gemm(xb, L["router"], bn=128)
                ops.count_launch(1)
                C.moe_route(logits, E, K, self.ids, self.wts, self.pos, self.counts)
            else:
                # a rank without tokens this step still serves its experts to the others
                x8 = self.recv_a()[:0]
        with tm("plan (count exchange)"):
            C.moe_plan(self.counts, self.peer("counts_all") if self.W > 1 else [],
                       self.peer("cflag") if self.W > 1 else [], self.counts_all(), self.cflag(),
                       self.plan, self.cum, self.rank, E, self.t_cap, self.epoch)
            C.moe_sort(self.ids, self.pos, M * K, self.plan, E, self.src_list)
        with tm("dispatch + gate_up"):
            C.moe_gate_up(x8, xsf, self.src_list, self.wts, self.plan, self.rank, E, K, self.t_cap,
                          self.peer("recv_a"), self.peer("recv_sf"), self.peer("recv_meta"),
                          self.peer("recv_count"), self.recv_a(), self.recv_sf(), self.recv_count(), L["wgu"],
                          L["sgu"], self.y, self.ysf, self.act)
        with tm("down + combine push"):
            C.moe_down(self.y, self.ysf, self.plan, E, self.t_cap, self.recv_meta(), L["wd"], L["sd"],
                       self.peer("comb"), self.peer("comb_counter"))
        self.comb_units = (self.comb_units + M * K * (self.H // 128)) & 0xFFFFFFFF
        want = self.comb_units  # compared modulo 2^32 on the device
        with tm("combine + norm"):
            if next_norm is None:
                C.moe_combine(self.comb(M), M, K, self.comb_counter(), want, h, None, eps, None, None)
                return None
            y8 = torch.empty(M, self.H, dtype=torch.float8_e4m3fn, device=h.device)
            ysf = torch.empty(ops.sf_bytes(M, self.H), dtype=torch.uint8, device=h.device)
            C.moe_combine(self.comb(M), M, K, self.comb_counter(), want, h, next_norm, eps, y8, ysf)
        return y8, ysf

    # ------------------------------------------------------------ NCCL baseline
    def forward_nccl(self, x8, xsf, xb, h, L, next_norm=None, eps: float = 1e-6):
        """The same MoE layer with NCCL all-to-all dispatch and combine (the baseline).

        Route on the device; per-expert counts exchanged with all_to_all and
        read on the host (the split sizes); token rows (e4m3 + row-major scale
        bytes) sorted by expert and sent with all_to_all_single; received rows
        laid out expert by expert for the same grouped GEMMs (no dispatch
        work in the kernel, no peer stores in the epilogue; the routing weight
        travels with the row and is applied in the down epilogue, as in the
        fused path); outputs sent home with a second all_to_all_single and
        summed into the residual.
        """
        import torch.distributed as dist
        from quail_b200 import ops
        from quail_b200.ops.quant import pack_sf_atoms, unpack_sf_atoms
        C = ops.native()
        M, H, K, E, Epr, W = h.shape[0], self.H, self.K, self.E, self.Epr, self.W
        dev = h.device
        g = self.group
        if not hasattr(self, "_nb"):
            self._nb = {"out": torch.empty(self.R_cap, H, dtype=torch.bfloat16, device=dev),
                        "ctr": torch.zeros(8, dtype=torch.int32, device=dev)}
        self.epoch += 1
        tm = self.timer
        with tm("route"):
            if M > 0:
                logits = ops.gemm(xb, L["router"], bn=128)
                C.moe_route(logits, E, K, self.ids, self.wts, self.pos, self.counts)
                ops.count_launch(1)
                ids = self.ids[:M * K].long()
            else:
                ids = torch.zeros(0, dtype=torch.long, device=dev)
        sp = tm("counts all-to-all + host split sizes + rows all-to-all + layout")
        sp.__enter__()
        self.counts.zero_()
        order = torch.argsort(ids, stable=True)
        cnt_e = torch.bincount(ids, minlength=E).to(torch.int32)
        recv_cnt = torch.empty(E, dtype=torch.int32, device=dev)     # [W sources][Epr local experts]
        dist.all_to_all_single(recv_cnt, cnt_e, group=g)
        host = torch.cat([cnt_e, recv_cnt]).cpu()                    # the host needs the split sizes
        send_sizes = host[:E].view(W, Epr).sum(1).tolist()
        rc = host[E:].view(W, Epr)
        recv_sizes = rc.sum(1).tolist()
        n_recv = int(sum(recv_sizes))
        # payload rows: e4m3 bytes + row-major scale bytes of each item's token
        tok = (order // K)
        RB = H + H // 32 + 4   # e4m3 row | scale bytes | routing weight (fp32)
        if M > 0:
            w4 = self.wts[:M * K][order].contiguous().view(torch.uint8).view(-1, 4)
            rows = torch.cat([torch.cat([x8.view(torch.uint8), unpack_sf_atoms(xsf, M, H)], dim=1)[tok], w4], dim=1)
        else:
            rows = torch.zeros(0, RB, dtype=torch.uint8, device=dev)
        recv = torch.empty(n_recv, RB, dtype=torch.uint8, device=dev)
        dist.all_to_all_single(recv, rows, output_split_sizes=recv_sizes, input_split_sizes=send_sizes, group=g)
        # expert-major padded layout of the received rows
        tot = rc.sum(0)                                               # rows per local expert
        padded = ((tot + 127) // 128) * 128
        base = torch.cumsum(padded, 0) - padded
        le = torch.repeat_interleave(torch.arange(Epr).repeat(W), rc.flatten())   # received order
        perm = torch.argsort(le, stable=True)
        le_s = le[perm]
        first = torch.cumsum(tot, 0) - tot
        dest = (base[le_s] + torch.arange(n_recv) - first[le_s]).to(dev)
        perm_d = perm.to(dev)
        R = int(padded.sum())
        ra = self.recv_a()
        ra.view(torch.uint8)[dest] = recv[perm_d, :H]
        sfm = torch.zeros(max(R, 128), H // 32, dtype=torch.uint8, device=dev)
        sfm[dest] = recv[perm_d, H:H + H // 32]
        packed = pack_sf_atoms(sfm)
        self.recv_sf()[:packed.numel()].copy_(packed)
        meta = self.recv_meta()
        meta[dest, 0] = (self.rank << 28) | perm_d.to(torch.int32)
        meta[dest, 1] = recv[perm_d, H + H // 32:].contiguous().view(torch.int32).flatten()
        # tile table on the host: (expert, first row, valid rows)
        tiles = []
        for j in range(Epr):
            for i in range(int(padded[j]) // 128):
                tiles.append((j, int(base[j]) + i * 128, min(128, int(tot[j]) - i * 128)))
        pv = torch.zeros(self.plan.numel(), dtype=torch.int32)
        pv[0], pv[1] = len(tiles), 0
        tofs = 8 + 4 * E + 1 + Epr
        if tiles:
            t = torch.tensor(tiles, dtype=torch.int32)
            pv[tofs:tofs + len(tiles)] = t[:, 0]
            pv[tofs + self.t_cap:tofs + self.t_cap + len(tiles)] = t[:, 1]
            pv[tofs + 2 * self.t_cap:tofs + 2 * self.t_cap + len(tiles)] = t[:, 2]
        self.plan.copy_(pv, non_blocking=False)
        sp.__exit__(None, None, None)
        ops.count_launch(2)
        e8 = x8[:0] if M > 0 else self.recv_a()[:0]
        with tm("gate_up"):
            C.moe_gate_up(e8, self.recv_sf(), self.src_list, self.wts, self.plan, self.rank, E, K, self.t_cap,
                          self.peer("recv_a")[self.rank:self.rank + 1] * W, self.peer("recv_sf")[:1] * W,
                          self.peer("recv_meta")[:1] * W, self.peer("recv_count")[:1] * W,
                          self.recv_a(), self.recv_sf(), self.recv_count(), L["wgu"], L["sgu"], self.y, self.ysf, self.act)
        out = self._nb["out"]
        with tm("down"):
            C.moe_down(self.y, self.ysf, self.plan, E, self.t_cap, meta, L["wd"], L["sd"],
                       [out.data_ptr()] * W, [self._nb["ctr"].data_ptr()] * W)
        back = torch.empty(M * K, H, dtype=torch.bfloat16, device=dev)
        with tm("outputs all-to-all"):
            dist.all_to_all_single(back, out[:n_recv], output_split_sizes=send_sizes,
                                   input_split_sizes=recv_sizes, group=g)
        if M == 0:
            return None
        with tm("combine + norm"):
            items = torch.empty_like(back)
            items[order] = back       # rows come back weighted by the expert owner's epilogue
            zero = self._nb["ctr"][4:5]
            ops.count_launch(1)
            if next_norm is None:
                C.moe_combine(items, M, K, zero, 0, h, None, eps, None, None)
                return None
            y8 = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
            ysf = torch.empty(ops.sf_bytes(M, H), dtype=torch.uint8, device=dev)
            C.moe_combine(items, M, K, zero, 0, h, next_norm, eps, y8, ysf)
        return y8, ysf


def run_lockstep(executor, pipe, cpu_group) -> None:
    """Run a stage executor on every rank of an expert-parallel job in lockstep.

    Each MoE layer exchanges per-expert counts with every peer, so every rank
    must run the same number of forward passes. Each round, every rank
    launches exactly one pass: its next chunk, or an idle pass (MoE layers
    only, no tokens of its own: it still computes its experts for the
    others' tokens). The rounds end when no rank has queued or in-flight
    work; that decision is a host-side all-reduce on `cpu_group` (gloo), so
    the GPU stream never waits for it.
    """
    import time

    import torch
    import torch.distributed as dist
    ex = executor
    t0 = time.perf_counter()
    flag = torch.zeros(1, dtype=torch.int32)
    while True:
        flag[0] = 1 if (ex.pending() or ex._inflight) else 0
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=cpu_group)
        if int(flag[0]) == 0:
            break
        specs = ex._admit() if ex.pending() else []
        if specs:
            ex._launch(specs)
            while len(ex._inflight) > 1:
                ex._collect_one()
        else:
            pipe.idle_pass()
            if ex._inflight:
                ex._collect_one()
    if ex.pending():
        raise RuntimeError(f"{len(ex.queue) + len(ex.follow) + len(ex.cont)} tasks were never admitted")
    ex.stats.wall_s += time.perf_counter() - t0
