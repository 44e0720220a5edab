"""Hybrid (Qwen3.5) kernels and pipeline against their fp32 PyTorch statements."""

import numpy as np
import pytest
import torch

from quail_b200 import ops
from quail_b200.models import qwen3_5 as Q
from quail_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp(min=1e-12)).item()


@pytest.fixture(autouse=True)
def _no_kernel_errors():
    torch.manual_seed(0)
    yield
    assert ops.read_and_clear_error(0) == 0


def _seqs(lengths, q_lens, P, KH, D, pages=1024):
    """One own segment per sequence (plus a shared 48-token prefix segment when lengths[i] > q_lens[i])."""
    from test_kernels_gpu import _segmented_case
    specs = []
    for n, q in zip(lengths, q_lens):
        specs.append((q, [48, n]) if n != q else (q, [n]))
    return _segmented_case(P, specs, QH=KH * 1, KH=KH, D=D, pages=pages)


@pytest.mark.parametrize("D,QH,KH", [(256, 4, 2), (256, 16, 4), (256, 12, 2), (64, 8, 2), (128, 16, 4)])
def test_small_attention_with_gate(D, QH, KH):
    from test_kernels_gpu import _segmented_case
    specs = [(100, [48, 100]), (1, [48, 300, 65]), (7, [48, 7]), (1, [17]), (40, [48, 200, 40]), (130, [130])]
    q, kc, vc, seqs, pl = _segmented_case(16, specs, QH=QH, KH=KH, D=D, pages=2048)
    scale = ref.softmax_scale(D)
    want = ref.segmented_attention(q, kc, vc, seqs, pl, scale).view(-1, QH, D)
    T = q.shape[0]
    gate_src = torch.randn(T, QH, 2 * D, device=DEV).bfloat16()
    tiles = ref.attention_tiles(seqs)
    one = [i for i, (n, _) in enumerate(specs) if n == 1]
    tiles = torch.tensor([t for t in tiles.tolist() if t[0] not in one], dtype=torch.int32, device=DEV)
    dseqs = torch.tensor(one, dtype=torch.int32, device=DEV)
    out = torch.empty(T, QH * D, dtype=torch.bfloat16, device=DEV)
    gate = gate_src.view(T, QH * 2 * D)[:, D:]
    ops.native().small_attention(q, kc, vc, seqs.to(DEV), tiles, dseqs, pl.to(DEV), scale, out, gate, 2 * D)
    want_g = want * torch.sigmoid(gate_src[:, :, D:].float())
    assert rel_err(out.view(T, QH, D), want_g) < 1e-2
    out2 = torch.empty_like(out)
    ops.native().small_attention(q, kc, vc, seqs.to(DEV), tiles, dseqs, pl.to(DEV), scale, out2, None, 0)
    assert rel_err(out2.view(T, QH, D), want) < 1e-2


def test_hybrid_qk_rope_kv():
    T, QH, KH, D, rd = 37, 4, 2, 256, 64
    proj = torch.randn(T, QH * 2 * D + 2 * KH * D, device=DEV).bfloat16()
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device=DEV)
    qw = (0.1 * torch.randn(D, device=DEV)).bfloat16()
    kw = (0.1 * torch.randn(D, device=DEV)).bfloat16()
    cs = ref.rope_cos_sin(8192, rd, 1e7, device=DEV)
    kc = torch.zeros(8, 16, KH, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(128, device=DEV)[:T].int()
    slots[3] = -1
    q = torch.empty(T, QH, D, dtype=torch.bfloat16, device=DEV)
    ops.native().hybrid_qk_rope_kv(proj, QH, KH, True, pos, qw, kw, True, cs, slots, kc, vc, q, 1e-6, 0, 0)
    qg = proj[:, :QH * 2 * D].view(T, QH, 2 * D)
    want_q = Q.rope_partial(Q.rmsnorm_offset(qg[..., :D], qw, 1e-6), pos, cs, rd)
    assert rel_err(q, want_q) < 1e-2
    k = proj[:, QH * 2 * D:QH * 2 * D + KH * D].view(T, KH, D)
    v = proj[:, QH * 2 * D + KH * D:].view(T, KH, D)
    want_k = Q.rope_partial(Q.rmsnorm_offset(k, kw, 1e-6), pos, cs, rd)
    ok = slots >= 0
    assert rel_err(kc.view(-1, KH, D)[slots[ok].long()], want_k[ok]) < 1e-2
    assert torch.equal(vc.view(-1, KH, D)[slots[ok].long()], v[ok])


@pytest.mark.parametrize("dk,mode", [(128, 1), (64, 1), (128, 2), (128, 3)])
def test_gdn_layer_against_recurrence(dk, mode):
    """mode 1: the per-token kernel (fp32 throughout); modes 2 and 3: the chunked tensor-core form
    in one kernel and split in three (bf16 operands, fp32 accumulation and state), sequences of
    1 to 3 chunks."""
    Hk, Hv, dv, W = 2, 4, dk, 4
    C = 2 * Hk * dk + Hv * dv
    lens = [5, 1, 70, 33] if mode == 1 else [5, 1, 150, 64, 33]
    T = sum(lens)
    G, slots = 3, 8
    gi = 1
    proj = (torch.randn(T, C + Hv * dv + 2 * Hv, device=DEV) * 0.5).bfloat16()
    conv_w = torch.randn(C, W, device=DEV) * 0.3
    A_log = torch.log(1 + 15 * torch.rand(Hv, device=DEV))
    dt_bias = torch.randn(Hv, device=DEV) - 3
    norm_w = (1 + 0.1 * torch.randn(dv, device=DEV)).bfloat16()
    seqs = torch.zeros(len(lens), 12, dtype=torch.int32)
    q0 = 0
    for i, n in enumerate(lens):
        seqs[i, 0], seqs[i, 1], seqs[i, 2], seqs[i, 4] = q0, n, 1, n
        q0 += n
    sio = torch.tensor([[-1, 0], [2, 1], [3, 3], [-1, 4], [5, 6]][:len(lens)], dtype=torch.int32)  # fresh, from a slot, continue
    conv_state = torch.randn(slots, G, W - 1, C, device=DEV)
    ssm_state = torch.randn(slots, G, Hv, dk, dv, device=DEV) * 0.1
    cs0, ss0 = conv_state.clone(), ssm_state.clone()
    conv_out = torch.empty(T, C, device=DEV)
    o = torch.empty(T, Hv * dv, device=DEV)
    y = torch.empty(T, Hv * dv, dtype=torch.bfloat16, device=DEV)
    ops.native().gdn_layer(proj, conv_w, A_log, dt_bias, norm_w, seqs.to(DEV), sio.to(DEV), conv_state, ssm_state,
                           gi, Hk, Hv, dk, dv, 1e-6, conv_out, o, y, mode)
    tol = 1e-3 if mode == 1 else 2e-2
    pf = proj.float()
    g, beta = Q.gdn_gates(pf[:, C + Hv * dv + Hv:C + Hv * dv + 2 * Hv], pf[:, C + Hv * dv:C + Hv * dv + Hv],
                          A_log, dt_bias)
    for i, n in enumerate(lens):
        a = int(seqs[i, 0])
        src, dst = sio[i].tolist()
        win = cs0[src, gi].clone() if src >= 0 else torch.zeros(W - 1, C, device=DEV)
        S = ss0[src, gi].clone() if src >= 0 else torch.zeros(Hv, dk, dv, device=DEV)
        c, win = Q.causal_conv(pf[a:a + n, :C], win, conv_w)
        qq = torch.nn.functional.normalize(c[:, :Hk * dk].view(n, Hk, dk), dim=-1) * dk ** -0.5
        kk = torch.nn.functional.normalize(c[:, Hk * dk:2 * Hk * dk].view(n, Hk, dk), dim=-1)
        vv = c[:, 2 * Hk * dk:].view(n, Hv, dv)
        rep = Hv // Hk
        out = Q.delta_rule(qq.repeat_interleave(rep, 1), kk.repeat_interleave(rep, 1), vv, g[a:a + n],
                           beta[a:a + n], S)
        assert rel_err(o[a:a + n].view(n, Hv, dv), out) < tol, (i, rel_err(o[a:a + n].view(n, Hv, dv), out))
        assert rel_err(conv_state[dst, gi], win) < 1e-5
        assert rel_err(ssm_state[dst, gi], S) < tol, (i, rel_err(ssm_state[dst, gi], S))
        z = pf[a:a + n, C:C + Hv * dv].view(n, Hv, dv)
        want_y = ref.rmsnorm(out, norm_w, 1e-6) * torch.nn.functional.silu(z)
        assert rel_err(y[a:a + n].view(n, Hv, dv), want_y) < 1e-2


@pytest.mark.parametrize("name", ["qwen3.5-gpu-tiny", "qwen3.5-gpu-tiny-fp8", "qwen3.6-moe-gpu-tiny",
                                  "qwen3.5-gpu-tiny-nvfp4"])
def test_hybrid_pipeline_matches_fp32_model(name):
    """bf16 and fp8 checkpoints (the fp8 one: attention and MLP on the block-scaled fp8 GEMM)
    against the fp32 model of the same (dequantized) weights."""
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor, Task
    from quail_b200.models.config import MODEL_CONFIGS
    from quail_b200.models.qwen3_5_gpu import Qwen35Pipeline
    from quail_b200.models.weights import random_checkpoint
    cfg = MODEL_CONFIGS[name]
    ckpt = random_checkpoint(cfg, seed=9, device=DEV)
    ids = list(range(16))
    pipe = Qwen35Pipeline(cfg, ckpt, DEV, head_rows=ids)
    exact = Q.Qwen35Reference(cfg, ckpt, device=DEV, head_rows=ids)

    def run(model, dtype):
        arena = KVArena.for_model(cfg, 128, 16, device=DEV, dtype=dtype, state_slots=32)
        ex = StageExecutor(model, arena, 256, min_piece=16)
        got = {}
        rng = np.random.default_rng(0)
        prefix = rng.integers(0, 4096, 48).astype(np.int32)
        docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 200, 64, 300)]
        suffix = rng.integers(0, 4096, 12).astype(np.int32)
        ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
        for i, d in enumerate(docs):
            ex.submit(Task(key=i, tokens=np.concatenate([d, suffix]), pos_start=48, reads=[("p", 48)], readout=True,
                           on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
        ex.run()
        return torch.stack([got[i] for i in range(len(docs))])

    got = run(pipe, torch.bfloat16)
    want = run(exact, torch.float32)
    assert ops.read_and_clear_error(0) == 0
    d = rel_err(got, want)
    print(f"hybrid {name} kernel-vs-fp32: {d:.4f}")
    if not cfg.fp8:
        assert d < 0.1
        return
    # fp8: as close to the exact model as an fp32 model that requantizes the
    # weights and quantizes every fp8 GEMM input where the kernels do
    emul = Q.Qwen35Reference(cfg, ckpt, device=DEV, head_rows=ids, emulate_kernels=True)
    d_emul = rel_err(run(emul, torch.float32), want)
    print(f"hybrid {name} emulated-vs-fp32: {d_emul:.4f}")
    assert d < 1.5 * d_emul + 0.02, (d, d_emul)


@pytest.mark.parametrize("name", ["qwen3.5-gpu-tiny", "qwen3.6-moe-gpu-tiny"])
def test_hybrid_session_on_gpu(name):
    import pyarrow as pa

    import quail_b200 as quail
    cfg = quail.EngineConfig(model=name, device="b200", chunk_tokens=512)
    t = pa.table({"id": list(range(6)), "body": ["the plot is long", "great music", "bad ending", "short story",
                                                  "money talk", "cast list"]})
    with quail.Session(config=cfg) as s:
        s.register("r", quail.DocumentProvider.from_table(t, id_col="id"))
        kept = s.sql("SELECT id FROM r WHERE AI.IF(PROMPT('Is it about music? {0}', body))").collect()
        assert set(kept.column("id").to_pylist()) <= set(range(6))
        out = s.sql("SELECT id, AI.MAP(body, 'Summarize', 4) AS m FROM r").collect()
        assert out.num_rows == 6


def test_short_conv_kernel():
    from quail_b200.models.lfm2 import short_conv_ref
    H, W = 384, 3
    lens = [4, 1, 50]
    T = sum(lens)
    bcx = torch.randn(T, 3 * H, device=DEV).bfloat16()
    w = torch.randn(H, W, device=DEV) * 0.4
    seqs = torch.zeros(len(lens), 12, dtype=torch.int32)
    q0 = 0
    for i, n in enumerate(lens):
        seqs[i, 0], seqs[i, 1], seqs[i, 2], seqs[i, 4] = q0, n, 1, n
        q0 += n
    sio = torch.tensor([[-1, 0], [2, 1], [3, 3]], dtype=torch.int32)
    state = torch.randn(6, 2, W - 1, H, device=DEV)
    s0 = state.clone()
    y = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.native().short_conv(bcx, w, seqs.to(DEV), sio.to(DEV), state, 1, y)
    for i, n in enumerate(lens):
        a = int(seqs[i, 0])
        src, dst = sio[i].tolist()
        win = s0[src, 1] if src >= 0 else torch.zeros(W - 1, H, device=DEV)
        out, win = short_conv_ref(bcx[a:a + n], win, w)
        assert rel_err(y[a:a + n], out) < 1e-2
        assert rel_err(state[dst, 1], win) < 1e-5


def test_lfm2_pipeline_matches_fp32_model():
    from quail_b200.engine.arena import KVArena
    from quail_b200.engine.stage_executor import StageExecutor, Task
    from quail_b200.models.config import LFM2_GPU_TINY
    from quail_b200.models.lfm2 import Lfm2Pipeline, Lfm2Reference
    from quail_b200.models.weights import random_checkpoint
    cfg = LFM2_GPU_TINY
    ckpt = random_checkpoint(cfg, seed=2, device=DEV)
    ids = list(range(16))

    def run(model, dtype):
        arena = KVArena.for_model(cfg, 128, 16, device=DEV, dtype=dtype, state_slots=32)
        ex = StageExecutor(model, arena, 256, min_piece=16)
        got = {}
        rng = np.random.default_rng(3)
        prefix = rng.integers(0, 4096, 48).astype(np.int32)
        docs = [rng.integers(0, 4096, n).astype(np.int32) for n in (10, 200, 64, 300)]
        suffix = rng.integers(0, 4096, 12).astype(np.int32)
        ex.submit(Task(key="p", tokens=prefix, pos_start=0, free_after=False))
        for i, d in enumerate(docs):
            ex.submit(Task(key=i, tokens=np.concatenate([d, suffix]), pos_start=48, reads=[("p", 48)], readout=True,
                           on_done=lambda t, row, i=i: got.__setitem__(i, row.float().cpu())))
        ex.run()
        return torch.stack([got[i] for i in range(len(docs))])

    got = run(Lfm2Pipeline(cfg, ckpt, DEV, head_rows=ids), torch.bfloat16)
    want = run(Lfm2Reference(cfg, ckpt, device=DEV, head_rows=ids), torch.float32)
    assert ops.read_and_clear_error(0) == 0
    d = rel_err(got, want)
    print(f"lfm2 kernel-vs-fp32: {d:.4f}")
    assert d < 0.1


def test_document_isolated_model_on_the_kernels():
    """mammoth-1's shape at the smallest size: the Qwen3.5 kernels with the document block and
    each question read both ways, answered by option-letter logits, against the fp32 model of the
    same weights (same SQL; scores to bf16 accuracy)."""
    import pyarrow as pa

    import quail_b200 as quail
    from quail_b200.api.engine import ModelEngine
    from quail_b200.engine.arena import KVArena
    from quail_b200.models.build import random_checkpoint_on
    rng = np.random.default_rng(3)
    words = ["refund", "late", "broken", "great", "thanks", "order", "invoice", "parcel"]
    bodies = [" ".join(rng.choice(words, size=int(rng.integers(3, 60)))) for _ in range(12)]
    q = ("SELECT id, AI.SCORE(PROMPT('Is {0} a refund request?', body)) AS s, "
         "AI.CLASSIFY(body, ['billing', 'shipping', 'praise']) AS c FROM t ORDER BY id")
    cfg = quail.EngineConfig(model="mammoth-gpu-tiny", device="b200", chunk_tokens=2048)
    with quail.Session(config=cfg) as s:
        s.register("t", pa.table({"id": list(range(12)), "body": bodies}))
        got = s.sql(q).collect()
        eng = s.engine()
        m = eng.cfg
        ref_model = Q.Qwen35Reference(m, random_checkpoint_on(m, eng.device, seed=0), device=eng.device)
        arena = KVArena.for_model(m, 2048, 16, device=eng.device, dtype=torch.float32, state_slots=64)
        s._engine = ModelEngine.from_replica(cfg, ref_model, arena, tokenizer=eng.tokenizer)
        want = s.sql(q).collect()
        s._engine = eng
    a, b = np.array(got.column("s").to_pylist()), np.array(want.column("s").to_pylist())
    da, db = np.log(a / (1 - a)), np.log(b / (1 - b))
    spread = db.max() - db.min()
    assert spread > 1e-3, f"the reference scores do not separate the rows: {db}"
    # bf16 Gated DeltaNet and attention against fp32: the row-to-row pattern must match
    assert np.abs(da - db).max() < 0.35 * spread, (da, db)
    assert np.corrcoef(da, db)[0, 1] > 0.9, (da, db)
    agree = np.mean(np.array(got.column("c").to_pylist()) == np.array(want.column("c").to_pylist()))
    assert agree >= 0.8
