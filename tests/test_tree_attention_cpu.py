"""The tree attention path: stacked readers of a shared segment, merged by log-sum-exp.

The reference's tree path reads a chunk's own rows in one call and the rows
that read a resident shared segment, stacked, in a second, then merges the two
(quail/backends/quail/executor/attention.py:1395-1441, merge_attn_quant). Here
the packer builds the two tables and the fp32 statement of the path must equal
the unified read of the same chunk; sessions give the same answers on either path.
"""

import numpy as np
import pyarrow as pa
import pytest
import torch

import quail_b200 as quail
from quail_b200.engine.arena import PagePool
from quail_b200.engine.chunk import ChunkPacker, SeqSpec, tree_saves
from quail_b200.ops import reference as ref


def _chunk(tree: str):
    pool = PagePool(200, 16)
    pool.alloc("prefix", 100)
    pool.alloc("anchor", 150)
    specs = []
    rng = np.random.default_rng(0)
    for i, n in enumerate((5, 40, 17, 33, 1)):
        key = ("doc", i)
        pool.alloc(key, n)
        reads = [("prefix", 100)] + ([("anchor", 150)] if i in (1, 3, 4) else [])
        specs.append(SeqSpec(reads=reads, own_key=key, own_start=0, tokens=rng.integers(0, 100, n),
                             pos_start=100, readout=True))
    return pool, ChunkPacker(pool, "cpu", pin=False, tree=tree).pack(specs)


def test_the_packer_stacks_the_longest_shared_segment():
    _, chunk = _chunk("tree")
    tree = chunk.tree
    assert tree is not None
    # readers 1 and 3 (prefix + the longer anchor, 40 and 33 rows) stack the anchor; 0, 2 the prefix;
    # the one-token sequence stays on the decode kernel
    seqs_b = tree["seqs_b"].numpy()
    assert sorted(seqs_b[:, 4].tolist()) == [100, 150] and (seqs_b[:, 3] == 1).all()
    assert tree["rows"].numel() == 5 + 40 + 17 + 33
    src = tree["source"].numpy()
    assert src[95] == -1 and (src[:95] >= 0).all()
    a = tree["seqs_a"].numpy()
    assert a[1, 2] == 2 and a[1, 4] == 100        # reader 1 keeps the prefix, stacks the anchor
    assert a[0, 2] == 1                            # reader 0 stacked its only earlier segment
    assert ChunkPacker(PagePool(4, 16), "cpu", pin=False).tree == "unified"


def test_the_tree_read_equals_the_unified_read():
    pool, chunk = _chunk("tree")
    g = torch.Generator().manual_seed(1)
    QH, KH, D = 4, 2, 32
    kc = torch.randn(200, 16, KH, D, generator=g)
    vc = torch.randn(200, 16, KH, D, generator=g)
    q = torch.randn(chunk.num_tokens, QH, D, generator=g)
    want = ref.segmented_attention(q, kc, vc, chunk.seqs, chunk.page_list, 0.3)
    got = ref.tree_attention(q, kc, vc, chunk.seqs, chunk.page_list, chunk.tree, 0.3)
    assert torch.allclose(got, want, atol=1e-5)


def test_the_cost_rule():
    assert tree_saves([20] * 40, 1024)            # many short readers of a long prefix
    assert not tree_saves([500, 700], 1024)       # long readers fill their blocks anyway
    assert not tree_saves([20, 20], 64)           # too little to save


@pytest.mark.parametrize("attention", ["tree", None])
def test_join_pairs_answer_the_same_on_either_path(attention):
    # an AI join's pairs read their anchor document's KV: pairs of one anchor in a chunk stack it
    from quail_b200.api.engine import CallSpec, ModelEngine
    anchors = [" ".join(f"clause{i}x{j}" for j in range(120)) for i in range(2)]
    pairs = [(k % 2, f"short note {k}") for k in range(12)]
    call = CallSpec(kind="score", tail="\nDo they match?\nANSWER:", name="m")
    got, passes = {}, {}
    for mode in (attention, "unified"):
        eng = ModelEngine(quail.EngineConfig(model="qwen3-tiny", device="cpu", attention=mode))
        got[mode] = [v["m"] for v in eng.run_pairs("Compare:\n", anchors, pairs, call).values]
        passes[mode] = eng.executor.stats.tree_passes
    assert passes["unified"] == 0 and passes[attention] > 0
    assert np.allclose(got[attention], got["unified"], atol=1e-4)
