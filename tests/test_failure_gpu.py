"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every device-side wait (mbarrier phases, peer flags and counters) has a
clock budget; when it runs out the kernel records an error code in the
device's status word, stops waiting and returns, and the host reads the
code after the stream. Here the reduce-norm kernel of the tensor-parallel
path waits on a peer counter that nothing raises, with the budget set to
about a millisecond: the launch must come back quickly with the peer-timeout
code (4), and the GPU must still compute correctly afterwards.
"""

import time

import pytest
import torch

from quail_b200 import ops

pytestmark = pytest.mark.gpu

PEER_TIMEOUT = 4


def test_a_peer_wait_that_runs_out_reports_and_leaves_the_gpu_usable():
    dev = "cuda"
    rpr, H = 8, 1024
    slots = torch.zeros(1, rpr, H, device=dev, dtype=torch.bfloat16)
    counters = torch.zeros(4, device=dev, dtype=torch.int32)        # nobody ever adds to these
    resid = torch.randn(rpr, H, device=dev).bfloat16()
    before = resid.clone()
    w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    a_sym = torch.zeros(128, H, device=dev, dtype=torch.uint8)
    sf_sym = torch.zeros(H // 128 * 512, device=dev, dtype=torch.uint8)
    done = torch.zeros(1, device=dev, dtype=torch.int32)
    flag = torch.zeros(1, device=dev, dtype=torch.int32)
    assert ops.read_and_clear_error(0) == 0
    ops.set_wait_budget(2_000_000)          # about a millisecond
    try:
        t0 = time.perf_counter()
        ops.native().tp_reduce_norm(slots, 1, counters, 1, resid, w, 1e-6, a_sym, sf_sym, 0, done, 0, flag, 1)
        err = ops.read_and_clear_error(0)
        elapsed = time.perf_counter() - t0
    finally:
        ops.set_wait_budget(0)
    assert err == PEER_TIMEOUT
    assert elapsed < 1.0, elapsed
    assert torch.equal(resid, before)        # a CTA that gave up wrote nothing
    assert int(flag.item()) == 1             # and still signalled that it is done
    # the context is intact: a GEMM right after matches fp32
    a = torch.randn(256, 512, device=dev)
    b = torch.randn(384, 512, device=dev) * 0.05
    got = ops.gemm(a.bfloat16(), b.bfloat16())
    want = a.bfloat16().float() @ b.bfloat16().float().t()
    assert ((got.float() - want).norm() / want.norm()).item() < 1e-2
    assert ops.read_and_clear_error(0) == 0


def test_the_default_budget_is_restored():
    # with the default budget a wait that is satisfied at once never trips
    counters = torch.ones(1, device="cuda", dtype=torch.int32)
    rpr, H = 8, 1024
    slots = torch.zeros(1, rpr, H, device="cuda", dtype=torch.bfloat16)
    resid = torch.randn(rpr, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    a_sym = torch.zeros(128, H, device="cuda", dtype=torch.uint8)
    sf_sym = torch.zeros(H // 128 * 512, device="cuda", dtype=torch.uint8)
    done = torch.zeros(1, device="cuda", dtype=torch.int32)
    flag = torch.zeros(1, device="cuda", dtype=torch.int32)
    ops.native().tp_reduce_norm(slots, 1, counters, 1, resid, w, 1e-6, a_sym, sf_sym, 0, done, 0, flag, 1)
    assert ops.read_and_clear_error(0) == 0
