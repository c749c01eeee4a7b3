"""Failure detection on the GPU without a fault: a bounded wait runs out.

The self-test kernel waits, through the same wait routine as the decode and
prefill pipelines, on an mbarrier phase nothing completes.  It must give up
after its limit, report B200_DEV_WAIT_TIMEOUT in the status word and return;
the context must stay usable (a decode afterwards is still exact).
"""
from __future__ import annotations

import time

import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from b200attn import _lib, selftest_bounded_wait

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    status = selftest_bounded_wait(limit_ns=20_000_000)  # 20 ms
    elapsed = time.perf_counter() - t0
    assert status & _lib.DEV_WAIT_TIMEOUT
    assert elapsed >= 0.01, "the wait gave up before its limit"


def test_context_usable_after_a_timeout():
    from b200attn import _lib, paged_attention_batch_b200, selftest_bounded_wait

    assert selftest_bounded_wait(limit_ns=1_000_000) & _lib.DEV_WAIT_TIMEOUT
    g = torch.Generator().manual_seed(3)
    B, H, D, S, P = 3, 4, 32, 16, 24
    k = torch.randn((1, P, S, H, D), generator=g)
    v = torch.randn((1, P, S, H, D), generator=g)
    table = torch.randperm(P, generator=g)[:12].view(3, 4)
    ctx = torch.tensor([64, 17, 40])
    q = torch.randn((B, H, D), generator=g)
    d = torch.device("cuda")
    pool = cases.Pool(k.to(d), v.to(d), S)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    out = paged_attention_batch_b200(q.to(d), pool, table.to(d), ctx.to(d), 0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = oracle.paged_decode_online(q, k, v, table, ctx, 0)
    assert (out.cpu() - want).abs().max().item() <= 1e-4
