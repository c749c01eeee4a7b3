"""Parity at the BASELINE configurations as written, on the benchmarked launches.

The inputs, the launch and its split-K plan are those of bench.py's own
workloads (DecodeWorkload / PrefillWorkload), so the launch these tests check
is the launch the bench times:

* configuration 3: H=32, D=128, S=16, batch 1/8/32/128/256, contexts
  ~U[1, 4096] with length 1 and a non-multiple of 16, pool = blocks + 10 %,
  fp32 KV (fp32 q and out, max abs error <= 1e-4, TF32 never used) and bf16
  KV (<= 2e-2 against the fp32 oracle on the upcast pool);
* configuration 4: 64 requests x 32768 tokens, bf16 KV, fused KV write, the
  bench's split plan;
* configuration 5: one batched tcgen05 prefill launch over 16 sequences,
  H=32, D=128, chunks 64 and 512, prefixes 16*U{0..252}.

Expected values come from the float64 oracle (oracle/) on compacted
per-sequence sub-pools copied back from the device.  The fused KV write is
checked bit-exactly: after the launch the pool equals its pre-launch copy
with k_new / v_new stored at each slot (the index_put of
minivllm/attention.py:382-392), everywhere.
"""
from __future__ import annotations

import importlib.util
import math
from pathlib import Path

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
FP32_ATOL = 1e-4
BF16_ATOL = 2e-2


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_for_parity", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _dev():
    return torch.device("cuda", 0)


def _bits(t: torch.Tensor) -> torch.Tensor:
    """The tensor's raw bits (NaN == NaN compares as equal bits)."""
    return t.view(torch.int32) if t.element_size() == 4 else t.view(torch.int16)


def _expected_pool_after_write(wl) -> tuple[torch.Tensor, torch.Tensor]:
    """A device copy of the pool with the step's k_new / v_new written at
    the slots by torch index_put, as the reference's decode write does."""
    S = wl.pool.block_size
    slots = wl.dev["slots"]
    blocks, offs = torch.div(slots, S, rounding_mode="floor"), slots % S
    k, v = wl.k.clone(), wl.v.clone()
    k[0, blocks, offs] = wl.dev["k_new"].to(k.dtype)
    v[0, blocks, offs] = wl.dev["v_new"].to(v.dtype)
    return k, v


def _check_decode_rows(wl, out: torch.Tensor, rows, tol: float) -> float:
    """Compares out[rows] with the float64 dense oracle on each row's
    compacted sub-pool; returns the largest error seen."""
    S = wl.pool.block_size
    tables = wl.host["tables"]
    worst = 0.0
    for b in rows:
        n = wl.lens[b]
        nb = math.ceil(n / S)
        phys = tables[b, :nb].to(wl.device)
        ks = wl.k[:, phys].cpu()
        vs = wl.v[:, phys].cpu()
        want = oracle.paged_decode_dense(wl.host["q"][b:b + 1].float(), ks, vs,
                                         torch.arange(nb)[None], torch.tensor([n]), 0,
                                         compute_dtype=torch.float64)
        got = out[b:b + 1].float().cpu().double()
        err = (got - want).abs().max().item()
        assert err <= tol, f"request {b} (context {n}): max abs {err:.3e} > {tol}"
        worst = max(worst, err)
    return worst


def _run_decode(wl):
    """One benchmarked launch (the prepared call with its own workspace and
    split plan); returns its output after checking the status and the
    fused write."""
    want_k, want_v = _expected_pool_after_write(wl)
    wl.prepare()
    out = wl.call()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert torch.equal(_bits(wl.k), _bits(want_k)), "K pool differs from the expected write"
    assert torch.equal(_bits(wl.v), _bits(want_v)), "V pool differs from the expected write"
    del want_k, want_v
    return out


@pytest.mark.parametrize("kv", ["f32", "bf16"])
@pytest.mark.parametrize("batch", [1, 8, 32, 128, 256])
def test_cfg3_ragged_sweep(bench, batch, kv):
    torch.backends.cuda.matmul.allow_tf32 = False
    # q, k_new, v_new and out share the KV dtype: fp32 throughout for fp32 KV.
    wl = bench.DecodeWorkload("cfg3", 0, _dev(), batch=batch, kv_dtype=kv)
    assert wl.host["q"].dtype == wl.k.dtype
    lens = wl.lens
    assert lens[0] == 1 and lens[-1] % 16 != 0 and max(lens) <= 4096
    assert wl.k.shape[1] == math.ceil(1.1 * sum(math.ceil(n / 16) for n in lens))
    out = _run_decode(wl)
    assert out.dtype == (torch.float32 if kv == "f32" else torch.bfloat16)
    _check_decode_rows(wl, out, range(batch), FP32_ATOL if kv == "f32" else BF16_ATOL)


def test_cfg4_exact_bench_launch(bench):
    """The headline launch itself: 64 x 32768 tokens, fused write, the
    bench's split plan; sampled requests against the oracle."""
    from b200attn import _lib

    wl = bench.DecodeWorkload("cfg4", 0, _dev())
    assert wl.B == 64 and set(wl.lens) == {32768}
    lib = _lib.load()
    nbytes = lib.b200_paged_decode_workspace_size(64, 32, 128, wl.host["tables"].shape[1], 16,
                                                  _lib.DTYPE_BF16, 0)
    assert nbytes > 0  # the launch splits the contexts
    out = _run_decode(wl)
    _check_decode_rows(wl, out, (0, 21, 42, 63), BF16_ATOL)


def test_cfg4_strong_scaling_shards(bench):
    """Configuration 4's 64 requests sharded over 8 ranks: every shard's
    launch (8 requests) matches the oracle on a sampled request."""
    for rank in (0, 7):
        wl = bench.DecodeWorkload("cfg4", rank, _dev(), world=8, strong=True)
        assert wl.B == 8
        out = _run_decode(wl)
        _check_decode_rows(wl, out, (0, 7), BF16_ATOL)
        del wl, out
        torch.cuda.empty_cache()


@pytest.mark.parametrize("T", [64, 512])
def test_cfg5_batched_prefill_launch(bench, T):
    """Configuration 5: the bench's single batched launch over 16 sequences;
    every sequence against the float64 SDPA-v2 oracle."""
    wl = bench.PrefillWorkload(T, 0, _dev())
    assert len(wl.prefix) == 16 and all(p % 16 == 0 and 0 <= p <= 4032 for p in wl.prefix)
    wl.prepare()
    outs = wl.call()
    torch.cuda.synchronize()
    S = wl.pool.block_size
    for i, (p, table) in enumerate(zip(wl.prefix, wl.tables_h)):
        nb = math.ceil((p + T) / S)
        phys = table[:nb].to(_dev())
        ks, vs = wl.k[:, phys].cpu(), wl.v[:, phys].cpu()
        want = oracle.prefix_prefill_from_pool(wl.q_h[i].float(), ks, vs, list(range(nb)), p, 0,
                                               compute_dtype=torch.float64)
        err = (outs[i].double().cpu() - want).abs().max().item()
        assert err <= BF16_ATOL, f"sequence {i} (prefix {p}): max abs {err:.3e}"
