"""Decode kernel parity on the GPU, through the C ABI (ctypes).

Tolerances: fp32 KV max abs error <= 1e-4 (TF32 never used), bf16 KV
<= 2e-2 against the fp32 oracle on the upcast pool.  Inputs are the seeded
fixtures of tests/golden/cases.py; expected values are the reference's own
outputs stored in tests/golden/decode_golden.npz and the CPU oracle.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
FP32_ATOL = 1e-4
BF16_ATOL = 2e-2


def _dev():
    return torch.device("cuda", 0)


def _on(case: cases.DecodeCase, index_dtype=torch.int64):
    d = _dev()
    return (case.q.to(d), case.pool.to(d), case.block_tables.to(d, index_dtype),
            case.context_lengths.to(d, index_dtype))


def _decode(q, pool, tables, lens, layer, **kw):
    from b200attn import paged_attention_batch_b200

    with torch.inference_mode():
        out = paged_attention_batch_b200(q, pool, tables, lens, layer, **kw)
    torch.cuda.synchronize()
    return out


def _fixture_cases():
    from test_oracle_golden import DECODE_CASES
    return DECODE_CASES


@pytest.mark.parametrize("case", _fixture_cases(), ids=lambda c: c.name)
@pytest.mark.parametrize("splits", [0, 3])
def test_decode_matches_reference_golden(case, splits):
    golden = np.load(GOLDEN / "decode_golden.npz")
    q, pool, tables, lens = _on(case)
    status = torch.zeros(1, dtype=torch.int32, device=_dev())
    out = _decode(q, pool, tables, lens, case.layer_idx, status=status, max_splits=splits)
    assert int(status.item()) == 0
    got = out.cpu()
    assert torch.isfinite(got).all()
    # The scale-8 large-logit case uses the reference's own tolerance for it
    # (tests/test_triton_paged_decode.py:66-71, atol 5e-4): outputs reach ~21
    # and the reference's two fp32 paths already differ by 1.3e-4 there.
    tol = 5e-4 if "_sc8.0_" in case.name else FP32_ATOL
    for key in ("online", "dense"):
        want = torch.from_numpy(golden[f"{case.name}/{key}"])
        err = (got - want).abs().max().item()
        assert err <= tol, f"{case.name} vs reference {key}: max abs {err:.3e}"


def test_workspace_reuse_across_shapes():
    # A split-K call of one shape leaves partials where a call of another
    # shape keeps its counters; the second call must still be exact.
    big = cases.bf16_case(40, 32, 128, 16, 3000, 21)
    small = cases.ragged_case(batch=4, length=129, heads=8, dim=32, seed=20261163)
    for _ in range(2):
        for case, tol in ((big, BF16_ATOL), (small, FP32_ATOL)):
            q, pool, tables, lens = _on(case)
            out = _decode(q, pool, tables, lens, case.layer_idx)
            want = oracle.paged_decode_dense(case.q, case.pool.k.float(), case.pool.v.float(),
                                             case.block_tables, case.context_lengths,
                                             case.layer_idx, compute_dtype=torch.float64).float()
            assert (out.cpu() - want).abs().max().item() <= tol


@pytest.mark.parametrize("case", [cases.cfg1_case(),
                                  cases.ragged_case(batch=4, length=257, heads=8, dim=64,
                                                    block_size=32)],
                         ids=lambda c: c.name)
def test_decode_int32_metadata_and_bf16_query(case):
    q, pool, tables, lens = _on(case, torch.int32)
    want = oracle.paged_decode_dense(case.q, case.pool.k, case.pool.v, case.block_tables,
                                     case.context_lengths, case.layer_idx)
    out = _decode(q, pool, tables, lens, case.layer_idx)
    assert (out.cpu() - want).abs().max().item() <= FP32_ATOL
    # bf16 q/out over the same fp32 pool: q rounding dominates the error.
    out16 = _decode(q.to(torch.bfloat16), pool, tables, lens, case.layer_idx)
    assert out16.dtype == torch.bfloat16
    want16 = oracle.paged_decode_dense(case.q.to(torch.bfloat16).float(), case.pool.k,
                                       case.pool.v, case.block_tables, case.context_lengths,
                                       case.layer_idx)
    assert (out16.float().cpu() - want16).abs().max().item() <= BF16_ATOL


@pytest.mark.parametrize("batch,max_len,seed", [(1, 1, 1), (3, 40, 2), (8, 700, 3),
                                                (16, 4096, 4), (33, 300, 5)])
@pytest.mark.parametrize("splits", [0, 1, 5])
def test_decode_bf16_kv_ragged(batch, max_len, seed, splits):
    case = cases.bf16_case(batch, 32, 128, 16, max_len, seed)
    q, pool, tables, lens = _on(case)
    want = oracle.paged_decode_dense(case.q, case.pool.k.float(), case.pool.v.float(),
                                     case.block_tables, case.context_lengths, 0,
                                     compute_dtype=torch.float64).float()
    out = _decode(q, pool, tables, lens, 0, max_splits=splits)
    err = (out.cpu() - want).abs().max().item()
    assert err <= BF16_ATOL, f"max abs {err:.3e}"


@pytest.mark.parametrize("dim,heads,bs", [(64, 8, 16), (32, 6, 8), (8, 2, 4), (16, 3, 32),
                                          (128, 5, 64)])
def test_decode_bf16_kv_shapes(dim, heads, bs):
    case = cases.bf16_case(5, heads, dim, bs, 300, 77 + dim)
    q, pool, tables, lens = _on(case)
    want = oracle.paged_decode_dense(case.q, case.pool.k.float(), case.pool.v.float(),
                                     case.block_tables, case.context_lengths, 0,
                                     compute_dtype=torch.float64).float()
    out = _decode(q, pool, tables, lens, 0)
    assert (out.cpu() - want).abs().max().item() <= BF16_ATOL


def _fused_inputs(case: cases.DecodeCase, dtype, seed):
    """New token K/V for each sequence, written at the slot of position ctx-1."""
    g = torch.Generator().manual_seed(seed)
    B, H, D = case.q.shape
    k_new = torch.randn((B, H, D), generator=g).to(dtype)
    v_new = torch.randn((B, H, D), generator=g).to(dtype)
    S = case.pool.block_size
    slots = []
    for b in range(B):
        pos = int(case.context_lengths[b]) - 1
        slots.append(int(case.block_tables[b, pos // S]) * S + pos % S)
    return k_new, v_new, torch.tensor(slots, dtype=torch.int64)


@pytest.mark.parametrize("case", [cases.cfg1_case(),
                                  cases.ragged_case(batch=4, length=129, heads=8, dim=32),
                                  cases.nan_padding_case(),
                                  cases.bf16_case(6, 32, 128, 16, 2000, 9)],
                         ids=lambda c: c.name)
@pytest.mark.parametrize("splits", [0, 4])
def test_fused_kv_write_then_attend(case, splits):
    k_new, v_new, slots = _fused_inputs(case, torch.float32, 123)
    # Oracle: scatter first (attention.py:370-392), then attend.
    kp, vp = case.pool.k.clone(), case.pool.v.clone()
    oracle.kv_scatter(kp, vp, k_new.to(kp.dtype), v_new.to(kp.dtype), slots, case.layer_idx)
    want = oracle.paged_decode_dense(case.q, kp.float(), vp.float(), case.block_tables,
                                     case.context_lengths, case.layer_idx,
                                     compute_dtype=torch.float64).float()
    q, pool, tables, lens = _on(case)
    d = _dev()
    status = torch.zeros(1, dtype=torch.int32, device=d)
    out = _decode(q, pool, tables, lens, case.layer_idx, k_new=k_new.to(d), v_new=v_new.to(d),
                  slot_mapping=slots.to(d), status=status, max_splits=splits)
    assert int(status.item()) == 0
    tol = FP32_ATOL if case.pool.k.dtype == torch.float32 else BF16_ATOL
    assert (out.cpu() - want).abs().max().item() <= tol
    # The written rows are bit-identical to the scatter (round-to-nearest-even).
    assert cases.digest(pool.k.cpu(), pool.v.cpu()) == cases.digest(kp, vp)


def test_device_status_reports_bad_metadata():
    from b200attn import _lib

    case = cases.cfg1_case()
    q, pool, tables, lens = _on(case)
    d = _dev()
    status = torch.zeros(1, dtype=torch.int32, device=d)
    bad_tables = tables.clone()
    bad_tables[1, 3] = pool.k.shape[1] + 5  # physical id past the pool: skipped, flagged
    _decode(q, pool, bad_tables, lens, 0, status=status)
    assert int(status.item()) & _lib.DEV_BAD_BLOCK
    status.zero_()
    bad_lens = lens.clone()
    bad_lens[0] = 0
    bad_lens[2] = tables.shape[1] * case.pool.block_size + 1
    out = _decode(q, pool, tables, bad_lens, 0, status=status)
    assert int(status.item()) & _lib.DEV_BAD_LENGTH
    assert torch.equal(out[0].cpu(), torch.zeros_like(out[0].cpu()))
    # Rows with valid metadata are unaffected.
    want = oracle.paged_decode_dense(case.q[[1, 3]], case.pool.k, case.pool.v,
                                     case.block_tables[[1, 3]], case.context_lengths[[1, 3]], 0)
    assert (out[[1, 3]].cpu() - want).abs().max().item() <= FP32_ATOL
    # A fused write whose slot is not the last context position is flagged.
    status.zero_()
    k_new, v_new, slots = _fused_inputs(case, torch.float32, 5)
    slots[0] += 1
    _decode(q, pool, tables, lens, 0, k_new=k_new.to(d), v_new=v_new.to(d),
            slot_mapping=slots.to(d), status=status)
    assert int(status.item()) & _lib.DEV_SLOT_MISMATCH


def test_host_validation_raises_like_the_reference():
    case = cases.cfg1_case()
    q, pool, tables, lens = _on(case)
    with pytest.raises(ValueError, match="layer_idx"):
        _decode(q, pool, tables, lens, 3)
    with pytest.raises(ValueError, match=r"\[B,H,D\]"):
        _decode(q[0], pool, tables, lens, 0)
    with pytest.raises(ValueError, match="block_tables"):
        _decode(q, pool, tables[:2], lens, 0)
    with pytest.raises(ValueError, match="integer"):
        _decode(q, pool, tables.float(), lens, 0)


def test_large_context_split_k_sampled():
    """Long contexts (many splits): exact check on a sampled subset of rows."""
    d = _dev()
    g = torch.Generator(device=d).manual_seed(7)
    B, H, D, S = 6, 32, 128, 16
    lens = torch.tensor([32768, 1, 17, 9000, 16384, 4095])
    counts = [math.ceil(int(n) / S) for n in lens]
    P = sum(counts) + 3
    k = torch.randn((1, P, S, H, D), generator=g, device=d).to(torch.bfloat16)
    v = torch.randn((1, P, S, H, D), generator=g, device=d).to(torch.bfloat16)
    perm = torch.randperm(P, generator=g, device=d).cpu()
    tables = torch.full((B, max(counts)), -1, dtype=torch.int64)
    nxt = 0
    for b, c in enumerate(counts):
        tables[b, :c] = perm[nxt:nxt + c]
        nxt += c
    q = torch.randn((B, H, D), generator=g, device=d)
    pool = cases.Pool(k, v, S)
    out = _decode(q, pool, tables.to(d), lens.to(d), 0)
    for b in (0, 1, 3):
        phys = tables[b, :counts[b]]
        sub = cases.Pool(k[:, phys.to(d)].cpu(), v[:, phys.to(d)].cpu(), S)
        want = oracle.paged_decode_dense(q[b:b + 1].cpu(), sub.k.float(), sub.v.float(),
                                         torch.arange(counts[b])[None], lens[b:b + 1], 0,
                                         compute_dtype=torch.float64).float()
        assert (out[b:b + 1].cpu() - want).abs().max().item() <= BF16_ATOL


def test_very_long_context_split_k():
    """A 256k-token context (the split-K plan at its 64-split cap, a 16384-wide
    table) and a 100k one, bf16 KV, checked against the float64 oracle on
    each sequence's compacted sub-pool."""
    d = _dev()
    g = torch.Generator(device=d).manual_seed(11)
    B, H, D, S = 2, 2, 128, 16
    lens = torch.tensor([262144, 100000])
    counts = [math.ceil(int(n) / S) for n in lens]
    P = sum(counts) + 5
    k = torch.randn((1, P, S, H, D), generator=g, device=d).to(torch.bfloat16)
    v = torch.randn((1, P, S, H, D), generator=g, device=d).to(torch.bfloat16)
    perm = torch.randperm(P, generator=g, device=d).cpu()
    tables = torch.full((B, max(counts)), -1, dtype=torch.int64)
    nxt = 0
    for b, c in enumerate(counts):
        tables[b, :c] = perm[nxt:nxt + c]
        nxt += c
    q = torch.randn((B, H, D), generator=g, device=d)
    pool = cases.Pool(k, v, S)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    out = _decode(q, pool, tables.to(d), lens.to(d), 0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for b in range(B):
        phys = tables[b, :counts[b]].to(d)
        want = oracle.paged_decode_dense(q[b:b + 1].cpu(), k[:, phys].cpu().float(),
                                         v[:, phys].cpu().float(), torch.arange(counts[b])[None],
                                         lens[b:b + 1], 0, compute_dtype=torch.float64).float()
        assert (out[b:b + 1].cpu() - want).abs().max().item() <= BF16_ATOL
