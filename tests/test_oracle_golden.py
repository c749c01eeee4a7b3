"""Pins the CPU oracle against golden outputs of the reference itself.

The fixtures were produced by tests/golden/make_golden.py from the
reference's paged_attention_batch_online_v1, paged_attention_batch_reference,
dense_gold and forward_prefill_chunk (SDPA v1/v2 and per-token paths).
Inputs are rebuilt here from tests/golden/cases.py and verified by digest.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
DEC = np.load(GOLDEN / "decode_golden.npz")
DEC_META = json.loads((GOLDEN / "decode_golden.json").read_text())
PRE = np.load(GOLDEN / "prefill_golden.npz")
PRE_META = json.loads((GOLDEN / "prefill_golden.json").read_text())

# Same tolerance the reference uses between its two fp32 decode paths
# (tests/test_paged_attention.py:27, tests/test_triton_paged_decode.py:21).
ATOL = RTOL = 1e-5


def all_decode_cases() -> list[cases.DecodeCase]:
    out = list(cases.unit_pool_cases()) + [cases.nan_padding_case()]
    for bs, length in cases.RAGGED_CPU_SHAPES:
        out.append(cases.ragged_case(batch=3, length=length, heads=4, dim=8, block_size=bs))
    for bs, length, batch, dim in cases.RAGGED_GPU_SHAPES:
        out.append(cases.ragged_case(batch=batch, length=length, heads=8, dim=dim, block_size=bs))
    out.append(cases.ragged_case(batch=2, length=65, heads=4, dim=32, block_size=16, scale=8.0))
    for batch, length in cases.RAGGED_CORRECTNESS:
        out.append(cases.ragged_case(batch=batch, length=length, heads=8, dim=32, block_size=16,
                                     seed=20261030 + batch + length))
    out.append(cases.cfg1_case())
    return out


DECODE_CASES = all_decode_cases()


def test_every_fixture_has_a_case():
    assert {c.name for c in DECODE_CASES} == set(DEC_META)


@pytest.mark.parametrize("case", DECODE_CASES, ids=lambda c: c.name)
def test_decode_oracle_matches_reference(case):
    assert cases.case_digest(case) == DEC_META[case.name]["digest"], "input generator drifted"
    args = (case.q, case.pool.k, case.pool.v, case.block_tables, case.context_lengths,
            case.layer_idx)
    online = oracle.paged_decode_online(*args)
    dense = oracle.paged_decode_dense(*args)
    assert torch.isfinite(online).all() and torch.isfinite(dense).all()
    want_online = torch.from_numpy(DEC[f"{case.name}/online"])
    want_dense = torch.from_numpy(DEC[f"{case.name}/dense"])
    # The scale-8 large-logit case (outputs up to ~21) is as sensitive to the
    # fp32 summation order as the reference's own test allows for it
    # (tests/test_triton_paged_decode.py:66-71, atol 5e-4); torch's CPU
    # reductions take a different order on other host CPUs.
    atol = 5e-4 if "_sc8.0_" in case.name else ATOL
    torch.testing.assert_close(online, want_online, atol=atol, rtol=RTOL)
    torch.testing.assert_close(dense, want_dense, atol=atol, rtol=RTOL)
    key = f"{case.name}/reference"
    if key in DEC.files:
        torch.testing.assert_close(online, torch.from_numpy(DEC[key]), atol=atol, rtol=RTOL)


def test_unit_cases_online_equals_per_request_single():
    # paged_attention_online (the single-sequence path) on the same pools.
    for case in cases.unit_pool_cases():
        for b in range(case.q.shape[0]):
            table = [int(x) for x in case.block_tables[b] if int(x) >= 0]
            got = oracle.paged_decode_single(case.q[b], case.pool.k, case.pool.v, table,
                                             case.layer_idx, int(case.context_lengths[b]))
            want = torch.from_numpy(DEC[f"{case.name}/online"])[b]
            torch.testing.assert_close(got, want, atol=ATOL, rtol=RTOL)


def _prefill_case(name: str) -> cases.PrefillCase:
    m = PRE_META[name]
    return cases.prefill_case(m["prefix_len"], m["T"], m["H"], m["D"], m["S"], m["seed"])


@pytest.mark.parametrize("name", sorted(PRE_META))
def test_prefill_oracle_matches_reference(name):
    c = _prefill_case(name)
    m = PRE_META[name]
    assert cases.digest(c.q, c.k, c.v, c.pool.k, c.pool.v) == m["input_digest"]
    k_pool, v_pool = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(k_pool, v_pool, c.k, c.v, c.slots, c.layer_idx)
    assert cases.digest(k_pool, v_pool) == m["pool_after_digest"], "scatter differs from reference"
    fast = oracle.prefix_prefill(c.q, c.k, c.v, k_pool, v_pool, c.block_table, c.prefix_len,
                                 c.layer_idx)
    from_pool = oracle.prefix_prefill_from_pool(c.q, k_pool, v_pool, c.block_table,
                                                c.prefix_len, c.layer_idx)
    per_token = oracle.prefill_per_token(c.q, k_pool, v_pool, c.block_table, c.prefix_len,
                                         c.layer_idx)
    want_fast = torch.from_numpy(PRE[f"{name}/sdpa"])
    want_ref = torch.from_numpy(PRE[f"{name}/reference"])
    # The reference's own prefill parity tolerance (test_prefill_prefix_sdpa_v2.py:61-63).
    torch.testing.assert_close(fast, want_fast, atol=2e-5, rtol=2e-4)
    torch.testing.assert_close(from_pool, want_fast, atol=2e-5, rtol=2e-4)
    torch.testing.assert_close(per_token, want_ref, atol=2e-5, rtol=2e-4)


def test_planted_mistake_is_caught():
    # A perturbed query in an oracle run must break parity (the last query of
    # a chunk with a prefix attends to many keys, so its output depends on q).
    name = next(n for n in sorted(PRE_META) if PRE_META[n]["prefix_len"] > 8)
    c = _prefill_case(name)
    k_pool, v_pool = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(k_pool, v_pool, c.k, c.v, c.slots, c.layer_idx)
    bad_q = c.q.clone()
    bad_q[-1, 0, 0] += 1.0
    got = oracle.prefix_prefill(bad_q, c.k, c.v, k_pool, v_pool, c.block_table, c.prefix_len,
                                c.layer_idx)
    want = torch.from_numpy(PRE[f"{name}/sdpa"])
    assert not torch.allclose(got, want, atol=2e-5, rtol=2e-4)


QKV_META = json.loads((GOLDEN / "qkv_golden.json").read_text())
QKV = np.load(GOLDEN / "qkv_golden.npz")


def _qkv_written(c, kp, vp):
    C = kp.shape[3] * kp.shape[4]
    rows = torch.tensor(c.slots)
    return (kp[c.layer_idx].reshape(-1, C)[rows], vp[c.layer_idx].reshape(-1, C)[rows])


@pytest.mark.parametrize("name", sorted(QKV_META))
def test_qkv_oracle_matches_reference_projection_and_write(name):
    """The oracle's projection + KV write matches the reference's own
    KVCacheCausalSelfAttention (real qkv Linear, chunk(3), per-token
    write_layer loop; attention.py:177-208): the rows written at the slots
    agree within the reference's fp32 tolerance (the fixture's digest is
    bit-exact on the host that made it; fp32 matmul bits differ between host
    CPUs), and every other pool row keeps its NaN."""
    m = QKV_META[name]
    c = cases.qkv_case(m["T"], m["H"], m["D"], m["S"], m["seed"])
    assert c.name == name
    assert cases.digest(c.x, c.w, c.pool.k, c.pool.v) == m["input_digest"]
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    q = oracle.qkv_project_kv_write(c.x, c.w, kp, vp, c.slots, c.layer_idx)
    k_rows, v_rows = _qkv_written(c, kp, vp)
    torch.testing.assert_close(k_rows, torch.from_numpy(QKV[f"{name}/k_rows"]), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(v_rows, torch.from_numpy(QKV[f"{name}/v_rows"]), atol=ATOL, rtol=RTOL)
    written = torch.zeros(kp.shape[:3], dtype=torch.bool)
    for s_ in c.slots:
        written[c.layer_idx, s_ // m["S"], s_ % m["S"]] = True
    assert torch.isnan(kp[~written]).all() and torch.isnan(vp[~written]).all()
    assert q.shape == (m["T"], m["H"], m["D"])


def test_qkv_planted_mistake_is_caught():
    """Swapping the k and v thirds (a plausible split bug) is caught."""
    name = sorted(QKV_META)[0]
    m = QKV_META[name]
    c = cases.qkv_case(m["T"], m["H"], m["D"], m["S"], m["seed"])
    C = m["H"] * m["D"]
    w_swapped = torch.cat([c.w[:C], c.w[2 * C:], c.w[C:2 * C]])
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    oracle.qkv_project_kv_write(c.x, w_swapped, kp, vp, c.slots, c.layer_idx)
    k_rows, _ = _qkv_written(c, kp, vp)
    assert not torch.allclose(k_rows, torch.from_numpy(QKV[f"{name}/k_rows"]), atol=ATOL, rtol=RTOL)
