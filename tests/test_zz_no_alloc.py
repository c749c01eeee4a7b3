"""b200_paged_decode_no_alloc: the decode entry point that allocates nothing.

Callers that may not allocate device memory (an engine that plans all of
its memory up front, a plugin that may only touch the buffers it is handed,
a step loop that must not call cudaMalloc) use this entry point; its split-K
scratch is a static device array inside the library.  This file checks,
through the C ABI, that two calls in a row give the same results as the
workspace-taking b200_paged_decode and with the float64 oracle, within the
tolerances of the other decode tests (also with a real split-K plan and
with the fused KV write), that a call needing more scratch than the array
holds is rejected, and that invalid arguments get the same error as from
b200_paged_decode.  It is named to be collected last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_ATOL = 2e-2


def _args(q, pool, tables, lens, out, max_splits=0, layer_idx=0):
    from b200attn import _lib, ops

    a = _lib.DecodeArgs()
    a.pool = ops._pool_struct(pool)
    a.layer_idx = layer_idx
    a.batch = q.shape[0]
    a.table_width = tables.shape[1]
    a.q = q.data_ptr()
    a.q_stride = ops._strides3(q)
    a.q_dtype = ops._DTYPES[q.dtype]
    a.out = out.data_ptr()
    a.out_stride = ops._strides3(out)
    a.out_dtype = ops._DTYPES[out.dtype]
    a.block_tables = tables.data_ptr()
    a.block_table_stride = (ctypes.c_int64 * 2)(*tables.stride())
    a.block_table_dtype = ops._INDEX[tables.dtype]
    a.context_lengths = lens.data_ptr()
    a.context_length_stride = lens.stride(0)
    a.context_length_dtype = ops._INDEX[lens.dtype]
    a.max_splits_hint = max_splits
    return a


def _fused_inputs(case, seed):
    """New-token K/V for each sequence, written at the slot of position ctx-1."""
    g = torch.Generator().manual_seed(seed)
    B, H, D = case.q.shape
    k_new = torch.randn((B, H, D), generator=g).to(case.pool.k.dtype)
    v_new = torch.randn((B, H, D), generator=g).to(case.pool.k.dtype)
    S = case.pool.block_size
    slots = [int(case.block_tables[b, (int(n) - 1) // S]) * S + (int(n) - 1) % S
             for b, n in enumerate(case.context_lengths)]
    return k_new, v_new, torch.tensor(slots, dtype=torch.int64)


@pytest.mark.parametrize("case,tol,splits,fused", [
    (cases.bf16_case(8, 32, 128, 16, 4096, 31), BF16_ATOL, 0, False),
    (cases.bf16_case(5, 32, 128, 16, 2500, 32), BF16_ATOL, 6, False),
    (cases.cfg1_case(), FP32_ATOL, 3, False),
    (cases.bf16_case(6, 32, 128, 16, 2000, 9), BF16_ATOL, 4, True),
], ids=["bf16_b8", "bf16_b5_splits6", "cfg1_fp32", "bf16_b6_fused_write"])
def test_no_alloc_matches_workspace_decode_twice(case, tol, splits, fused):
    """Two calls in a row through the C ABI: each must agree with the
    workspace-taking b200_paged_decode and with the float64 oracle (the
    reference's dense decode, after the KV write when it is fused)."""
    import oracle
    from b200attn import _lib, paged_attention_batch_b200

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    q = case.q.to(dev)
    tables = case.block_tables.to(dev)
    lens = case.context_lengths.to(dev)
    B, H, D = case.q.shape
    if splits > 1:
        # The hint really splits these contexts (split-K partials go through
        # the static scratch).
        assert lib.b200_paged_decode_workspace_size(B, H, D, tables.shape[1],
                                                    case.pool.block_size,
                                                    ops_dtype(case.pool.k.dtype), splits) > 0
    kp, vp = case.pool.k.clone(), case.pool.v.clone()
    fused_kw = {}
    if fused:
        k_new, v_new, slots = _fused_inputs(case, 77)
        oracle.kv_scatter(kp, vp, k_new, v_new, slots, case.layer_idx)
        fused_kw = {"k_new": k_new.to(dev), "v_new": v_new.to(dev), "slot_mapping": slots.to(dev)}
    want_oracle = oracle.paged_decode_dense(case.q, kp.float(), vp.float(), case.block_tables,
                                            case.context_lengths, case.layer_idx,
                                            compute_dtype=torch.float64).float()
    pool = case.pool.to(dev)
    with torch.inference_mode():
        want = paged_attention_batch_b200(q, pool, tables, lens, case.layer_idx,
                                          max_splits=splits, **fused_kw)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        pool = case.pool.to(dev)  # each call starts from the unwritten pool
        out = torch.full_like(want, float("nan"))
        a = _args(q, pool, tables, lens, out, splits, case.layer_idx)
        if fused:
            _fused_args(a, fused_kw)
        rc = lib.b200_paged_decode_no_alloc(ctypes.byref(a), stream)
        assert rc == 0, _lib.last_error(lib)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        err = (out.float() - want.float()).abs().max().item()
        assert err <= tol, f"call {call}: vs b200_paged_decode max abs {err:.3e}"
        err = (out.float().cpu() - want_oracle).abs().max().item()
        assert err <= tol, f"call {call}: vs oracle max abs {err:.3e}"
        if fused:
            # The written rows, and every other row, equal the reference's
            # index_put of k_new / v_new (bit for bit).
            assert cases.digest(pool.k.cpu(), pool.v.cpu()) == cases.digest(kp, vp)


def ops_dtype(dtype):
    from b200attn import ops
    return ops._POOL_DTYPES[dtype]


def _fused_args(a, kw):
    from b200attn import ops

    a.k_new = kw["k_new"].data_ptr()
    a.v_new = kw["v_new"].data_ptr()
    a.k_new_stride = ops._strides3(kw["k_new"])
    a.v_new_stride = ops._strides3(kw["v_new"])
    a.kv_new_dtype = ops._DTYPES[kw["k_new"].dtype]
    a.slot_mapping = kw["slot_mapping"].data_ptr()
    a.slot_stride = kw["slot_mapping"].stride(0)
    a.slot_dtype = ops._INDEX[kw["slot_mapping"].dtype]


def test_no_alloc_rejects_sizes_beyond_the_static_scratch():
    from b200attn import _lib

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    pool = cases.Pool(torch.zeros((1, 4, 16, 32, 128), dtype=torch.bfloat16, device=dev),
                      torch.zeros((1, 4, 16, 32, 128), dtype=torch.bfloat16, device=dev), 16)
    q = torch.zeros((64, 32, 128), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    tables = torch.zeros((64, 2048), dtype=torch.int64, device=dev)
    lens = torch.ones(64, dtype=torch.int64, device=dev)
    need = lib.b200_paged_decode_workspace_size(64, 32, 128, 2048, 16, _lib.DTYPE_BF16, 16)
    assert need > _lib.NO_ALLOC_SCRATCH_BYTES
    rc = lib.b200_paged_decode_no_alloc(ctypes.byref(_args(q, pool, tables, lens, out, 16)),
                                        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.ERR_UNSUPPORTED
    assert "static scratch" in _lib.last_error(lib)


def test_no_alloc_validates_arguments_first():
    """Invalid arguments are rejected with b200_paged_decode's own status and
    message, before any scratch-size arithmetic on them."""
    from b200attn import _lib

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    case = cases.cfg1_case()
    pool = case.pool.to(dev)
    q = case.q.to(dev)
    out = torch.empty_like(q)
    tables = case.block_tables.to(dev)
    lens = case.context_lengths.to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    bad = _args(q, pool, tables, lens, out, 0, layer_idx=5)  # past the pool's layers
    rc_ws = lib.b200_paged_decode(ctypes.byref(bad), stream)
    msg_ws = _lib.last_error(lib)
    rc = lib.b200_paged_decode_no_alloc(ctypes.byref(bad), stream)
    assert rc == rc_ws == _lib.ERR_INVALID_ARGUMENT
    assert _lib.last_error(lib) == msg_ws and "layer_idx" in msg_ws
    bad = _args(q, pool, tables, lens, out)
    bad.batch = 1 << 40  # garbage size: rejected by the checks, not by the scratch size
    rc = lib.b200_paged_decode_no_alloc(ctypes.byref(bad), stream)
    assert rc == _lib.ERR_UNSUPPORTED and "batch too large" in _lib.last_error(lib)
