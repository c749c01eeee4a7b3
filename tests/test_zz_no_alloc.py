"""b200_paged_decode_no_alloc: the decode entry point that allocates nothing.

Callers that may not allocate device memory (an engine that plans all of
its memory up front, a plugin that may only touch the buffers it is handed,
a step loop that must not call cudaMalloc) use this entry point; its split-K
scratch is a static device array inside the library.  This file checks,
through the C ABI, that two calls in a row give the same results as the
workspace-taking b200_paged_decode, within the tolerances of the other
decode tests, and that a call needing more scratch than the array holds is
rejected.  It is named to be collected last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

FP32_ATOL = 1e-4
BF16_ATOL = 2e-2


def _args(q, pool, tables, lens, out, max_splits=0):
    from b200attn import _lib, ops

    a = _lib.DecodeArgs()
    a.pool = ops._pool_struct(pool)
    a.layer_idx = 0
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


@pytest.mark.parametrize("case,tol,splits", [
    (cases.bf16_case(8, 32, 128, 16, 4096, 31), BF16_ATOL, 0),
    (cases.bf16_case(5, 32, 128, 16, 2500, 32), BF16_ATOL, 6),
    (cases.cfg1_case(), FP32_ATOL, 3),
], ids=["bf16_b8", "bf16_b5_splits6", "cfg1_fp32"])
def test_no_alloc_matches_workspace_decode_twice(case, tol, splits):
    from b200attn import _lib, paged_attention_batch_b200

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    q = case.q.to(dev)
    pool = case.pool.to(dev)
    tables = case.block_tables.to(dev)
    lens = case.context_lengths.to(dev)
    with torch.inference_mode():
        want = paged_attention_batch_b200(q, pool, tables, lens, 0, max_splits=splits)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(2):
        out = torch.full_like(want, float("nan"))
        rc = lib.b200_paged_decode_no_alloc(ctypes.byref(_args(q, pool, tables, lens, out, splits)),
                                            stream)
        assert rc == 0, _lib.last_error(lib)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        err = (out.float() - want.float()).abs().max().item()
        assert err <= tol, f"max abs {err:.3e}"


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
