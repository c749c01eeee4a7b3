"""The C-ABI library loads and exports every function the header declares.

CPU-only: no entry point that launches device work is called here.
"""
from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "b200_paged_attn.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_api():
    names = declared_functions()
    for fn in ("b200_kv_scatter", "b200_paged_decode", "b200_chunked_prefill",
               "b200_chunked_prefill_batch", "b200_last_error"):
        assert fn in names


def test_library_exports_every_declared_symbol():
    from b200attn import _lib

    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from {_lib.LIB_PATH}"
    assert set(declared_functions()) <= set(_lib.SIGNATURES)
    assert lib.b200_abi_version() == 1
    assert lib.b200_built_arch() == 100


def test_ctypes_struct_sizes_match_c_layout():
    import ctypes
    from b200attn import _lib

    # Sizes computed from the C declarations on LP64 (8-byte pointers/int64,
    # 4-byte enums padded to 8 where the next field is 8-aligned).
    assert ctypes.sizeof(_lib.KVPool) == 64
    assert ctypes.sizeof(_lib.ScatterArgs) == 64 + 8 * 4 + 48 + 8 + 8 + 8 + 8 + 8
    assert ctypes.sizeof(_lib.PrefillBatchArgs) == 16
    assert ctypes.sizeof(_lib.QkvKvWriteArgs) == 64 + 10 * 8 + 8 + 8


def test_qkv_kv_write_rejects_bad_arguments_without_gpu():
    """Host validation of the fused QKV projection runs before any CUDA call."""
    from b200attn import _lib

    lib = _lib.load()

    def args(**kw):
        a = _lib.QkvKvWriteArgs()
        a.pool = _lib.KVPool(1 << 20, 2 << 20, 2, 8, 16, 4, 64, _lib.DTYPE_BF16)
        a.layer_idx, a.num_tokens, a.hidden = 1, 5, 256
        a.x, a.x_row_stride, a.weight = 3 << 20, 256, 4 << 20
        a.q_out, a.q_row_stride, a.slot_mapping = 5 << 20, 256, 6 << 20
        a.slot_stride, a.slot_dtype = 1, _lib.INDEX_I64
        for k, v in kw.items():
            setattr(a, k, v)
        return ctypes.byref(a)

    import ctypes

    bad = {
        "hidden not a multiple of 64": dict(hidden=96),
        "heads x head_dim != hidden": dict(hidden=192),
        "x rows not 16-byte aligned": dict(x_row_stride=260),
        "q rows overlap": dict(q_row_stride=128),
        "x misaligned": dict(x=(3 << 20) + 8),
        "null weight": dict(weight=None),
        "f32 pool": dict(pool=_lib.KVPool(1 << 20, 2 << 20, 2, 8, 16, 4, 64, _lib.DTYPE_F32)),
        "layer outside pool": dict(layer_idx=2),
        "bad slot dtype": dict(slot_dtype=7),
        "too many output tiles": dict(num_tokens=(1 << 30) - 1,
                                      pool=_lib.KVPool(1 << 20, 2 << 20, 2, 8, 16, 4096, 128,
                                                       _lib.DTYPE_BF16),
                                      hidden=1 << 19, x_row_stride=1 << 19, q_row_stride=1 << 19),
    }
    for why, kw in bad.items():
        rc = lib.b200_qkv_kv_write(args(**kw), None)
        assert rc in (_lib.ERR_INVALID_ARGUMENT, _lib.ERR_UNSUPPORTED), why
    assert lib.b200_qkv_kv_write(None, None) == _lib.ERR_INVALID_ARGUMENT
    k = ctypes.c_int32()
    assert lib.b200_qkv_kv_write_plan(5, 96, ctypes.byref(k), ctypes.byref(k),
                                      ctypes.byref(k)) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_qkv_kv_write_plan(5, 256, None, None, None) == _lib.ERR_INVALID_ARGUMENT
    # Zero tokens is a no-op that succeeds without touching the device.
    assert lib.b200_qkv_kv_write(args(num_tokens=0), None) == _lib.OK


def test_last_error_and_invalid_arguments_without_gpu():
    import ctypes
    from b200attn import _lib

    lib = _lib.load()
    # A null argument struct is rejected on the host before any CUDA call.
    assert lib.b200_paged_decode(None, None) == _lib.ERR_INVALID_ARGUMENT
    assert "null" in _lib.last_error(lib)
    args = _lib.DecodeArgs()  # all-zero pool: rejected as invalid, nothing launched
    assert lib.b200_paged_decode(ctypes.byref(args), None) == _lib.ERR_INVALID_ARGUMENT
    assert "KV pool" in _lib.last_error(lib)
    sargs = _lib.ScatterArgs()
    assert lib.b200_kv_scatter(ctypes.byref(sargs), None) == _lib.ERR_INVALID_ARGUMENT
    sargs.pool = _lib.KVPool(1 << 20, 2 << 20, 1, 4, 16, 2, 64, _lib.DTYPE_BF16)
    sargs.num_tokens = 1 << 31
    assert lib.b200_kv_scatter(ctypes.byref(sargs), None) == _lib.ERR_UNSUPPORTED
    assert "2^31" in _lib.last_error(lib)
    pargs = _lib.PrefillArgs()
    pargs.pool = _lib.KVPool(1 << 20, 2 << 20, 1, 4, 16, 2, 64, _lib.DTYPE_BF16)
    pargs.num_tokens, pargs.prefix_len = 1 << 24, 0
    assert lib.b200_chunked_prefill(ctypes.byref(pargs), None) == _lib.ERR_UNSUPPORTED
    pargs.num_tokens, pargs.prefix_len = 16, (1 << 31) - 8
    assert lib.b200_chunked_prefill(ctypes.byref(pargs), None) == _lib.ERR_UNSUPPORTED


def test_workspace_size_queries():
    from b200attn import _lib

    lib = _lib.load()
    small = lib.b200_paged_decode_workspace_size(1, 8, 32, 1, 16, _lib.DTYPE_F32, 0)
    assert small == 0  # one tile -> no split, no workspace
    big = lib.b200_paged_decode_workspace_size(2, 32, 128, 2048, 16, _lib.DTYPE_BF16, 0)
    assert big > 0


def test_decode_split_plan_fills_one_wave_when_ctas_stay_short():
    """bf16 decode at 32 heads of 128: the fewest splits that give about one wave
    of CTAs while a CTA covers <= 8192 tokens (32 x 1024 tokens: 256 CTAs, no
    split, no workspace); longer CTAs keep the two-wave rule (64 x 32768 tokens
    splits)."""
    from b200attn import _lib

    lib = _lib.load()
    bf16 = _lib.DTYPE_BF16
    assert lib.b200_paged_decode_workspace_size(32, 32, 128, 64, 16, bf16, 0) == 0
    assert lib.b200_paged_decode_workspace_size(1, 32, 128, 2048, 16, bf16, 0) > 0
    assert lib.b200_paged_decode_workspace_size(64, 32, 128, 2048, 16, bf16, 0) > 0
    # 8 x 4096 tokens takes 4 splits: its workspace holds 4 partial rows per head
    w8 = lib.b200_paged_decode_workspace_size(8, 32, 128, 256, 16, bf16, 0)
    w8_hint4 = lib.b200_paged_decode_workspace_size(8, 32, 128, 256, 16, bf16, 4)
    assert w8 == w8_hint4 > 0


def test_prefill_workspace_size_asks_for_a_key_split_only_when_the_launch_is_small():
    """bf16 prefill: a launch of fewer CTAs than about 85 % of the SMs asks for a
    workspace to split its keys over CTAs (>= 16 key tiles per split); a launch
    with enough CTAs, or too few keys, asks for none."""
    from b200attn import _lib

    lib = _lib.load()
    bf16 = _lib.DTYPE_BF16
    # one sequence, chunk 64 over a 4032-token prefix at 32 heads: 32 CTAs, 32 key tiles
    one = lib.b200_chunked_prefill_workspace_size(64, 32, 128, 256, 16, bf16)
    assert one > 0
    # chunk 2048 at 32 heads: 8 query pairs x 32 heads = 256 CTAs, no split
    assert lib.b200_chunked_prefill_workspace_size(2048, 32, 128, 640, 16, bf16) == 0
    # too few keys for two ranges of 16 tiles (700 tokens = 6 tiles of 128)
    assert lib.b200_chunked_prefill_workspace_size(1, 8, 128, 44, 16, bf16) == 0
    # more heads, fewer splits: the workspace never grows past 32 splits' rows
    few = lib.b200_chunked_prefill_workspace_size(1, 1, 128, 4096, 16, bf16)
    assert 0 < few <= 32 * 256 * 130 * 4 + 256


def test_ops_reject_cpu_tensors_loudly():
    from b200attn import paged_attention_batch_b200
    import cases

    c = cases.cfg1_case()
    with pytest.raises(ValueError, match="CUDA"):
        paged_attention_batch_b200(c.q, c.pool, c.block_tables, c.context_lengths, 0)


def test_selftest_rejects_bad_arguments_without_gpu():
    from b200attn import _lib

    lib = _lib.load()
    # Validation happens on the host before any CUDA call.
    assert lib.b200_selftest_bounded_wait(None, 1000, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_selftest_bounded_wait(8, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.b200_selftest_bounded_wait(8, 3_000_000_000, None) == _lib.ERR_INVALID_ARGUMENT


def test_ops_are_inference_only():
    """Inputs that require grad are refused while grad mode is on (as the
    reference's triton_v0 branch does, minivllm/attention.py:404-405), before
    any device check, so this runs on CPU."""
    from types import SimpleNamespace

    from b200attn import chunked_prefill_b200, kv_scatter_b200, paged_attention_batch_b200

    q = torch.zeros(2, 2, 8, requires_grad=True)
    pool = SimpleNamespace(k=torch.zeros(1, 2, 4, 2, 8), v=torch.zeros(1, 2, 4, 2, 8), block_size=4)
    with pytest.raises(RuntimeError, match="inference-only"):
        paged_attention_batch_b200(q, pool, torch.zeros(2, 1, dtype=torch.long),
                                   torch.ones(2, dtype=torch.long), 0)
    with pytest.raises(RuntimeError, match="inference-only"):
        chunked_prefill_b200(q, pool, [0], 0, 0)
    with pytest.raises(RuntimeError, match="inference-only"):
        kv_scatter_b200(q, q, pool, [0, 1], 0)
    with torch.inference_mode():  # no grad mode: the CUDA check comes next
        with pytest.raises(ValueError, match="CUDA"):
            paged_attention_batch_b200(torch.zeros(2, 2, 8), pool, torch.zeros(2, 1, dtype=torch.long),
                                       torch.ones(2, dtype=torch.long), 0)


@pytest.mark.parametrize("entry", ["b200_paged_decode", "b200_paged_decode_no_alloc",
                                   "b200_kv_scatter", "b200_chunked_prefill"])
def test_pool_row_limit_boundary_without_gpu(entry):
    """The kernels address pool rows (layer, block, slot) as 32-bit TMA
    coordinates and element offsets; the host rejects pools of 2^31 or more
    token rows before any CUDA call, and accepts 2^31 - 1 rows (the next
    check that fails then is an unrelated one: null q / k pointers)."""
    import ctypes
    from b200attn import _lib

    lib = _lib.load()
    fn = getattr(lib, entry)
    struct = {"b200_kv_scatter": _lib.ScatterArgs, "b200_chunked_prefill": _lib.PrefillArgs}.get(
        entry, _lib.DecodeArgs)
    for rows, over in (((1 << 31), True), ((1 << 31) - 16, False)):
        a = struct()
        # L * P * S rows with S = 16; the pointers are never dereferenced.
        a.pool = _lib.KVPool(1 << 20, 2 << 20, 1, rows // 16, 16, 2, 64, _lib.DTYPE_BF16)
        if struct is _lib.ScatterArgs:
            a.num_tokens = 1
        elif struct is _lib.PrefillArgs:
            a.num_tokens, a.block_table_len = 1, 1
        else:
            a.batch, a.table_width = 1, 1
        rc = fn(ctypes.byref(a), None)
        msg = _lib.last_error(lib)
        if over:
            assert rc == _lib.ERR_UNSUPPORTED and "2^31 token rows" in msg, (entry, msg)
        else:
            assert rc == _lib.ERR_INVALID_ARGUMENT and "2^31" not in msg, (entry, msg)
