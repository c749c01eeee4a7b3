"""ctypes binding of libb200attn.so (the C ABI declared in include/b200_paged_attn.h).

The structures below mirror the C structs field by field; the library is
loaded lazily on first use and a missing or unloadable library raises
RuntimeError (there is no fallback implementation).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200attn.so"

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
INDEX_I32, INDEX_I64 = 0, 1

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4

DEV_BAD_BLOCK = 1
DEV_BAD_LENGTH = 2
DEV_BAD_SLOT = 4
DEV_WAIT_TIMEOUT = 8
DEV_SLOT_MISMATCH = 16

# Static split-K scratch of b200_paged_decode_no_alloc (B200_NO_ALLOC_SCRATCH_BYTES).
NO_ALLOC_SCRATCH_BYTES = 4 << 20

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


class KVPool(ctypes.Structure):
    _fields_ = [("k", _p), ("v", _p), ("num_layers", _i64), ("num_blocks", _i64),
                ("block_size", _i64), ("num_heads", _i64), ("head_dim", _i64),
                ("dtype", ctypes.c_int)]


class ScatterArgs(ctypes.Structure):
    _fields_ = [("pool", KVPool), ("layer_idx", _i64), ("num_tokens", _i64),
                ("k", _p), ("v", _p), ("k_stride", _i64 * 3), ("v_stride", _i64 * 3),
                ("kv_in_dtype", ctypes.c_int), ("slot_mapping", _p), ("slot_stride", _i64),
                ("slot_dtype", ctypes.c_int), ("status", _p)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("pool", KVPool), ("layer_idx", _i64), ("batch", _i64), ("table_width", _i64),
                ("q", _p), ("q_stride", _i64 * 3), ("q_dtype", ctypes.c_int),
                ("out", _p), ("out_stride", _i64 * 3), ("out_dtype", ctypes.c_int),
                ("block_tables", _p), ("block_table_stride", _i64 * 2),
                ("block_table_dtype", ctypes.c_int),
                ("context_lengths", _p), ("context_length_stride", _i64),
                ("context_length_dtype", ctypes.c_int), ("ctx_base", _i64),
                ("k_new", _p), ("v_new", _p), ("k_new_stride", _i64 * 3),
                ("v_new_stride", _i64 * 3), ("kv_new_dtype", ctypes.c_int),
                ("slot_mapping", _p), ("slot_stride", _i64), ("slot_dtype", ctypes.c_int),
                ("workspace", _p), ("workspace_bytes", ctypes.c_size_t), ("status", _p),
                ("max_splits_hint", ctypes.c_int32)]


class PrefillArgs(ctypes.Structure):
    _fields_ = [("pool", KVPool), ("layer_idx", _i64), ("num_tokens", _i64),
                ("prefix_len", _i64), ("q", _p), ("q_stride", _i64 * 3),
                ("q_dtype", ctypes.c_int), ("out", _p), ("out_stride", _i64 * 3),
                ("out_dtype", ctypes.c_int), ("block_table", _p), ("block_table_len", _i64),
                ("block_table_stride", _i64), ("block_table_dtype", ctypes.c_int),
                ("workspace", _p), ("workspace_bytes", ctypes.c_size_t), ("status", _p)]


class QkvKvWriteArgs(ctypes.Structure):
    _fields_ = [("pool", KVPool), ("layer_idx", _i64), ("num_tokens", _i64), ("hidden", _i64),
                ("x", _p), ("x_row_stride", _i64), ("weight", _p), ("q_out", _p),
                ("q_row_stride", _i64), ("slot_mapping", _p), ("slot_stride", _i64),
                ("slot_dtype", ctypes.c_int), ("status", _p)]


class PrefillBatchArgs(ctypes.Structure):
    _fields_ = [("num_seqs", _i64), ("seqs", ctypes.POINTER(PrefillArgs))]


# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "b200_kv_scatter": (ctypes.c_int, [ctypes.POINTER(ScatterArgs), _p]),
    "b200_paged_decode": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), _p]),
    "b200_chunked_prefill": (ctypes.c_int, [ctypes.POINTER(PrefillArgs), _p]),
    "b200_chunked_prefill_batch": (ctypes.c_int, [ctypes.POINTER(PrefillBatchArgs), _p]),
    "b200_paged_decode_no_alloc": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), _p]),
    "b200_qkv_kv_write": (ctypes.c_int, [ctypes.POINTER(QkvKvWriteArgs), _p]),
    "b200_qkv_kv_write_plan": (ctypes.c_int, [_i64, _i64, ctypes.POINTER(ctypes.c_int32),
                                              ctypes.POINTER(ctypes.c_int32),
                                              ctypes.POINTER(ctypes.c_int32)]),
    "b200_paged_decode_workspace_size": (
        ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int32]),
    "b200_chunked_prefill_workspace_size": (
        ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, ctypes.c_int]),
    "b200_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "b200_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_void_p, _i64, _p]),
    "b200_abi_version": (ctypes.c_int, []),
    "b200_built_arch": (ctypes.c_int, []),
}

_lib = None
_lock = threading.Lock()


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads (once) and returns the native library; RuntimeError if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"b200attn native library not found at {p}; build it with "
                "`python mini-gpt-inference_b200/csrc/build.py` (or __graft_entry__.build())")
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:  # pragma: no cover - depends on the host
            raise RuntimeError(f"cannot load b200attn native library {p}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.b200_abi_version() != 1:
            raise RuntimeError("b200attn native library ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    lib = lib or load()
    buf = ctypes.create_string_buffer(1024)
    lib.b200_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    """Maps a C status to the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)
