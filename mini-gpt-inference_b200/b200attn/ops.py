"""Reference-facing ops of the sm_100a paged-attention backend.

These are drop-ins for the attention backends of minivllm
(zyyh-ops/mini-gpt-inference):

* :func:`paged_attention_batch_b200` has the signature and error behaviour of
  ``paged_attention_batch_triton_v0`` (minivllm/triton_paged_decode.py:102-155)
  and the semantics of ``paged_attention_batch_online_v1``
  (minivllm/paged_attention_batch.py:121-278), optionally fused with the
  decode KV write of minivllm/attention.py:370-392.
* :func:`kv_scatter_b200` replaces the KV writes of attention.py:370-392 and
  the per-token ``KVBlockPool.write_layer`` loop of attention.py:193-208.
* :func:`qkv_kv_write_b200` is the attention's QKV projection (the
  bias-free ``qkv`` Linear, attention.py:79-83) with the KV write of
  attention.py:193-208 / :370-392 in the GEMM epilogue: it returns q and
  leaves k and v in the pool.
* :func:`chunked_prefill_b200` replaces the prefill attention branches of
  ``forward_prefill_chunk`` (attention.py:215-299): first-chunk SDPA, the
  prefix-aware SDPA v2 and the per-token reference.

All ops run only through libb200attn.so on CUDA tensors; there is no CPU or
library fallback (a CPU tensor raises ValueError, a missing library raises
RuntimeError), matching tests/test_decode_backend_integration.py:67-76 of the
reference ("never silently falls back").
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
           torch.float16: _lib.DTYPE_F16}
_POOL_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}
_INDEX = {torch.int32: _lib.INDEX_I32, torch.int64: _lib.INDEX_I64}


def is_available() -> bool:
    """True when the native library loads and a CUDA device is visible."""
    try:
        _lib.load()
    except RuntimeError:
        return False
    return torch.cuda.is_available()


def _inference_only(*tensors) -> None:
    """The ops have no backward: like the reference's triton_v0 branch
    (minivllm/attention.py:404-405) they refuse inputs that require grad
    while grad mode is on."""
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise RuntimeError("the b200 backend is inference-only; run under torch.inference_mode()")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _pool_struct(pool) -> _lib.KVPool:
    k, v = pool.k, pool.v
    if k.ndim != 5 or v.shape != k.shape:
        raise ValueError("KV tensors must have matching [L,P,S,H,D] shape")
    if k.dtype not in _POOL_DTYPES or v.dtype != k.dtype:
        raise ValueError("KV pool dtype must be float32 or bfloat16")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("KV pool tensors must be contiguous [L,P,S,H,D]")
    L, P, S, H, D = k.shape
    if S != pool.block_size:
        raise ValueError("pool.block_size does not match the KV tensor shape")
    return _lib.KVPool(k.data_ptr(), v.data_ptr(), L, P, S, H, D, _POOL_DTYPES[k.dtype])


def _strides3(t: torch.Tensor):
    return (ctypes.c_int64 * 3)(*t.stride())


class _Workspace:
    """Per (device, stream) split-K scratch, grown on demand.

    Its contents need not be initialised: every decode launch clears its
    split counters on the stream first.
    """

    def __init__(self):
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
        if nbytes == 0:
            return None
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WORKSPACE = _Workspace()


class PreparedCall:
    """One op with its C argument struct built once (``prepare=True``).

    Calling it launches the op on the device's current stream and returns
    the op's result tensor(s).  It keeps every tensor the struct points to
    alive and owns a private split-K workspace, so repeated calls cost one
    ctypes call each; calls of one PreparedCall must not overlap on the GPU.
    """

    def __init__(self, fn, args, device: torch.device, result, what: str, keep=()):
        self._fn, self._args, self._device = fn, args, device
        self._result, self._what, self._keep = result, what, keep
        self._ref = ctypes.byref(args)

    def __call__(self):
        _lib.check(self._fn(self._ref, _stream_ptr(self._device)), self._what)
        return self._result


def _workspace(device: torch.device, stream: int, nbytes: int, private: bool):
    if private:
        return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device) if nbytes else None
    return _WORKSPACE.get(device, stream, nbytes)


def _index_tensor(x, device: torch.device, name: str) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        if x.dtype not in _INDEX:
            raise ValueError(f"{name} must contain integer indices")
        if x.device != device:
            raise ValueError("all inputs must reside on same CUDA device")
        return x
    return torch.tensor(list(x), dtype=torch.int64).pin_memory().to(device, non_blocking=True)


def paged_attention_batch_b200(q: torch.Tensor, pool, block_tables: torch.Tensor,
                               context_lengths: torch.Tensor, layer_idx: int, *,
                               k_new: torch.Tensor | None = None,
                               v_new: torch.Tensor | None = None,
                               slot_mapping: torch.Tensor | None = None,
                               status: torch.Tensor | None = None,
                               out: torch.Tensor | None = None,
                               max_splits: int = 0, prepare: bool = False):
    """One batched paged decode-attention launch (optionally fused KV write).

    q: [B, H, D] (any strides); pool.k / pool.v: contiguous [L, P, S, H, D];
    block_tables: [B, M] int32/int64 with -1 only in the unused tail;
    context_lengths: [B] (>= 1, including the token being decoded).
    When k_new / v_new ([B, H, D]) and slot_mapping ([B]) are given, they are
    written into the pool first (the caller must then NOT write them itself).
    Returns a fresh [B, H, D] tensor of q.dtype (or fills ``out``); with
    prepare=True returns a PreparedCall that launches it.
    """
    _inference_only(q, k_new, v_new)
    lib = _lib.load()
    if not q.is_cuda:
        raise ValueError("CUDA q required for the b200 backend")
    if q.ndim != 3:
        raise ValueError("q must have shape [B,H,D]")
    b, h, d = q.shape
    if b == 0 or h == 0 or d == 0:
        raise ValueError("q dimensions must be nonzero")
    if q.dtype not in _DTYPES:
        raise ValueError("q must be float32, bfloat16 or float16")
    pstruct = _pool_struct(pool)
    if pool.k.shape[2:] != (pool.block_size, h, d):
        raise ValueError("KV head dimensions or block size do not match q")
    if block_tables.ndim != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must have shape [B,M]")
    if context_lengths.shape != (b,):
        raise ValueError("context_lengths must have shape [B]")
    if block_tables.dtype not in _INDEX:
        raise ValueError("block_tables must contain integer indices")
    if context_lengths.dtype not in _INDEX:
        raise ValueError("context_lengths must be integer")
    if not (0 <= layer_idx < pool.k.shape[0]):
        raise ValueError("layer_idx outside KV pool")
    dev = q.device
    if any(x.device != dev for x in (pool.k, pool.v, block_tables, context_lengths)):
        raise ValueError("all inputs must reside on same CUDA device")
    if block_tables.shape[1] < 1:
        raise ValueError("block_tables need at least one block column")
    fused = (k_new is not None, v_new is not None, slot_mapping is not None)
    if any(fused) and not all(fused):
        raise ValueError("k_new, v_new and slot_mapping must be given together")
    args = _lib.DecodeArgs()
    args.pool = pstruct
    args.layer_idx = layer_idx
    args.batch = b
    args.table_width = block_tables.shape[1]
    args.q = q.data_ptr()
    args.q_stride = _strides3(q)
    args.q_dtype = _DTYPES[q.dtype]
    if out is None:
        out = torch.empty((b, h, d), dtype=q.dtype, device=dev)
    elif out.shape != (b, h, d) or out.dtype not in _DTYPES or out.device != dev:
        raise ValueError("out must be a [B,H,D] tensor on the q device")
    args.out = out.data_ptr()
    args.out_stride = _strides3(out)
    args.out_dtype = _DTYPES[out.dtype]
    args.block_tables = block_tables.data_ptr()
    args.block_table_stride = (ctypes.c_int64 * 2)(*block_tables.stride())
    args.block_table_dtype = _INDEX[block_tables.dtype]
    args.context_lengths = context_lengths.data_ptr()
    args.context_length_stride = context_lengths.stride(0)
    args.context_length_dtype = _INDEX[context_lengths.dtype]
    if all(fused):
        for t in (k_new, v_new):
            if t.shape != (b, h, d) or t.device != dev or t.dtype not in _DTYPES:
                raise ValueError("k_new/v_new must be [B,H,D] CUDA tensors")
        if k_new.dtype != v_new.dtype:
            raise ValueError("k_new and v_new must share a dtype")
        if slot_mapping.shape != (b,) or slot_mapping.dtype not in _INDEX or slot_mapping.device != dev:
            raise ValueError("slot_mapping must be a [B] integer CUDA tensor")
        args.k_new = k_new.data_ptr()
        args.v_new = v_new.data_ptr()
        args.k_new_stride = _strides3(k_new)
        args.v_new_stride = _strides3(v_new)
        args.kv_new_dtype = _DTYPES[k_new.dtype]
        args.slot_mapping = slot_mapping.data_ptr()
        args.slot_stride = slot_mapping.stride(0)
        args.slot_dtype = _INDEX[slot_mapping.dtype]
    stream = _stream_ptr(dev)
    nbytes = lib.b200_paged_decode_workspace_size(
        b, h, d, block_tables.shape[1], pool.block_size, pstruct.dtype, max_splits)
    ws = _workspace(dev, stream, nbytes, prepare)
    if ws is not None:
        args.workspace = ws.data_ptr()
        args.workspace_bytes = ws.numel()
    args.max_splits_hint = max_splits
    if status is not None:
        args.status = status.data_ptr()
    call = PreparedCall(lib.b200_paged_decode, args, dev, out, "paged decode",
                        (q, pool.k, pool.v, block_tables, context_lengths, k_new, v_new,
                         slot_mapping, status, ws, out))
    return call if prepare else call()


def kv_scatter_b200(k: torch.Tensor, v: torch.Tensor, pool, slot_mapping,
                    layer_idx: int, *, status: torch.Tensor | None = None,
                    prepare: bool = False):
    """pool[layer, slot // S, slot % S] = k / v for each of the N tokens.

    k, v: [N, H, D] (any strides, any float dtype; converted to the pool's);
    slot_mapping: [N] integer CUDA tensor or a host sequence of ints.
    """
    _inference_only(k, v)
    lib = _lib.load()
    if not k.is_cuda:
        raise ValueError("CUDA k/v required for the b200 backend")
    if k.ndim != 3 or v.shape != k.shape:
        raise ValueError("k and v must have matching shape [N,H,D]")
    if k.dtype not in _DTYPES or v.dtype != k.dtype:
        raise ValueError("k/v must share a float dtype")
    pstruct = _pool_struct(pool)
    n, h, d = k.shape
    if pool.k.shape[3:] != (h, d):
        raise ValueError("k/v head dimensions do not match the KV pool")
    if not (0 <= layer_idx < pool.k.shape[0]):
        raise ValueError("layer_idx outside KV pool")
    dev = k.device
    if any(x.device != dev for x in (v, pool.k, pool.v)):
        raise ValueError("all inputs must reside on same CUDA device")
    slots = _index_tensor(slot_mapping, dev, "slot_mapping")
    if slots.shape != (n,):
        raise ValueError("slot_mapping must have shape [N]")
    args = _lib.ScatterArgs()
    args.pool = pstruct
    args.layer_idx = layer_idx
    args.num_tokens = n
    args.k = k.data_ptr()
    args.v = v.data_ptr()
    args.k_stride = _strides3(k)
    args.v_stride = _strides3(v)
    args.kv_in_dtype = _DTYPES[k.dtype]
    args.slot_mapping = slots.data_ptr()
    args.slot_stride = slots.stride(0) if n > 0 else 1
    args.slot_dtype = _INDEX[slots.dtype]
    if status is not None:
        args.status = status.data_ptr()
    call = PreparedCall(lib.b200_kv_scatter, args, dev, None, "kv scatter",
                        (k, v, pool.k, pool.v, slots, status))
    return call if prepare else call()


def qkv_kv_write_b200(x: torch.Tensor, weight: torch.Tensor, pool, slot_mapping,
                      layer_idx: int, *, q_out: torch.Tensor | None = None,
                      status: torch.Tensor | None = None, prepare: bool = False):
    """q = (x W^T)[:, :C] as [T, H, D]; k and v go straight into the pool.

    Same result as the reference's ``q, k, v = self.qkv(x).chunk(3, -1)``
    followed by the KV write at ``slot_mapping`` (attention.py:177-208,
    :360-392), computed as one tcgen05 GEMM whose epilogue stores the k and
    v thirds of each output row at the token's slot.

    x: [T, C] bf16 (rows 16-byte aligned, unit inner stride); weight: the
    [3C, C] bf16 ``qkv.weight``; pool: a bf16 KVBlockPool with H * D = C;
    slot_mapping: [T] integer CUDA tensor or host ints.  Returns q_out
    ([T, C] bf16, allocated when not given) viewed as [T, H, D].
    """
    _inference_only(x, weight)
    lib = _lib.load()
    if not x.is_cuda:
        raise ValueError("CUDA x required for the b200 backend")
    if x.ndim != 2 or weight.ndim != 2:
        raise ValueError("x must be [T, C] and weight [3C, C]")
    t, c = x.shape
    if weight.shape != (3 * c, c):
        raise ValueError(f"weight must have shape [3C, C] = [{3 * c}, {c}]")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("x and weight must be bfloat16")
    if x.stride(1) != 1 or not weight.is_contiguous():
        raise ValueError("x rows and weight must be contiguous")
    pstruct = _pool_struct(pool)
    if pool.k.dtype != torch.bfloat16:
        raise ValueError("the fused QKV projection needs a bfloat16 KV pool")
    h, d = pool.k.shape[3:]
    if h * d != c:
        raise ValueError("pool num_heads * head_dim must equal the hidden size")
    if not (0 <= layer_idx < pool.k.shape[0]):
        raise ValueError("layer_idx outside KV pool")
    dev = x.device
    if any(z.device != dev for z in (weight, pool.k, pool.v)):
        raise ValueError("all inputs must reside on same CUDA device")
    slots = _index_tensor(slot_mapping, dev, "slot_mapping")
    if slots.shape != (t,):
        raise ValueError("slot_mapping must have shape [T]")
    if q_out is None:
        q_out = torch.empty((t, c), dtype=torch.bfloat16, device=dev)
    elif (q_out.shape != (t, c) or q_out.dtype != torch.bfloat16 or q_out.device != dev
          or q_out.stride(1) != 1):
        raise ValueError("q_out must be a [T, C] bfloat16 tensor with contiguous rows")
    args = _lib.QkvKvWriteArgs()
    args.pool = pstruct
    args.layer_idx = layer_idx
    args.num_tokens = t
    args.hidden = c
    args.x = x.data_ptr()
    args.x_row_stride = x.stride(0) if t > 1 else c
    args.weight = weight.data_ptr()
    args.q_out = q_out.data_ptr()
    args.q_row_stride = q_out.stride(0) if t > 1 else c
    args.slot_mapping = slots.data_ptr()
    args.slot_stride = slots.stride(0) if t > 0 else 1
    args.slot_dtype = _INDEX[slots.dtype]
    if status is not None:
        args.status = status.data_ptr()
    q = q_out.view(t, h, d)
    call = PreparedCall(lib.b200_qkv_kv_write, args, dev, q, "qkv projection",
                        (x, weight, pool.k, pool.v, slots, q_out, status))
    return call if prepare else call()


def _prefill_struct(q, pool, pstruct, table, prefix_len, layer_idx, out, status):
    t, h, d = q.shape
    a = _lib.PrefillArgs()
    a.pool = pstruct
    a.layer_idx = layer_idx
    a.num_tokens = t
    a.prefix_len = prefix_len
    a.q = q.data_ptr()
    a.q_stride = _strides3(q)
    a.q_dtype = _DTYPES[q.dtype]
    a.out = out.data_ptr()
    a.out_stride = _strides3(out)
    a.out_dtype = _DTYPES[out.dtype]
    a.block_table = table.data_ptr()
    a.block_table_len = table.shape[0]
    a.block_table_stride = table.stride(0)
    a.block_table_dtype = _INDEX[table.dtype]
    if status is not None:
        a.status = status.data_ptr()
    return a


def _check_prefill_inputs(q, pool, prefix_len, layer_idx):
    if not q.is_cuda:
        raise ValueError("CUDA q required for the b200 backend")
    if q.ndim != 3:
        raise ValueError("q must have shape [T,H,D]")
    if q.dtype not in _DTYPES:
        raise ValueError("q must be float32, bfloat16 or float16")
    t, h, d = q.shape
    if t == 0 or h == 0 or d == 0:
        raise ValueError("q dimensions must be nonzero")
    if pool.k.ndim != 5 or pool.k.shape[3:] != (h, d):
        raise ValueError("KV head dimensions do not match q")
    if prefix_len < 0:
        raise ValueError("prefix_len must be >= 0")
    if not (0 <= layer_idx < pool.k.shape[0]):
        raise ValueError("layer_idx outside KV pool")


def chunked_prefill_b200(q: torch.Tensor, pool, block_table, prefix_len: int,
                         layer_idx: int, *, out: torch.Tensor | None = None,
                         status: torch.Tensor | None = None, prepare: bool = False):
    """Prefix-aware causal attention of one prefill chunk over paged KV.

    q: [T, H, D] (any strides) for absolute positions prefix_len .. prefix_len+T-1;
    block_table: the sequence's logical->physical block list (host ints or a
    1-D integer CUDA tensor) covering prefix_len + T tokens.  The chunk's K/V
    must already be in the pool (see :func:`kv_scatter_b200`).
    Returns [T, H, D] in q.dtype.
    """
    _inference_only(q)
    lib = _lib.load()
    _check_prefill_inputs(q, pool, prefix_len, layer_idx)
    pstruct = _pool_struct(pool)
    dev = q.device
    if pool.k.device != dev:
        raise ValueError("all inputs must reside on same CUDA device")
    table = _index_tensor(block_table, dev, "block_table")
    if table.ndim != 1:
        raise ValueError("block_table must be 1-D")
    t, h, d = q.shape
    if table.shape[0] * pool.block_size < prefix_len + t:
        raise RuntimeError("incomplete KV block table for prefix")
    if out is None:
        out = torch.empty((t, h, d), dtype=q.dtype, device=dev)
    a = _prefill_struct(q, pool, pstruct, table, prefix_len, layer_idx, out, status)
    stream = _stream_ptr(dev)
    nbytes = lib.b200_chunked_prefill_workspace_size(t, h, d, table.shape[0],
                                                     pool.block_size, pstruct.dtype)
    ws = _workspace(dev, stream, nbytes, prepare)
    if ws is not None:
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
    call = PreparedCall(lib.b200_chunked_prefill, a, dev, out, "chunked prefill",
                        (q, pool.k, pool.v, table, status, ws, out))
    return call if prepare else call()


def chunked_prefill_batch_b200(qs: Sequence[torch.Tensor], pool, block_tables: Sequence,
                               prefix_lens: Sequence[int], layer_idx: int, *,
                               outs: Sequence[torch.Tensor] | None = None,
                               status: torch.Tensor | None = None, prepare: bool = False):
    """Several independent prefill chunks (same pool and layer) in one call."""
    lib = _lib.load()
    if not (len(qs) == len(block_tables) == len(prefix_lens)):
        raise ValueError("qs, block_tables and prefix_lens must have equal length")
    if len(qs) == 0:
        return []
    pstruct = _pool_struct(pool)
    dev = qs[0].device
    structs = (_lib.PrefillArgs * len(qs))()
    results = []
    keep = []
    total_ws = 0
    for i, (q, bt, pl) in enumerate(zip(qs, block_tables, prefix_lens)):
        _inference_only(q)
        _check_prefill_inputs(q, pool, pl, layer_idx)
        if q.device != dev or q.dtype != qs[0].dtype:
            raise ValueError("batched prefill chunks must share device and dtype")
        table = _index_tensor(bt, dev, "block_table")
        keep.append(table)
        if table.shape[0] * pool.block_size < pl + q.shape[0]:
            raise RuntimeError("incomplete KV block table for prefix")
        o = outs[i] if outs is not None else torch.empty(q.shape, dtype=q.dtype, device=dev)
        results.append(o)
        structs[i] = _prefill_struct(q, pool, pstruct, table, pl, layer_idx, o, status)
        total_ws = max(total_ws, lib.b200_chunked_prefill_workspace_size(
            q.shape[0], q.shape[1], q.shape[2], table.shape[0], pool.block_size, pstruct.dtype))
    stream = _stream_ptr(dev)
    ws = _workspace(dev, stream, total_ws, prepare)
    if ws is not None:
        for i in range(len(qs)):
            structs[i].workspace = ws.data_ptr()
            structs[i].workspace_bytes = ws.numel()
    batch = _lib.PrefillBatchArgs(len(qs), structs)
    call = PreparedCall(lib.b200_chunked_prefill_batch, batch, dev, results, "chunked prefill",
                        (tuple(qs), pool.k, pool.v, tuple(keep), status, ws, tuple(results),
                         structs))
    return call if prepare else call()


def decode_bytes(context_lengths: Sequence[int], num_heads: int, head_dim: int,
                 block_size: int, kv_bytes: int, q_bytes: int = 4, out_bytes: int = 4,
                 idx_bytes: int = 8, fused_in_bytes: int = 0) -> int:
    """Algorithmic HBM bytes of one decode launch.

    sum_b ctx_b*H*D*2*kv  (K and V rows read once)
    + B*H*D*(q+out)       (query in, output out)
    + sum_b ceil(ctx_b/S)*idx + B*idx  (block-table entries, context lengths)
    + B*H*D*2*(in+kv) when the KV write is fused (k_new/v_new read, stored).
    """
    B = len(context_lengths)
    tokens = sum(int(c) for c in context_lengths)
    blocks = sum(math.ceil(int(c) / block_size) for c in context_lengths)
    total = tokens * num_heads * head_dim * 2 * kv_bytes
    total += B * num_heads * head_dim * (q_bytes + out_bytes)
    total += blocks * idx_bytes + B * idx_bytes
    if fused_in_bytes:
        total += B * num_heads * head_dim * 2 * (fused_in_bytes + kv_bytes) + B * idx_bytes
    return total


def selftest_bounded_wait(limit_ns: int = 10_000_000, device=None) -> int:
    """Runs the device self-test of the bounded-wait error path: one warp
    waits, through the kernels' own wait routine, on a barrier phase that
    nothing completes; after ``limit_ns`` it gives up, sets
    B200_DEV_WAIT_TIMEOUT and returns.  Returns the status word."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.b200_selftest_bounded_wait(status.data_ptr(), int(limit_ns), _stream_ptr(dev)),
               "bounded-wait selftest")
    return int(status.item())
