"""torch.ops.b200attn.*: the backend's ops registered with the PyTorch dispatcher.

Registered with ``torch.library.custom_op`` (schema below). Each op has a fake
(meta) implementation, so tracing and CUDA-graph capture see shapes and
mutations without running a kernel. The CUDA implementations call the same
C-ABI entry points as :mod:`b200attn.ops`.

    b200attn::paged_decode(Tensor q, Tensor(a!) k_pool, Tensor(b!) v_pool,
                           Tensor block_tables, Tensor context_lengths, int layer_idx,
                           Tensor? k_new, Tensor? v_new, Tensor? slot_mapping) -> Tensor
    b200attn::kv_scatter(Tensor k, Tensor v, Tensor(a!) k_pool, Tensor(b!) v_pool,
                         Tensor slot_mapping, int layer_idx) -> ()
    b200attn::chunked_prefill(Tensor q, Tensor k, Tensor v, Tensor(a!) k_pool,
                              Tensor(b!) v_pool, Tensor block_table, Tensor slot_mapping,
                              int prefix_len, int layer_idx) -> Tensor
    b200attn::qkv_kv_write(Tensor x, Tensor weight, Tensor(a!) k_pool, Tensor(b!) v_pool,
                           Tensor slot_mapping, int layer_idx) -> Tensor

The pools are the KVBlockPool tensors ``[L, P, S, H, D]`` (S = block size).
``paged_decode`` writes k_new/v_new into the pools when they are given
(minivllm/attention.py:370-392). ``chunked_prefill`` scatters the chunk's k/v
at ``slot_mapping`` (attention.py:193-208) and returns the prefix-aware
attention of the chunk (attention.py:215-299). ``qkv_kv_write`` is the bf16
QKV projection (attention.py:79-83) that stores k and v at ``slot_mapping``
from its epilogue and returns q as [T, H, D] (attention.py:177-208,
:360-392). Importing this module registers the ops.
"""
from __future__ import annotations

from types import SimpleNamespace
from typing import Optional

import torch

from . import ops

__all__ = ["paged_decode", "kv_scatter", "chunked_prefill", "qkv_kv_write"]


def _pool(k_pool: torch.Tensor, v_pool: torch.Tensor) -> SimpleNamespace:
    if k_pool.ndim != 5:
        raise ValueError("k_pool must have shape [L,P,S,H,D]")
    return SimpleNamespace(k=k_pool, v=v_pool, block_size=int(k_pool.shape[2]))


@torch.library.custom_op("b200attn::paged_decode", mutates_args=("k_pool", "v_pool"))
def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_tables: torch.Tensor, context_lengths: torch.Tensor, layer_idx: int,
                 k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                 slot_mapping: Optional[torch.Tensor] = None) -> torch.Tensor:
    return ops.paged_attention_batch_b200(q, _pool(k_pool, v_pool), block_tables,
                                          context_lengths, layer_idx, k_new=k_new, v_new=v_new,
                                          slot_mapping=slot_mapping)


@paged_decode.register_fake
def _(q, k_pool, v_pool, block_tables, context_lengths, layer_idx, k_new=None, v_new=None,
      slot_mapping=None):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


@torch.library.custom_op("b200attn::kv_scatter", mutates_args=("k_pool", "v_pool"))
def kv_scatter(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
               slot_mapping: torch.Tensor, layer_idx: int) -> None:
    ops.kv_scatter_b200(k, v, _pool(k_pool, v_pool), slot_mapping, layer_idx)


@kv_scatter.register_fake
def _(k, v, k_pool, v_pool, slot_mapping, layer_idx):
    return None


@torch.library.custom_op("b200attn::chunked_prefill", mutates_args=("k_pool", "v_pool"))
def chunked_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                    v_pool: torch.Tensor, block_table: torch.Tensor, slot_mapping: torch.Tensor,
                    prefix_len: int, layer_idx: int) -> torch.Tensor:
    pool = _pool(k_pool, v_pool)
    ops.kv_scatter_b200(k, v, pool, slot_mapping, layer_idx)
    return ops.chunked_prefill_b200(q, pool, block_table, prefix_len, layer_idx)


@chunked_prefill.register_fake
def _(q, k, v, k_pool, v_pool, block_table, slot_mapping, prefix_len, layer_idx):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


@torch.library.custom_op("b200attn::qkv_kv_write", mutates_args=("k_pool", "v_pool"))
def qkv_kv_write(x: torch.Tensor, weight: torch.Tensor, k_pool: torch.Tensor,
                 v_pool: torch.Tensor, slot_mapping: torch.Tensor, layer_idx: int) -> torch.Tensor:
    q = x.new_empty((x.shape[0], k_pool.shape[3], k_pool.shape[4]))
    ops.qkv_kv_write_b200(x, weight, _pool(k_pool, v_pool), slot_mapping, layer_idx,
                          q_out=q.view(x.shape[0], -1))
    return q


@qkv_kv_write.register_fake
def _(x, weight, k_pool, v_pool, slot_mapping, layer_idx):
    return x.new_empty((x.shape[0], k_pool.shape[3], k_pool.shape[4]))
