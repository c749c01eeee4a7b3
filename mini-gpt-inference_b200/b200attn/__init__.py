"""b200attn -- sm_100a paged-attention backend for the minivllm runtime.

Public API (CUDA only, no fallback):
  paged_attention_batch_b200  -- batched paged decode attention (+ fused KV write)
  kv_scatter_b200             -- slot-mapping KV-cache scatter
  chunked_prefill_b200        -- prefix-aware chunked-prefill attention
  chunked_prefill_batch_b200  -- several prefill chunks in one launch
  qkv_kv_write_b200           -- QKV projection with the KV write in its epilogue (bf16)
  selftest_bounded_wait       -- device check of the kernels' bounded-wait error path
Importing the package also registers torch.ops.b200attn.{paged_decode,
kv_scatter, chunked_prefill, qkv_kv_write} (see torch_ops.py).
"""
from .ops import (chunked_prefill_b200, chunked_prefill_batch_b200, decode_bytes,
                  is_available, kv_scatter_b200, paged_attention_batch_b200,
                  qkv_kv_write_b200, selftest_bounded_wait)
from ._lib import LIB_PATH, load as load_library
from . import torch_ops  # registers torch.ops.b200attn.*

__all__ = [
    "paged_attention_batch_b200", "kv_scatter_b200", "chunked_prefill_b200",
    "chunked_prefill_batch_b200", "qkv_kv_write_b200", "selftest_bounded_wait", "decode_bytes", "is_available",
    "load_library", "LIB_PATH",
]
