"""CPU oracle of the paged-attention path (test infrastructure only).

Imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline
leg, always as the checker or the timed CPU reference -- never by the product
package.
"""
from .paged_attention import (kv_scatter, paged_decode_dense, paged_decode_online,
                              paged_decode_single, prefill_per_token, prefix_prefill,
                              prefix_prefill_from_pool, qkv_project_kv_write)

__all__ = ["kv_scatter", "paged_decode_dense", "paged_decode_online", "paged_decode_single",
           "prefill_per_token", "prefix_prefill", "prefix_prefill_from_pool",
           "qkv_project_kv_write"]
