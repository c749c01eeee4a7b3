"""Attention backend for the runtime harness built on the CPU oracle.

Test infrastructure: it lets the CPU tests run the harness end to end
(scheduler, block manager, model, runner) against the reference's golden
tokens, with the oracle standing in for the sm_100a kernels.
"""
from __future__ import annotations

import oracle


class OracleBackend:
    def decode(self, q, k, v, pool, metadata, layer_idx):
        oracle.kv_scatter(pool.k, pool.v, k, v, metadata.slot_mapping, layer_idx)
        return oracle.paged_decode_online(q, pool.k, pool.v, metadata.block_tables,
                                          metadata.context_lengths, layer_idx).to(q.dtype)

    def prefill(self, q, k, v, pool, block_table, start_pos, slot_mapping, layer_idx):
        oracle.kv_scatter(pool.k, pool.v, k, v, slot_mapping, layer_idx)
        table = [int(x) for x in block_table.tolist()]
        return oracle.prefix_prefill(q, k, v, pool.k, pool.v, table, start_pos,
                                     layer_idx).to(q.dtype)
