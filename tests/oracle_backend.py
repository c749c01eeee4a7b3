"""Attention backend for the runtime harness built on the CPU oracle.

Test infrastructure: it lets the CPU tests run the harness end to end
(scheduler, block manager, model, runner) against the reference's golden
tokens, with the oracle standing in for the sm_100a kernels.
"""
from __future__ import annotations

import torch

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


class OracleFusedQKVBackend(OracleBackend):
    """The fused-QKV backend's interface (B200FusedQKVBackend) on the oracle:
    the projection and the KV write come from oracle.qkv_project_kv_write,
    attention then reads k and v from the pool."""

    fused_qkv = True

    def __init__(self, decode: bool = False):
        self.fused_qkv_decode = decode
        self.calls = {"prefill_fused": 0, "decode_fused": 0, "decode": 0}

    def decode(self, q, k, v, pool, metadata, layer_idx):
        self.calls["decode"] += 1
        return super().decode(q, k, v, pool, metadata, layer_idx)

    def decode_fused(self, x, weight, pool, metadata, layer_idx):
        self.calls["decode_fused"] += 1
        q = oracle.qkv_project_kv_write(x, weight, pool.k, pool.v, metadata.slot_mapping, layer_idx)
        return oracle.paged_decode_online(q, pool.k, pool.v, metadata.block_tables,
                                          metadata.context_lengths, layer_idx).to(x.dtype)

    def prefill_fused(self, x, weight, pool, block_table, start_pos, slot_mapping, layer_idx):
        self.calls["prefill_fused"] += 1
        q = oracle.qkv_project_kv_write(x, weight, pool.k, pool.v, slot_mapping, layer_idx)
        T = q.shape[0]
        table = [int(t) for t in block_table.tolist()]
        rows = torch.tensor(slot_mapping if not isinstance(slot_mapping, torch.Tensor)
                            else slot_mapping.tolist())
        S = pool.k.shape[2]
        k = pool.k[layer_idx, rows // S, rows % S]
        v = pool.v[layer_idx, rows // S, rows % S]
        return oracle.prefix_prefill(q, k, v, pool.k, pool.v, table, start_pos,
                                     layer_idx).to(x.dtype).reshape(T, *q.shape[1:])
