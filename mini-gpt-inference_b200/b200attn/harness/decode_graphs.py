"""CUDA-graph replay of the decode step.

minivllm runs the decode step eagerly, with host syncs inside it
(model_runner.py:303, mini_runtime.py:235-238) and no CUDA Graphs
(the project README of mini-gpt-inference, lines 236-237).  Here the
whole step -- embeddings, every layer's
LayerNorm / QKV projection / fused KV write + paged decode attention /
output projection / MLP, the final LayerNorm, LM head and the greedy
argmax -- is captured once per batch bucket and replayed; the host reads
back only the B token ids.

Buckets: every size 1..8, then powers of two up to max_rows.  A step of B
requests replays the smallest bucket >= B; rows B.. of the bucket point at
a scratch block past the block manager's range (context length 1, its own
slot), so their fused KV writes and reads never touch a live sequence and
their tokens are dropped.  Every replay reads the static input buffers,
which the step fills on the device from DeviceDecodeState's upload.
"""
from __future__ import annotations

import torch

from .decode_state import DeviceDecodeState
from .kv_pool import DecodeBatchMetadata


def bucket_sizes(max_rows: int) -> list[int]:
    sizes = list(range(1, min(max_rows, 8) + 1))
    b = 16
    while sizes[-1] < max_rows:
        sizes.append(min(b, max_rows))
        b *= 2
    return sizes


class _Bucket:
    def __init__(self, size: int, max_blocks: int, device, scratch_block: int, block_size: int):
        self.size = size
        self.input_ids = torch.zeros((size, 1), dtype=torch.int64, device=device)
        self.positions = torch.zeros(size, dtype=torch.int64, device=device)
        self.context_lengths = torch.ones(size, dtype=torch.int64, device=device)
        self.slot_mapping = torch.full((size,), scratch_block * block_size, dtype=torch.int64,
                                       device=device)
        self.block_tables = torch.full((size, max_blocks), scratch_block, dtype=torch.int64,
                                       device=device)
        self.meta = DecodeBatchMetadata(positions=self.positions,
                                        context_lengths=self.context_lengths,
                                        block_tables=self.block_tables,
                                        slot_mapping=self.slot_mapping)
        self.graph = None
        self.tokens = None


class DecodeGraphs:
    def __init__(self, model, kv_pool, state: DeviceDecodeState, scratch_block: int):
        if kv_pool.k.device.type != "cuda":
            raise ValueError("decode graphs need a CUDA KV pool")
        if not 0 <= scratch_block < kv_pool.num_blocks:
            raise ValueError("scratch block outside the KV pool")
        self.model, self.kv_pool, self.state = model, kv_pool, state
        self.scratch_block = scratch_block
        self.device = kv_pool.k.device
        self._pool = torch.cuda.graph_pool_handle()
        self._buckets = {n: _Bucket(n, state.max_blocks, self.device, scratch_block,
                                    kv_pool.block_size)
                         for n in bucket_sizes(state.max_rows)}
        self.replays = 0

    def _step(self, bk: _Bucket) -> torch.Tensor:
        logits = self.model.decode_batch(bk.input_ids, bk.meta, self.kv_pool)
        return torch.argmax(logits[:, -1, :], dim=-1)

    def _capture(self, bk: _Bucket) -> None:
        # Warm-up on a side stream (lazy library init, workspace allocation),
        # then capture; the static buffers hold only padding rows here, so
        # the warm-up and capture runs write nothing but the scratch block.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                self._step(bk)
        torch.cuda.current_stream(self.device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._pool):
            bk.tokens = self._step(bk)
        bk.graph = g

    def capture_all(self) -> None:
        for bk in self._buckets.values():
            if bk.graph is None:
                self._capture(bk)

    def max_batch(self) -> int:
        return max(self._buckets)

    def run(self, input_ids: torch.Tensor, meta: DecodeBatchMetadata,
            rows: torch.Tensor) -> torch.Tensor:
        """Greedy tokens [B] of one decode step (device tensor)."""
        B = input_ids.shape[0]
        size = min(n for n in self._buckets if n >= B)
        bk = self._buckets[size]
        if bk.graph is None:
            self._capture(bk)
        bk.input_ids[:B].copy_(input_ids)
        bk.positions[:B].copy_(meta.positions)
        bk.context_lengths[:B].copy_(meta.context_lengths)
        bk.slot_mapping[:B].copy_(meta.slot_mapping)
        torch.index_select(self.state.tables, 0, rows, out=bk.block_tables[:B])
        if B < size:  # rows past B return to padding
            bk.input_ids[B:].zero_()
            bk.positions[B:].zero_()
            bk.context_lengths[B:].fill_(1)
            bk.slot_mapping[B:].fill_(self.scratch_block * self.kv_pool.block_size)
            bk.block_tables[B:].fill_(self.scratch_block)
        bk.graph.replay()
        self.replays += 1
        return bk.tokens[:B]
