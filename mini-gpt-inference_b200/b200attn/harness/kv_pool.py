"""Paged KV storage and decode metadata of the runtime harness.

KVBlockPool keeps minivllm's layout unchanged -- two tensors
[n_layer, num_blocks, block_size, n_head, head_dim], uninitialised
(minivllm/kv_block_pool.py:32-68) -- which is the layout the kernels read.
DecodeBatchMetadata has the fields of minivllm/decode_batch_metadata.py:6-14.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .sequence import SequenceState


class KVBlockPool:
    def __init__(self, n_layer: int, num_blocks: int, block_size: int, n_head: int,
                 head_dim: int, device="cpu", dtype=torch.float32):
        self.n_layer = n_layer
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_head = n_head
        self.head_dim = head_dim
        self.dtype = dtype
        shape = (n_layer, num_blocks, block_size, n_head, head_dim)
        self.k = torch.empty(shape, dtype=dtype, device=device)
        self.v = torch.empty(shape, dtype=dtype, device=device)

    def gather_sequence(self, seq: SequenceState) -> tuple[torch.Tensor, torch.Tensor]:
        """Logical K/V of a sequence, [n_layer, length, n_head, head_dim], on the CPU."""
        n = seq.length
        nb = -(-n // self.block_size)
        idx = torch.tensor(seq.block_table[:nb], dtype=torch.long, device=self.k.device)
        k = self.k[:, idx].reshape(self.n_layer, -1, self.n_head, self.head_dim)[:, :n]
        v = self.v[:, idx].reshape(self.n_layer, -1, self.n_head, self.head_dim)[:, :n]
        return k.cpu(), v.cpu()


@dataclass
class DecodeBatchMetadata:
    positions: torch.Tensor
    context_lengths: torch.Tensor
    block_tables: torch.Tensor
    slot_mapping: torch.Tensor
