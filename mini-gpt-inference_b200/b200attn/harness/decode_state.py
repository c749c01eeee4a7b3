"""Device-resident decode metadata, updated incrementally.

minivllm rebuilds DecodeBatchMetadata on the host every step
(ModelRunner._prepare_decode_batch, minivllm/model_runner.py:123-216): one
torch.tensor per field, and the whole -1-padded [B, M] block table crosses
PCIe each step (1 MB per step for 64 requests of 32k tokens).  Here every
running sequence owns a row of a persistent [rows, max_blocks] int64 device
table.  A step packs into one pinned buffer the batch's token ids,
positions, context lengths, slots and row ids plus only the table entries
appended since each sequence's previous step; one host-to-device copy
moves it, the device applies the new entries and gathers the batch's rows.
A sequence's row is released when the block manager frees its blocks
(finish or recompute preemption), so a re-admitted sequence is re-synced
from its first block.  Table entries past a sequence's context are never
read by the decode kernel, so a reused row needs no clearing.
"""
from __future__ import annotations

import numpy as np
import torch

from .kv_pool import DecodeBatchMetadata
from .sequence import SequenceState


class DeviceDecodeState:
    def __init__(self, block_manager, max_rows: int, max_blocks: int, device):
        if max_rows < 1 or max_blocks < 1:
            raise ValueError("max_rows and max_blocks must be positive")
        self.device = torch.device(device)
        self.max_rows, self.max_blocks = max_rows, max_blocks
        self.tables = torch.full((max_rows, max_blocks), -1, dtype=torch.int64,
                                 device=self.device)
        self._free_rows = list(range(max_rows - 1, -1, -1))
        self.row_of: dict[str, int] = {}
        self._synced: dict[str, int] = {}
        self._host = torch.empty(0, dtype=torch.int64)
        self._dev = torch.empty(0, dtype=torch.int64, device=self.device)
        self._copied = None  # event of the last host->device copy (CUDA)
        self.uploaded_entries = 0  # table entries sent so far (for tests)
        block_manager.add_free_listener(self.release)

    def release(self, seq: SequenceState) -> None:
        row = self.row_of.pop(seq.seq_id, None)
        if row is not None:
            self._synced.pop(seq.seq_id, None)
            self._free_rows.append(row)

    def _buffers(self, n: int) -> None:
        if self._host.numel() < n:
            cap = max(n, 2 * self._host.numel(), 256)
            pin = self.device.type == "cuda"
            self._host = torch.empty(cap, dtype=torch.int64, pin_memory=pin)
            self._dev = torch.empty(cap, dtype=torch.int64, device=self.device)

    def build(self, sequences: list[SequenceState], slots: list[int]):
        """(input_ids [B,1], DecodeBatchMetadata) on the device for one step.

        `slots` are the append slots already reserved for the step (so every
        block the step touches is in the sequences' block tables)."""
        B = len(sequences)
        rows: list[int] = []
        u_row: list[int] = []
        u_col: list[int] = []
        u_val: list[int] = []
        width = 1
        for s in sequences:
            row = self.row_of.get(s.seq_id)
            if row is None:
                if not self._free_rows:
                    raise RuntimeError("no free decode-table row (max_rows too small)")
                row = self._free_rows.pop()
                self.row_of[s.seq_id] = row
                self._synced[s.seq_id] = 0
            n = len(s.block_table)
            if n > self.max_blocks:
                raise ValueError(f"sequence {s.seq_id} needs {n} blocks > max_blocks")
            k = self._synced[s.seq_id]
            if n < k:  # table rebuilt without a free(): resend it whole
                k = 0
            for j in range(k, n):
                u_row.append(row)
                u_col.append(j)
                u_val.append(s.block_table[j])
            self._synced[s.seq_id] = n
            rows.append(row)
            width = max(width, n)
        U = len(u_val)
        total = 5 * B + 3 * U
        self._buffers(total)
        if self._copied is not None:
            self._copied.synchronize()  # the previous step's copy has read the buffer
        h = self._host.numpy()
        h[0:B] = [s.last_token for s in sequences]
        h[B:2 * B] = [s.length for s in sequences]
        h[2 * B:3 * B] = [s.length + 1 for s in sequences]
        h[3 * B:4 * B] = slots
        h[4 * B:5 * B] = rows
        if U:
            h[5 * B:5 * B + U] = u_row
            h[5 * B + U:5 * B + 2 * U] = u_col
            h[5 * B + 2 * U:total] = u_val
        d = self._dev[:total]
        d.copy_(self._host[:total], non_blocking=True)
        if self.device.type == "cuda":
            self._copied = torch.cuda.Event()
            self._copied.record()
        if U:
            self.tables.index_put_((d[5 * B:5 * B + U], d[5 * B + U:5 * B + 2 * U]),
                                   d[5 * B + 2 * U:total])
            self.uploaded_entries += U
        rows_d = d[4 * B:5 * B]
        meta = DecodeBatchMetadata(positions=d[B:2 * B], context_lengths=d[2 * B:3 * B],
                                   block_tables=self.tables.index_select(0, rows_d)[:, :width],
                                   slot_mapping=d[3 * B:4 * B])
        return d[0:B].view(B, 1), meta, rows_d
