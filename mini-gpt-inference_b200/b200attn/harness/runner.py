"""Model runner of the runtime harness: host -> device metadata and sampling.

Follows ModelRunner (minivllm/model_runner.py:68-304): a prefill chunk
reserves its slots first and feeds the request's (possibly recompute)
input tokens (:68-120); a decode step reserves one append slot per request,
builds DecodeBatchMetadata with context length = length + 1 and -1-padded
block tables (:123-216), and samples greedily with argmax (:272-304).
The device copies of a step's metadata are made once per step and shared by
every layer.  With device_tables the step's metadata comes from
DeviceDecodeState (persistent device block tables, one packed upload per
step); with graphs the decode step is also replayed from a CUDA graph.
"""
from __future__ import annotations

import torch

from .block_manager import BlockManager
from .decode_graphs import DecodeGraphs
from .decode_state import DeviceDecodeState
from .kv_pool import DecodeBatchMetadata, KVBlockPool
from .model import MiniGPT
from .sequence import SequenceState


def _to_device(values, device) -> torch.Tensor:
    t = torch.tensor(values, dtype=torch.int64)
    if torch.device(device).type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


class ModelRunner:
    def __init__(self, model: MiniGPT, kv_pool: KVBlockPool, block_manager: BlockManager, *,
                 device_tables: bool = False, graphs: bool = False, max_rows: int = 0,
                 max_blocks: int = 0, scratch_block: int = -1):
        self.model, self.kv_pool, self.block_manager = model, kv_pool, block_manager
        self.state = None
        self.graphs = None
        if device_tables or graphs:
            self.state = DeviceDecodeState(block_manager, max_rows, max_blocks, kv_pool.k.device)
        if graphs:
            self.graphs = DecodeGraphs(model, kv_pool, self.state, scratch_block)

    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    def prefill_chunk(self, seq: SequenceState, start_pos: int, num_tokens: int) -> torch.Tensor:
        assert start_pos == seq.prompt_pos == seq.length
        tokens = seq.prefill_input_tokens[start_pos:start_pos + num_tokens]
        assert len(tokens) == num_tokens, "prefill chunk exceeds input prefix"
        dev = self.device
        input_ids = _to_device([tokens], dev)
        slots = self.block_manager.reserve_slots(seq, num_tokens)
        table = _to_device(seq.block_table, dev)
        logits = self.model.prefill_chunk(input_ids, self.kv_pool, start_pos, table,
                                          _to_device(slots, dev))
        seq.length += num_tokens
        return logits

    def prepare_decode_batch(self, sequences: list[SequenceState]):
        assert sequences
        dev = self.device
        input_ids = _to_device([[s.last_token] for s in sequences], dev)
        slots = [self.block_manager.reserve_append_slot(s)[2] for s in sequences]
        width = max(len(s.block_table) for s in sequences)
        table = [s.block_table + [-1] * (width - len(s.block_table)) for s in sequences]
        meta = DecodeBatchMetadata(
            positions=_to_device([s.length for s in sequences], dev),
            context_lengths=_to_device([s.length + 1 for s in sequences], dev),
            block_tables=_to_device(table, dev),
            slot_mapping=_to_device(slots, dev))
        return input_ids, meta

    def decode_batch(self, sequences: list[SequenceState]):
        """(last-position logits or None, greedy token ids) of one decode step."""
        if not sequences:
            return []
        if self.state is not None:
            slots = [self.block_manager.reserve_append_slot(s)[2] for s in sequences]
            input_ids, meta, rows = self.state.build(sequences, slots)
            if self.graphs is not None and len(sequences) <= self.graphs.max_batch():
                tokens = self.graphs.run(input_ids, meta, rows).tolist()
                for s in sequences:
                    s.length += 1
                return None, tokens
        else:
            input_ids, meta = self.prepare_decode_batch(sequences)
        logits = self.model.decode_batch(input_ids, meta, self.kv_pool)
        for s in sequences:
            s.length += 1
        last = logits[:, -1, :]
        return last, torch.argmax(last, dim=-1).tolist()
