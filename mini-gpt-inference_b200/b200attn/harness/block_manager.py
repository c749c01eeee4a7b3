"""Physical KV block allocator of the runtime harness.

Same allocation order and slot arithmetic as minivllm's BlockManager
(minivllm/block_manager.py:4-177), because block tables and slot mappings
-- and therefore which physical blocks the kernels read -- must match the
reference step for step: a LIFO free list initialised so block 0 is handed
out first (:9-11), one block appended when a sequence's length reaches a
block boundary (:61-110), and blocks returned in table order on free
(:131-147).
"""
from __future__ import annotations

from .sequence import SequenceState


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free_blocks = list(range(num_blocks - 1, -1, -1))
        self.block_owner: dict[int, str] = {}
        self._free_listeners: list = []

    def add_free_listener(self, fn) -> None:
        """fn(seq) runs after free() returns a sequence's blocks (finish or
        preemption), e.g. to drop device-side copies of its block table."""
        self._free_listeners.append(fn)

    def _take_block(self, seq: SequenceState) -> int:
        if not self.free_blocks:
            raise RuntimeError("KV block pool exhausted")
        blk = self.free_blocks.pop()
        if blk in self.block_owner:
            raise AssertionError(f"block {blk} handed out twice")
        self.block_owner[blk] = seq.seq_id
        seq.block_table.append(blk)
        return blk

    def num_new_blocks_needed(self, seq: SequenceState, num_tokens: int) -> int:
        target = -(-(seq.length + num_tokens) // self.block_size)
        return max(0, target - len(seq.block_table))

    def can_reserve(self, seq: SequenceState, num_tokens: int) -> bool:
        return self.num_new_blocks_needed(seq, num_tokens) <= len(self.free_blocks)

    def _slot_at(self, seq: SequenceState, pos: int) -> tuple[int, int, int]:
        blk_idx, off = divmod(pos, self.block_size)
        if blk_idx == len(seq.block_table):
            self._take_block(seq)
        phys = seq.block_table[blk_idx]
        return phys, off, phys * self.block_size + off

    def reserve_append_slot(self, seq: SequenceState) -> tuple[int, int, int]:
        """(physical block, offset, slot) of the token at position seq.length."""
        return self._slot_at(seq, seq.length)

    def reserve_slots(self, seq: SequenceState, num_tokens: int) -> list[int]:
        return [self._slot_at(seq, seq.length + i)[2] for i in range(num_tokens)]

    def logical_to_slot(self, seq: SequenceState, logical_pos: int) -> int:
        if not 0 <= logical_pos < seq.length:
            raise IndexError(f"logical_pos={logical_pos}, length={seq.length}")
        blk_idx, off = divmod(logical_pos, self.block_size)
        return seq.block_table[blk_idx] * self.block_size + off

    def free(self, seq: SequenceState) -> list[int]:
        released = list(seq.block_table)
        for blk in released:
            if self.block_owner.pop(blk) != seq.seq_id:
                raise AssertionError(f"block {blk} not owned by {seq.seq_id}")
            self.free_blocks.append(blk)
        seq.block_table.clear()
        seq.length = 0
        for fn in self._free_listeners:
            fn(seq)
        return released

    def check_invariants(self, sequences: list[SequenceState]) -> None:
        free = set(self.free_blocks)
        owned = set(self.block_owner)
        assert len(free) == len(self.free_blocks), "duplicate free block"
        assert not (free & owned), "block both free and owned"
        assert free | owned == set(range(self.num_blocks)), "block lost"
        for seq in sequences:
            assert len(seq.block_table) == len(set(seq.block_table))
            for blk in seq.block_table:
                assert self.block_owner[blk] == seq.seq_id
            assert len(seq.block_table) == -(-seq.length // self.block_size)
