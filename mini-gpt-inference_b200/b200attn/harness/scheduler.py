"""Continuous-batching scheduler of the runtime harness.

The scheduling policy must match minivllm's Scheduler
(minivllm/scheduler.py:24-242) decision for decision, because greedy
token equality with the reference runtime (including recompute-preemption
runs) depends on identical batches, chunk sizes, victims and block tables:

* decode first: every RUNNING sequence gets one token if a block is
  available, preempting others under the recompute policy (:162-178);
* then in-flight prefills, chunked by the remaining token budget and, under
  recompute, by the blocks already held plus free ones (:136-149, :180-206);
* then admissions from the waiting queue, never in a step that preempted
  (:208-236); the conservative policy admits only when the sum of every
  active request's maximum KV demand still fits (:46-49);
* victims: newest partial prefill first, then newest decode, never a
  request already planned this step (:99-113); a preempted RUNNING request
  keeps prompt + generated[:-1] to recompute (:65-85).
"""
from __future__ import annotations

from dataclasses import dataclass

from .block_manager import BlockManager
from .sequence import SequenceState, Status


@dataclass
class PrefillWorkItem:
    seq: SequenceState
    start_pos: int
    num_tokens: int

    @property
    def end_pos(self) -> int:
        return self.start_pos + self.num_tokens


@dataclass
class ScheduleOutput:
    prefill: list[PrefillWorkItem]
    decode: list[SequenceState]
    num_scheduled_tokens: int


class Scheduler:
    def __init__(self, block_manager: BlockManager, max_running: int,
                 max_num_batched_tokens: int, preemption_policy: str = "conservative"):
        if preemption_policy not in ("conservative", "recompute"):
            raise ValueError("preemption_policy must be 'conservative' or 'recompute'")
        self.waiting: list[SequenceState] = []
        self.prefilling: list[SequenceState] = []
        self.running: list[SequenceState] = []
        self.block_manager = block_manager
        self.max_running = max_running
        self.max_num_batched_tokens = max_num_batched_tokens
        self.preemption_policy = preemption_policy
        self.num_preemptions = 0

    # -------------------------------------------------------------- helpers
    def _max_kv_blocks(self, seq: SequenceState) -> int:
        return -(-(seq.max_tokens - 1) // self.block_manager.block_size)

    def _fits_without_preemption(self, seq: SequenceState) -> bool:
        committed = sum(self._max_kv_blocks(s) for s in self.running + self.prefilling)
        return committed + self._max_kv_blocks(seq) <= self.block_manager.num_blocks

    def _chunk_size(self, seq: SequenceState, budget: int, free_blocks: int) -> int:
        want = min(seq.remaining_prompt_tokens, budget)
        if self.preemption_policy != "recompute":
            return want
        room = (len(seq.block_table) + free_blocks) * self.block_manager.block_size - seq.length
        return min(want, max(0, room))

    def _victim(self, target: SequenceState, planned: set[int]) -> SequenceState | None:
        for seq in [*reversed(self.prefilling), *reversed(self.running)]:
            if seq is target or id(seq) in planned:
                continue
            if seq.block_table:
                return seq
        return None

    def _reclaim(self, target: SequenceState, needed: int, free_blocks: int,
                 planned: set[int]) -> tuple[int, bool]:
        if self.preemption_policy != "recompute":
            return free_blocks, False
        preempted = False
        while free_blocks < needed:
            victim = self._victim(target, planned)
            if victim is None:
                break
            freed = len(victim.block_table)
            self.preempt(victim)
            free_blocks += freed
            preempted = True
        return free_blocks, preempted

    # -------------------------------------------------------------- public
    def add_request(self, seq: SequenceState) -> None:
        if not seq.prompt_tokens or seq.max_tokens <= seq.prompt_length:
            raise ValueError("prompt must be nonempty and output token must be positive")
        if self._max_kv_blocks(seq) > self.block_manager.num_blocks:
            raise ValueError("request's maximum KV demand exceeds total block capacity")
        self.waiting.append(seq)

    def preempt(self, seq: SequenceState) -> None:
        """Evict a request's KV and queue it for recomputation (between steps)."""
        if any(s is seq for s in self.running):
            assert seq.generated_tokens and seq.last_token == seq.generated_tokens[-1]
            seq.recompute_tokens = seq.prompt_tokens + seq.generated_tokens[:-1]
            assert len(seq.recompute_tokens) == seq.length
            self.running = [s for s in self.running if s is not seq]
        elif any(s is seq for s in self.prefilling):
            self.prefilling = [s for s in self.prefilling if s is not seq]
        else:
            raise ValueError("Only active requests may be preempted")
        self.num_preemptions += 1
        seq.num_preemptions += 1
        self.block_manager.free(seq)
        seq.prompt_pos = 0
        seq.status = Status.WAITING
        self.waiting.insert(0, seq)

    def retire_finished(self) -> None:
        alive = []
        for seq in self.running:
            if seq.is_finished():
                seq.status = Status.FINISHED
                self.block_manager.free(seq)
            else:
                alive.append(seq)
        self.running = alive

    def schedule(self) -> ScheduleOutput:
        prefill: list[PrefillWorkItem] = []
        decode: list[SequenceState] = []
        budget = self.max_num_batched_tokens
        free_blocks = len(self.block_manager.free_blocks)
        planned: set[int] = set()
        preempted = False

        for seq in list(self.running):
            if budget < 1:
                break
            if seq.status != Status.RUNNING:
                continue
            need = self.block_manager.num_new_blocks_needed(seq, 1)
            if need > free_blocks:
                free_blocks, did = self._reclaim(seq, need, free_blocks, planned)
                preempted |= did
            if need > free_blocks:
                continue
            decode.append(seq)
            planned.add(id(seq))
            budget -= 1
            free_blocks -= need

        for seq in list(self.prefilling):
            if budget <= 0:
                break
            if seq.status != Status.PREFILLING or seq.remaining_prompt_tokens <= 0:
                continue
            n = self._chunk_size(seq, budget, free_blocks)
            if n == 0 and self.preemption_policy == "recompute":
                free_blocks, did = self._reclaim(seq, 1, free_blocks, planned)
                preempted |= did
                n = self._chunk_size(seq, budget, free_blocks)
            if n <= 0:
                continue
            need = self.block_manager.num_new_blocks_needed(seq, n)
            if need > free_blocks:
                continue
            prefill.append(PrefillWorkItem(seq, seq.prompt_pos, n))
            planned.add(id(seq))
            budget -= n
            free_blocks -= need

        while self.waiting and budget > 0 and not preempted:
            if len(self.running) + len(self.prefilling) >= self.max_running:
                break
            seq = self.waiting[0]
            if self.preemption_policy == "conservative" and not self._fits_without_preemption(seq):
                break
            n = self._chunk_size(seq, budget, free_blocks)
            if n <= 0:
                break
            need = self.block_manager.num_new_blocks_needed(seq, n)
            if need > free_blocks:
                break
            self.waiting.pop(0)
            seq.status = Status.PREFILLING
            self.prefilling.append(seq)
            prefill.append(PrefillWorkItem(seq, seq.prompt_pos, n))
            planned.add(id(seq))
            budget -= n
            free_blocks -= need

        return ScheduleOutput(prefill, decode, self.max_num_batched_tokens - budget)
