"""Request state of the runtime harness.

Mirrors SequenceState / Status (minivllm/sequence.py:4-56): a request's
prompt, generated tokens, logical length, block table and the
recompute-preemption prefix (recompute_tokens, minivllm/sequence.py:25-32).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum


class Status(Enum):
    WAITING = "waiting"
    PREFILLING = "prefilling"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass
class SequenceState:
    seq_id: str
    max_tokens: int
    prompt_tokens: list[int]
    prompt_pos: int = 0
    last_token: int | None = None
    generated_tokens: list[int] = field(default_factory=list)
    status: Status = Status.WAITING
    length: int = 0
    block_table: list[int] = field(default_factory=list)
    # Cached token prefix to rebuild after a recompute preemption; the
    # pending last_token is not part of it.
    recompute_tokens: list[int] | None = None
    num_preemptions: int = 0
    arrival_iter: int = 0
    first_schedule_iter: int | None = None
    first_token_iter: int | None = None
    finish_iter: int | None = None

    @property
    def prefill_input_tokens(self) -> list[int]:
        return self.prompt_tokens if self.recompute_tokens is None else self.recompute_tokens

    @property
    def prompt_length(self) -> int:
        return len(self.prompt_tokens)

    @property
    def remaining_prompt_tokens(self) -> int:
        return len(self.prefill_input_tokens) - self.prompt_pos

    @property
    def prompt_finished(self) -> bool:
        return self.prompt_pos == len(self.prefill_input_tokens)

    def is_finished(self) -> bool:
        return len(self.generated_tokens) >= self.max_tokens - self.prompt_length
