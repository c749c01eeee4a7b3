"""Engine loop of the runtime harness.

MiniRuntime.step follows minivllm/mini_runtime.py:166-315: schedule, run the
decode batch first, then every prefill chunk of the plan; a request whose
prompt finishes samples its first token unless it was rebuilding a
preempted prefix (then it resumes decoding with its pending last token,
:222-233); finished requests retire; one IterationRecord per step
(:14-44), summed by metrics_summary (:124-141).  Repeated-KV accounting
keeps a per-request high-watermark of executed logical positions
(:110-122).
"""
from __future__ import annotations

import time
from dataclasses import asdict, dataclass

import torch

from .block_manager import BlockManager
from .kv_pool import KVBlockPool
from .model import MiniGPT
from .runner import ModelRunner
from .scheduler import Scheduler
from .sequence import SequenceState, Status


@dataclass
class IterationRecord:
    iteration: int
    prefill_requests: int
    decode_requests: int
    prefill_tokens: int
    decode_tokens: int
    scheduled_tokens: int
    waiting: int
    prefilling: int
    running: int
    used_blocks: int
    free_blocks: int
    kv_utilization: float
    prefill_ms: float
    decode_ms: float
    iteration_ms: float
    schedule_ms: float = 0.0
    preemptions: int = 0
    repeated_kv_tokens: int = 0
    output_tokens: int = 0
    finished_requests: int = 0


class MiniRuntime:
    def __init__(self, runner: ModelRunner, scheduler: Scheduler, sync_cuda_timing: bool = False):
        self.runner = runner
        self.scheduler = scheduler
        self.block_manager = scheduler.block_manager
        self.iteration = 0
        self.records: list[IterationRecord] = []
        self.sync_cuda_timing = sync_cuda_timing
        self._kv_high_watermark: dict[str, int] = {}

    def _sync(self) -> None:
        if self.sync_cuda_timing and torch.cuda.is_available():
            torch.cuda.synchronize()

    def _track_executed_kv(self, seq: SequenceState, start: int, count: int) -> int:
        prev = self._kv_high_watermark.get(seq.seq_id, 0)
        end = start + count
        self._kv_high_watermark[seq.seq_id] = max(prev, end)
        return max(0, min(end, prev) - start)

    def add_request(self, seq: SequenceState) -> None:
        self.scheduler.add_request(seq)

    def metrics_summary(self) -> dict:
        r = self.records
        return {
            "iterations": len(r),
            "scheduled_tokens": sum(x.scheduled_tokens for x in r),
            "prefill_tokens": sum(x.prefill_tokens for x in r),
            "decode_tokens": sum(x.decode_tokens for x in r),
            "output_tokens": sum(x.output_tokens for x in r),
            "preemptions": sum(x.preemptions for x in r),
            "repeated_kv_tokens": sum(x.repeated_kv_tokens for x in r),
            "peak_used_blocks_at_step_end": max((x.used_blocks for x in r), default=0),
            "average_kv_utilization_at_step_end":
                sum(x.kv_utilization for x in r) / len(r) if r else 0.0,
            "total_iteration_ms": sum(x.iteration_ms for x in r),
        }

    def records_as_dicts(self) -> list[dict]:
        return [asdict(x) for x in self.records]

    def step(self) -> None:
        sch = self.scheduler
        self.iteration += 1
        self._sync()
        t_begin = time.perf_counter()
        preempt_before = sch.num_preemptions
        plan = sch.schedule()
        schedule_ms = (time.perf_counter() - t_begin) * 1e3
        assert len(sch.running) + len(plan.prefill) <= sch.max_running
        repeated = 0
        outputs = 0

        t_dec = time.perf_counter()
        if plan.decode:
            starts = [(s, s.length) for s in plan.decode]
            _, tokens = self.runner.decode_batch(plan.decode)
            for s, start in starts:
                repeated += self._track_executed_kv(s, start, 1)
            outputs += len(tokens)
            for s, tok in zip(plan.decode, tokens):
                s.generated_tokens.append(tok)
                s.last_token = tok
        self._sync()
        decode_ms = (time.perf_counter() - t_dec) * 1e3

        t_pre = time.perf_counter()
        for item in plan.prefill:
            seq = item.seq
            if seq.first_schedule_iter is None:
                seq.first_schedule_iter = self.iteration
            logits = self.runner.prefill_chunk(seq, item.start_pos, item.num_tokens)
            repeated += self._track_executed_kv(seq, item.start_pos, item.num_tokens)
            seq.prompt_pos += item.num_tokens
            assert seq.prompt_pos == seq.length
            if seq.prompt_finished:
                if seq.recompute_tokens is not None:
                    # Rebuilt prefix of a preempted request: its last output
                    # was already sampled, so nothing is sampled here.
                    assert seq.generated_tokens and seq.last_token == seq.generated_tokens[-1]
                    assert seq.length == len(seq.recompute_tokens)
                    seq.recompute_tokens = None
                    seq.prompt_pos = seq.prompt_length
                else:
                    tok = int(torch.argmax(logits[:, -1], dim=-1).item())
                    seq.generated_tokens.append(tok)
                    seq.last_token = tok
                    seq.first_token_iter = self.iteration
                    outputs += 1
                seq.status = Status.RUNNING
                sch.prefilling = [s for s in sch.prefilling if s is not seq]
                sch.running.append(seq)
        self._sync()
        prefill_ms = (time.perf_counter() - t_pre) * 1e3

        prefill_tokens = sum(i.num_tokens for i in plan.prefill)
        decode_tokens = len(plan.decode)
        assert prefill_tokens + decode_tokens == plan.num_scheduled_tokens
        assert plan.num_scheduled_tokens <= sch.max_num_batched_tokens
        assert {id(i.seq) for i in plan.prefill}.isdisjoint({id(s) for s in plan.decode})

        finished = 0
        for s in sch.running:
            if s.is_finished():
                s.finish_iter = self.iteration
                finished += 1
        sch.retire_finished()

        self._sync()
        iteration_ms = (time.perf_counter() - t_begin) * 1e3
        free = len(self.block_manager.free_blocks)
        used = self.block_manager.num_blocks - free
        self.records.append(IterationRecord(
            iteration=self.iteration, prefill_requests=len(plan.prefill),
            decode_requests=len(plan.decode), prefill_tokens=prefill_tokens,
            decode_tokens=decode_tokens, scheduled_tokens=plan.num_scheduled_tokens,
            waiting=len(sch.waiting), prefilling=len(sch.prefilling), running=len(sch.running),
            used_blocks=used, free_blocks=free, kv_utilization=used / self.block_manager.num_blocks,
            prefill_ms=prefill_ms, decode_ms=decode_ms, iteration_ms=iteration_ms,
            schedule_ms=schedule_ms, preemptions=sch.num_preemptions - preempt_before,
            repeated_kv_tokens=repeated, output_tokens=outputs, finished_requests=finished))

    def run_to_completion(self, requests: list[SequenceState], max_steps: int = 10_000) -> None:
        for _ in range(max_steps):
            if all(r.status is Status.FINISHED for r in requests):
                return
            self.step()
        raise RuntimeError(f"requests unfinished after {max_steps} steps")


def build_runtime(model: MiniGPT, *, num_blocks: int, block_size: int, max_running: int,
                  token_budget: int, policy: str, n_head: int, head_dim: int,
                  kv_dtype: torch.dtype = torch.float32, device_tables: bool = False,
                  graphs: bool = False) -> MiniRuntime:
    """A runtime over a fresh (uninitialised) KV pool on the model's device.

    device_tables: decode metadata from persistent device block tables.
    graphs: also replay the decode step from CUDA graphs (implies
    device_tables); the pool then holds one extra block past the block
    manager's range, the padding rows' scratch block.
    """
    device = next(model.parameters()).device
    bm = BlockManager(num_blocks, block_size)
    pool_blocks = num_blocks + (1 if graphs else 0)
    pool = KVBlockPool(model.n_layer, pool_blocks, block_size, n_head, head_dim, device=device,
                       dtype=kv_dtype)
    sch = Scheduler(bm, max_running=max_running, max_num_batched_tokens=token_budget,
                    preemption_policy=policy)
    max_blocks = -(-model.block_size // block_size)  # positions bound the sequence length
    runner = ModelRunner(model, pool, bm, device_tables=device_tables, graphs=graphs,
                         max_rows=max_running, max_blocks=max_blocks, scratch_block=num_blocks)
    return MiniRuntime(runner, sch)
