"""Runtime harness: the minivllm caller chain (scheduler, block manager,
model, runner, engine loop) restated so the sm_100a backend can be run end
to end -- token for token against the reference runtime -- on machines
where the reference package is not installed."""
from .block_manager import BlockManager
from .kv_pool import DecodeBatchMetadata, KVBlockPool
from .model import B200Backend, MiniGPT, init_weights
from .runner import ModelRunner
from .runtime import IterationRecord, MiniRuntime, build_runtime
from .scheduler import PrefillWorkItem, ScheduleOutput, Scheduler
from .sequence import SequenceState, Status

__all__ = ["BlockManager", "DecodeBatchMetadata", "KVBlockPool", "B200Backend", "MiniGPT",
           "init_weights", "ModelRunner", "IterationRecord", "MiniRuntime", "build_runtime",
           "PrefillWorkItem", "ScheduleOutput", "Scheduler", "SequenceState", "Status"]
