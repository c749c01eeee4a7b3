"""End to end on the GPU: configuration 2 through the runtime harness with the
sm_100a kernels (fused KV-write decode, scatter, chunked prefill), fp32 with
TF32 off.  Greedy tokens and lifecycle counts must equal the reference
MiniRuntime's, with ample KV and with capped KV (recompute preemption), for
host-built decode metadata, persistent device block tables, and CUDA-graph
replay of the decode step."""
from __future__ import annotations

import pytest
import torch

from e2e_common import GOLDEN, run_cfg2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["eager", "device_tables", "graphs"])
@pytest.mark.parametrize("run_name", ["ample", "capped"])
def test_cfg2_token_exact_on_gpu(run_name, mode):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    tokens, counts, rt = run_cfg2(run_name, "cuda", mode=mode)
    want = GOLDEN[f"{run_name}/sdpa_v2"]
    assert tokens == want["tokens"]
    assert counts == want["counts"]
    if mode != "eager":
        assert not rt.runner.state.row_of
    if mode == "graphs":
        assert rt.runner.graphs.replays == sum(r.decode_requests > 0 for r in rt.records)

