"""The documented host diff, run on minivllm's own code (CPU).

INTEGRATION.md's change to minivllm is committed as an insertion-only patch
(mini-gpt-inference_b200/integration/minivllm_sm100.patch).  This test
applies it to a copy of the reference checkout and runs configuration 2
through the reference's own MiniRuntime with the "sm100" backends, the
b200attn entry points standing in as oracle-backed CPU functions that also
check how the diff calls them (tests/integration_minivllm.py).  The greedy
tokens and lifecycle counts must equal the golden ones the reference
produced with its own backends (tests/golden/e2e_golden.json), ample and
capped KV, including the recompute-preemption run.

The checkout is found through $MINIVLLM_REFERENCE, else a ``reference``
directory beside this repository; without one the test is skipped (a GPU
box has none).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from e2e_common import GOLDEN

REPO = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("MINIVLLM_REFERENCE", REPO.parent / "reference"))

needs_reference = pytest.mark.skipif(not (REFERENCE / "minivllm" / "attention.py").is_file(),
                                     reason="no minivllm checkout to patch")


@needs_reference
def test_patched_minivllm_gives_the_golden_tokens(tmp_path):
    res = subprocess.run([sys.executable, str(REPO / "tests" / "integration_minivllm.py"),
                          "--reference", str(REFERENCE), "--workdir", str(tmp_path)],
                         capture_output=True, text=True, timeout=1200, cwd=REPO)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["hunks"] == 4
    assert len(out["runs"]) == 4
    for key, run in out["runs"].items():
        run_name, prefill_mode, decode_backend = key.split("/")
        want = GOLDEN[f"{run_name}/sdpa_v2"]
        assert run["tokens"] == want["tokens"], key
        assert run["counts"] == want["counts"], key
        if run_name == "capped":
            assert run["counts"]["preemptions"] > 0
        calls = run["calls"]
        assert (calls["decode"] > 0) == (decode_backend == "sm100"), key
        if prefill_mode == "sm100":
            assert calls["scatter"] == calls["prefill"] > 0, key
        else:
            assert calls["scatter"] == calls["prefill"] == 0, key


def test_patch_is_insertion_only():
    """The patch carries no line of the reference: only its own added lines
    and hunk headers (so it holds none of the reference's source)."""
    text = (REPO / "mini-gpt-inference_b200" / "integration" / "minivllm_sm100.patch").read_text()
    body = text[text.index("diff --git"):]
    for line in body.splitlines():
        assert line.startswith(("diff --git", "--- ", "+++ ", "@@ ", "+")), line
        if line.startswith("@@"):
            assert ",0 +" in line
