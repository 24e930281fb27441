"""Tensor-parallel LLM driver on 2+ GPUs (torchrun, NCCL): TP=world logits and
greedy ids against the oracle decoder (tests/tp_worker.py).  A second run sends
every fused decode all-reduce through its 16-bit form (EVKCU_FUSED_AR_HALF=1,
which the driver otherwise uses only for calls above 32,768 elements)."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("half", [0, 1])
def test_llm_tensor_parallel_matches_single_gpu(half):
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EVKCU_FUSED_AR_HALF=str(half))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}", "--master-addr",
           "127.0.0.1", "--master-port", str(29533 + half), os.path.join(ROOT, "tests", "tp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_OK" in r.stdout, r.stdout[-3000:]
