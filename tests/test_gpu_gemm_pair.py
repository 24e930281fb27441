"""The paired-SM GEMM (two CTAs on neighbouring SMs share one
tcgen05.mma.cta_group::2 of M = 256; persistent over 256 x 256 tiles).

By default it takes only outputs of at least one 256 x 256 tile per resident
SM pair, so the small parity shapes run the one-SM kernel.  Here the matmul
and LLM-config parity suites run again in a child process with
EVKCU_GEMM_PAIR=1 (read when the library creates its device state), which
sends every shape with M >= 256 through the paired kernel: ragged M / N / K,
both transposes, batch broadcast, C += A B, the GELU epilogue and the fused
QKV + RoPE + KV-cache epilogue of a prefill (C4 / C5 at full width)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pair_kernel_available():
    import evk_b200

    evk_b200.init(0)
    n = evk_b200.lib().evkcu_debug_gemm_pair_clusters()
    assert n >= 32, f"paired-SM GEMM resident pairs: {n}"


def test_parity_suites_with_pair_kernel_forced():
    env = dict(os.environ, EVKCU_GEMM_PAIR="1")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "tests/test_gpu_gemm.py",
         "tests/test_gpu_llm_configs.py", "-k", "not C3 and not persistent"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=1500)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
