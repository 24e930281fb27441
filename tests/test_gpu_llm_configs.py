"""LLM-driver parity on the benchmark's model configurations.

- C3 as the benchmark runs it: 6 layers, d_model 512, 8 heads (Dh 64), GELU
  MLP 4x, vocab 32000, tied embeddings, fp16 weights ~N(0, 0.02), eps 1e-5,
  RoPE base 1e4; a 128-token prompt, then 256 greedy decode steps, batch 1.
- C4 and C5 at full width with 2 of their layers (bf16, Dh 128, untied head;
  C5 has vocab 128256 and therefore 32-bit ids): a prompt, then 8 decode steps.

Protocol and tolerances: tests/llm_parity.py (teacher-forced against the
oracle decoder; ids bit-exact except where the oracle's top-2 logit gap is
within twice the step's logit error; the fused-argmax CUDA-graph ids equal the
logits path's ids).
"""
import numpy as np
import pytest

import oracle
from llm_parity import load_weights, teacher_forced_parity
from llm_ref import RefModel

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CONFIGS = {
    # name: (layers, D, H, F, V, tied, dtype, B, S, steps)
    "C3": (6, 512, 8, 2048, 32000, True, 0, 1, 128, 256),
    "C4-2L": (2, 2048, 16, 8192, 32000, False, 1, 4, 128, 8),
    "C5-2L": (2, 4096, 32, 14336, 128256, False, 1, 2, 64, 8),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_llm_config_greedy_vs_oracle(name):
    import evk_b200

    L, D, H, F, V, tied, dt, B, S, steps = CONFIGS[name]
    evk_b200.init(0)
    tdt = torch.float16 if dt == 0 else torch.bfloat16
    ref = RefModel(L, D, H, F, V, tied, dtype=dt, seed=42)
    max_len = S + steps + 1
    m = evk_b200.Llm(L, D, H, F, V, B, max_len, dtype=dt, tied_embeddings=tied)
    try:
        load_weights(m, ref, tdt)
        prompt = oracle.uniform_ids(B * S, 7, 0, V, 4).astype(np.int64).reshape(B, S)
        stats = teacher_forced_parity(ref, m, prompt, steps, dt, tdt, max_len, name)
    finally:
        m.close()
    assert stats["checked"] == B * (steps + 1)
    evk_b200.check_device_error()


def test_c3_persistent_decode_step_vs_oracle(monkeypatch):
    """The persistent one-kernel decode step (opt-in, EVKCU_DECODE_MEGA=1 at
    model creation) on the C3 model: same protocol as above (32 steps)."""
    import evk_b200

    monkeypatch.setenv("EVKCU_DECODE_MEGA", "1")
    L, D, H, F, V, tied, dt, B, S, _ = CONFIGS["C3"]
    steps = 32
    evk_b200.init(0)
    ref = RefModel(L, D, H, F, V, tied, dtype=dt, seed=42)
    max_len = S + steps + 1
    m = evk_b200.Llm(L, D, H, F, V, B, max_len, dtype=dt, tied_embeddings=tied)
    try:
        load_weights(m, ref, torch.float16)
        prompt = oracle.uniform_ids(B * S, 7, 0, V, 4).astype(np.int64).reshape(B, S)
        stats = teacher_forced_parity(ref, m, prompt, steps, dt, torch.float16, max_len, "C3 persistent step")
    finally:
        m.close()
    assert stats["checked"] == B * (steps + 1)
    evk_b200.check_device_error()
