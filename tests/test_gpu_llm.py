"""GPU parity of the LLM driver (evkcu_llm_*) against a decoder composed from
the CPU oracle's ops (tests/llm_ref.py): prefill logits and greedy ids, then
free-running decode steps (eager first step, CUDA-graph replays after) whose
logits and ids are checked against a full-sequence recompute of the same
prefix.

Greedy ids are compared bit-exactly wherever the oracle's top-2 logit gap
exceeds the logit tolerance; closer calls may legitimately flip on
accumulation-order differences and are counted, with their gaps, instead.
"""
import numpy as np
import pytest

import oracle
from conftest import dev, u16
from llm_ref import RefModel

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def build(tied, dtype, layers=2, D=256, H=4, F=512, V=1000, max_batch=2, max_seq=64):
    import evk_b200

    evk_b200.init(0)
    tdt = torch.float16 if dtype == 0 else torch.bfloat16
    ref = RefModel(layers, D, H, F, V, tied, dtype=dtype)
    m = evk_b200.Llm(layers, D, H, F, V, max_batch, max_seq, dtype=dtype, tied_embeddings=tied)
    m.set_weight("embedding", dev(ref.emb, tdt))
    if not tied:
        m.set_weight("lm_head", dev(ref.lm_head, tdt))
    for l, w in enumerate(ref.w):
        for n in ("wqkv", "wo", "w1", "w2"):
            m.set_weight(n, dev(w[n], tdt), layer=l)
    # set_weight copies on the default stream; the tests then run on their
    # own (non-blocking) streams.
    torch.cuda.synchronize()
    return ref, m, tdt


def check_step(ref, tokens, got_logits, got_ids, dtype, stats):
    rl = ref.forward_last_logits(tokens)
    rid = ref.greedy(rl)
    g = oracle.to_float(u16(got_logits).ravel(), dtype).reshape(rl.shape).astype(np.float64)
    r = oracle.to_float(rl.ravel(), dtype).reshape(rl.shape).astype(np.float64)
    err = np.abs(g - r).max()
    rel = np.linalg.norm(g - r) / np.linalg.norm(r)
    assert rel <= (5e-3 if dtype == 0 else 2e-2), f"logits rel-L2 {rel:.3g}"
    tol = max(4 * err, 1e-3)
    for b in range(rl.shape[0]):
        top2 = np.sort(r[b])[-2:]
        gap = top2[1] - top2[0]
        if got_ids[b] != rid[b]:
            assert gap <= tol, f"greedy id {got_ids[b]} != oracle {rid[b]} with top-2 gap {gap:.4g} > tol {tol:.4g}"
            stats["close_calls"] += 1
        stats["checked"] += 1


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("tied", [True, False])
def test_llm_prefill_and_decode_vs_oracle(tied, dtype):
    ref, m, tdt = build(tied, dtype)
    B, S, steps = 2, 24, 6
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, ref.V, size=(B, S)).astype(np.int32)
    tokens = torch.from_numpy(prompt).cuda()
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, ref.V, dtype=tdt, device="cuda")
    stream = torch.cuda.Stream()
    stats = {"checked": 0, "close_calls": 0}
    with torch.cuda.stream(stream):
        m.prefill(tokens, nxt, logits, stream=stream)
    torch.cuda.synchronize()
    seq = prompt.copy()
    check_step(ref, seq, logits, nxt.cpu().numpy(), dtype, stats)
    cur = nxt.clone()
    for step in range(steps):
        seq = np.concatenate([seq, cur.cpu().numpy().reshape(B, 1)], axis=1)
        out = torch.zeros(B, dtype=torch.int32, device="cuda")
        with torch.cuda.stream(stream):
            m.decode(cur, out, logits, stream=stream)  # with logits: eager path
        torch.cuda.synchronize()
        check_step(ref, seq, logits, out.cpu().numpy(), dtype, stats)
        cur = out
    assert m.length == S + steps
    assert stats["close_calls"] <= 2, stats
    m.close()


def test_llm_graph_decode_matches_eager():
    """The captured CUDA-graph decode reproduces the eager decode bit-exactly."""
    runs = []
    for graph in (False, True):
        ref, m, tdt = build(True, 0)
        B, S = 2, 16
        prompt = torch.from_numpy(np.random.default_rng(9).integers(0, ref.V, size=(B, S)).astype(np.int32)).cuda()
        nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
        stream = torch.cuda.Stream()
        ids = []
        with torch.cuda.stream(stream):
            m.prefill(prompt, nxt, stream=stream)
            cur = nxt.clone()
            for _ in range(12):
                out = torch.zeros(B, dtype=torch.int32, device="cuda")
                if graph:
                    m.decode(cur, out, stream=stream)
                else:
                    scratch = torch.empty(B, ref.V, dtype=tdt, device="cuda")
                    m.decode(cur, out, scratch, stream=stream)  # logits requested: eager every step
                cur = out
                ids.append(out)
        torch.cuda.synchronize()
        runs.append(torch.stack(ids).cpu().numpy())
        m.close()
    assert np.array_equal(runs[0], runs[1]), (runs[0], runs[1])


def test_llm_random_init_is_deterministic():
    import evk_b200

    evk_b200.init(0)
    outs = []
    for _ in range(2):
        m = evk_b200.Llm(2, 256, 4, 512, 1000, 1, 32)
        m.init_random(seed=11, std=0.02)
        tok = torch.arange(8, dtype=torch.int32, device="cuda").view(1, 8)
        nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
        lg = torch.empty(1, 1000, dtype=torch.float16, device="cuda")
        m.prefill(tok, nxt, lg)
        torch.cuda.synchronize()
        outs.append(lg.clone())
        m.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("tied", [True, False])
def test_llm_fused_head_argmax_vs_oracle(tied):
    """Without logits the LM-head GEMV reduces its outputs to greedy keys
    (fused argmax).  Its ids must equal the logits + greedy_sample path's bit
    for bit, and the oracle's greedy ids (teacher-forced, gap rule of
    tests/llm_parity.py), prefill and decode."""
    import evk_b200
    from llm_parity import load_weights, teacher_forced_parity

    evk_b200.init(0)
    V = 4000  # 32 slabs of 128 columns, a ragged last one
    ref = RefModel(2, 256, 4, 512, V, tied, dtype=1, seed=21, std=0.05)
    m = evk_b200.Llm(2, 256, 4, 512, V, 3, 48, dtype=1, tied_embeddings=tied)
    load_weights(m, ref, torch.bfloat16)
    prompt = np.random.default_rng(4).integers(0, V, size=(3, 20))
    stats = teacher_forced_parity(ref, m, prompt, 5, 1, torch.bfloat16, 48, f"fused-head tied={tied}")
    m.close()
    assert stats["fused_ids_equal_oracle"] + len(stats["close_calls"]) == stats["checked"]


@pytest.mark.parametrize("dtype", [0, 1])
def test_llm_tile_aligned_prefill_vs_oracle(dtype):
    """A prompt of 128 tokens puts every 128-row GEMM tile inside one sequence,
    so the fused QKV projection takes the staged (TMA) epilogue that stores
    q and the K / V cache rows by tile; prefill and the decode steps that read
    that cache must still match the oracle."""
    ref, m, tdt = build(False, dtype, max_seq=160)
    B, S, steps = 2, 128, 3
    prompt = np.random.default_rng(12).integers(0, ref.V, size=(B, S)).astype(np.int32)
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, ref.V, dtype=tdt, device="cuda")
    stream = torch.cuda.Stream()
    stats = {"checked": 0, "close_calls": 0}
    with torch.cuda.stream(stream):
        m.prefill(torch.from_numpy(prompt).cuda(), nxt, logits, stream=stream)
    torch.cuda.synchronize()
    seq = prompt.copy()
    check_step(ref, seq, logits, nxt.cpu().numpy(), dtype, stats)
    cur = nxt.clone()
    for _ in range(steps):
        seq = np.concatenate([seq, cur.cpu().numpy().reshape(B, 1)], axis=1)
        out = torch.zeros(B, dtype=torch.int32, device="cuda")
        with torch.cuda.stream(stream):
            m.decode(cur, out, logits, stream=stream)
        torch.cuda.synchronize()
        check_step(ref, seq, logits, out.cpu().numpy(), dtype, stats)
        cur = out
    assert stats["close_calls"] <= 1, stats
    m.close()
