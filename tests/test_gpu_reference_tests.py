"""The drop-in boundary on the GPU: the reference's own tests and a Graph
program run through the C++ evk::ai layer (libevk_ai.so over libevkcu.so).

- evk_b200/reftests/ref_tests_cuda is the reference's example/tests.h
  compiled against this backend's evk.h / evk_ai.h (built at build time from
  the reference checkout; the binary travels with the package).  Its TEST()
  checks exit non-zero on the first failure.
- evk_b200/reftests/graph_attention_check builds a Graph with
  causal_attention + mse_loss, runs eval(backward = true) and one SGD step;
  the results are compared with the same computation composed from the CPU
  oracle's ops (fp16 intermediates rounded where the graph stores them).
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
from conftest import ROOT, assert_close

pytestmark = pytest.mark.gpu

REFTESTS = os.path.join(ROOT, "evk_b200", "reftests", "ref_tests_cuda")
GRAPH = os.path.join(ROOT, "evk_b200", "reftests", "graph_attention_check")


def _run(args, timeout=900):
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.skipif(not os.path.exists(REFTESTS), reason="ref_tests_cuda not built (needs the reference checkout)")
def test_reference_tests_h_through_the_cpp_layer():
    """tests.h:1565-1585 (run_ai_kernel_tests) plus the tests outside the
    default list, on the GPU through libevk_ai.so."""
    rc, out = _run([REFTESTS])
    assert rc == 0 and "REFERENCE TESTS PASSED" in out, out[-4000:]
    assert "[FAIL]" not in out
    assert out.count("[PASS]") >= 140, out[-2000:]


@pytest.mark.skipif(not os.path.exists(REFTESTS), reason="ref_tests_cuda not built (needs the reference checkout)")
def test_reference_flash_vs_unfused_through_the_cpp_layer():
    """tests.h:473-563: flash_attention vs matmul -> softmax -> matmul at
    N = 32768 (2 GB score matrices), through evk::ai on the GPU."""
    rc, out = _run([REFTESTS, "test_flash_attention_cmp_softmax"])
    assert rc == 0 and "REFERENCE TESTS PASSED" in out, out[-4000:]


def _graph_oracle(q, k, v, tgt, B, N, D):
    """The graph's computation from oracle ops, rounding where the graph
    stores a tensor (scores, probs, out, each gradient)."""
    dt = 0
    n = B * N * D
    scale = 1.0 / np.sqrt(D)
    scores = np.empty(B * N * N, np.uint16)
    oracle.matmul(q, k, scores, B, N, D, N, N * D, N * D, N * N, 2, dt)  # q k^T
    oracle.causal_mask(scores, B, N, dt)
    probs = np.empty_like(scores)
    oracle.softmax(scores, probs, B * N, N, scale, dt)
    out = np.empty(n, np.uint16)
    oracle.matmul(probs, v, out, B, N, N, D, N * N, N * D, N * D, 0, dt)
    dout, loss = np.empty(n, np.uint16), np.empty(1, np.uint16)
    oracle.mse_loss(out, tgt, dout, loss, dt)
    dprobs = np.empty_like(scores)
    oracle.matmul(dout, v, dprobs, B, N, D, N, N * D, N * D, N * N, 2, dt)  # dO v^T
    dv = np.zeros(n, np.uint16)
    oracle.matmul(probs, dout, dv, B, N, N, D, N * N, N * D, N * D, 1 | 4, dt)  # += P^T dO
    dscores = np.zeros_like(scores)
    oracle.softmax_backward(probs, dprobs, dscores, B * N, N, scale, dt)
    dq, dk = np.zeros(n, np.uint16), np.zeros(n, np.uint16)
    oracle.matmul(dscores, k, dq, B, N, N, D, N * N, N * D, N * D, 4, dt)  # += dS k
    oracle.matmul(dscores, q, dk, B, N, N, D, N * N, N * D, N * D, 1 | 4, dt)  # += dS^T q
    q2 = q.copy()
    oracle.sgd(q2, dq, 0.5, dt)
    return out, loss, dq, dk, dv, q2


@pytest.mark.skipif(not os.path.exists(GRAPH), reason="graph_attention_check not built")
@pytest.mark.parametrize("B,N,D", [(2, 64, 32), (1, 200, 64)])
def test_graph_causal_attention_eval_backward_vs_oracle(tmp_path, B, N, D):
    n = B * N * D
    q, k, v = (oracle.normal(n, s, 0.5) for s in (31, 32, 33))
    tgt = oracle.normal(n, 34, 20.0)  # large residuals keep the fp16 gradients out of the subnormal range
    fin, fout = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(fin, "wb") as f:
        f.write(np.array([B, N, D], np.uint32).tobytes())
        for a in (q, k, v, tgt):
            f.write(a.tobytes())
    rc, out = _run([GRAPH, str(fin), str(fout)], timeout=300)
    assert rc == 0 and "GRAPH_OK" in out, out[-3000:]
    got = np.fromfile(fout, np.uint16)
    assert got.size == 5 * n + 1, got.size
    o, loss, dq, dk, dv, q2 = (got[:n], got[n:n + 1], got[n + 1:2 * n + 1], got[2 * n + 1:3 * n + 1],
                               got[3 * n + 1:4 * n + 1], got[4 * n + 1:5 * n + 1])
    r = _graph_oracle(q, k, v, tgt, B, N, D)
    assert_close(o, r[0], 0, what="Graph out")
    assert_close(loss, r[1], 0, rel_l2=2e-3, what="Graph loss")
    # dv goes through one more fp16-stored tensor (dout).  dq and dk also go
    # through dP and dS = p (dP - sum p dP), whose cancellation turns a
    # 1-ulp difference in a stored dP into a larger relative one: 3e-2.
    assert_close(dv, r[4], 0, rel_l2=5e-3, what="Graph dv")
    for g, rr, name in ((dq, r[2], "dq"), (dk, r[3], "dk")):
        assert_close(g, rr, 0, rel_l2=3e-2, what=f"Graph {name}")
    assert_close(q2, r[5], 0, rel_l2=1e-3, what="q after Graph::step")


EXT = os.path.join(ROOT, "evk_b200", "reftests", "ext_check")


@pytest.mark.skipif(not os.path.exists(EXT), reason="ext_check not built")
def test_cpp_extensions_vs_oracle(tmp_path):
    """evk_ai_ext.h through libevk_ai.so (shapes in ext_check.cpp) against the
    oracle: bf16 GQA causal flash attention, decode attention, per-head RoPE
    with an offset, RMSNorm with a gain, and 32-bit ids for a 70,000-token
    vocabulary (embed and greedy_sample, bit-exact)."""
    bf = 1
    q1, k1, v1 = oracle.normal(160 * 256, 41, dtype=bf), oracle.normal(160 * 128, 42, dtype=bf), \
        oracle.normal(160 * 128, 43, dtype=bf)
    q2, kc, vc = oracle.normal(2 * 256, 44, dtype=bf), oracle.normal(2 * 100 * 128, 45, dtype=bf), \
        oracle.normal(2 * 100 * 128, 46, dtype=bf)
    x3 = oracle.normal(2 * 5 * 256, 47, dtype=bf)
    x4, g4 = oracle.normal(6 * 256, 48, dtype=bf), oracle.normal(256, 49, dtype=bf)
    E5 = oracle.normal(70000 * 16, 50)
    ids5 = oracle.uniform_ids(10, 51, 0, 70000, 4)
    l6 = oracle.normal(2 * 70000, 52, 3.0)
    fin, fout = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(fin, "wb") as f:
        for a in (q1, k1, v1, q2, kc, vc, x3, x4, g4, E5, ids5.view(np.uint16), l6):
            f.write(np.ascontiguousarray(a).tobytes())
    rc, out = _run([EXT, str(fin), str(fout)], timeout=300)
    assert rc == 0 and "EXT_OK" in out, out[-3000:]
    got = np.fromfile(fout, np.uint16)
    sizes = [160 * 256, 2 * 256, 2 * 5 * 256, 6 * 256, 10 * 16, 4]
    assert got.size == sum(sizes)
    parts, o = [], 0
    for s in sizes:
        parts.append(got[o:o + s])
        o += s
    r1 = np.empty_like(q1)
    oracle.flash_attention(q1, k1, v1, r1, 1, 160, 4, 2, 64, 0.0, 1, bf)
    assert_close(parts[0], r1, bf, rel_l2=8e-3, what="flash_attention_ex")
    r2 = np.empty_like(q2)
    oracle.single_query_attention(q2, kc, vc, r2, 2, 4, 2, 64, 100, 77, 0.0, bf)
    assert_close(parts[1], r2, bf, rel_l2=4e-3, what="single_query_attention")
    r3 = np.empty_like(x3)
    oracle.rope(x3, r3, 2, 5, 256, 64, 11, 10000.0, bf)
    assert_close(parts[2], r3, bf, rel_l2=4e-3, what="rope_ex")
    r4 = np.empty_like(x4)
    oracle.rms_norm(x4, r4, 6, 256, 1e-5, gamma=g4, dtype=bf)
    assert_close(parts[3], r4, bf, rel_l2=4e-3, what="rms_norm_ex")
    r5 = np.empty(10 * 16, np.uint16)
    oracle.embed(E5, ids5, r5, 70000, 16)
    assert np.array_equal(parts[4], r5), "embed_ex with 32-bit ids"
    r6 = np.zeros(2, np.uint32)
    oracle.greedy_sample(l6, r6, 2, 1, 70000, 0, 0, 70000, 0)
    assert np.array_equal(parts[5].view(np.uint32), r6), "greedy_sample_ex with 32-bit ids"
