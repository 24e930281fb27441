"""The reference's own known-answer tests (carloshgsilva/evk
example/tests.h), restated against the CPU oracle, plus the harness binary
that compiles the reference's tests.h itself against the oracle."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from conftest import ROOT

f16 = lambda x: oracle.from_float(np.asarray(x, np.float32))  # noqa: E731
flt = lambda a: oracle.to_float(a)  # noqa: E731


def test_add_exact():  # tests.h:139-161
    a = f16([0, 1, 2, 3])
    b = f16([0, 2, 4, 6])
    c = np.empty(4, np.uint16)
    oracle.add(a, b, c)
    assert np.array_equal(c, f16([0, 3, 6, 9]))


def identity(n, val):
    x = np.zeros(n * n, np.float32)
    x[:: n + 1] = val  # i % (shape[0]+1) == 0, evk_ai.h:296-303
    return f16(x)


def test_matmul_identity_400():  # tests.h:163-194
    n = 400
    a, b = identity(n, 2.0), identity(n, 2.0)
    c = np.empty(n * n, np.uint16)
    oracle.matmul(a, b, c, 1, n, n, n, n * n, n * n, n * n, 0)
    expect = identity(n, 4.0)
    assert np.array_equal(c, expect)


def test_matmul_broadcast():  # tests.h:196-219
    B, M, K, N = 3, 32, 32, 32
    a = f16(np.ones(M * K))
    b = identity(K, 1.0)
    c = np.empty(B * M * N, np.uint16)
    oracle.matmul(a, b, c, B, M, K, N, 0, 0, M * N, 0)
    assert np.all(flt(c) == 1.0)


def test_softmax_rows_and_mask():  # tests.h:619-679
    x = f16(np.tile(np.arange(5, dtype=np.float32) - 2, 6))
    y = np.empty_like(x)
    oracle.softmax(x, y, 6, 5, 1.0)
    assert np.all(np.abs(flt(y).reshape(6, 5).sum(1) - 1) <= 5e-3)
    m = f16([0.0, -65504.0, 1.0, -65504.0])
    o = np.empty_like(m)
    oracle.softmax(m, o, 1, 4, 1e-5)
    p = flt(o)
    assert p[1] == 0 and p[3] == 0 and abs(p[0] + p[2] - 1) <= 5e-3 and p[0] > 0.49 and p[2] > 0.49


def gelu_ref(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def test_gelu_points():  # tests.h:1169-1197
    x = f16([-1.0, 0.0, 1.0])
    y = np.empty_like(x)
    oracle.gelu(x, y)
    assert np.all(np.abs(flt(y) - gelu_ref(np.array([-1.0, 0.0, 1.0]))) <= 2e-2)


def test_rope_b1_n2_d4():  # tests.h:1318-1356
    xin = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32)
    y = np.empty(8, np.uint16)
    oracle.rope(f16(xin), y, 1, 2, 4, 0, 0, 10000.0)
    got = flt(y)
    for t in range(2):
        for p in range(2):
            i = t * 4 + 2 * p
            ang = t * 10000.0 ** (-2 * p / 4)
            c, s = np.cos(ang), np.sin(ang)
            assert abs(got[i] - (xin[i] * c - xin[i + 1] * s)) <= 3e-2
            assert abs(got[i + 1] - (xin[i] * s + xin[i + 1] * c)) <= 3e-2


def test_rms_norm_2x4():  # tests.h:1411-1444
    xin = np.array([3, 4, 0, 0, 1, 2, 3, 4], np.float32)
    y = np.empty(8, np.uint16)
    oracle.rms_norm(f16(xin), y, 2, 4, 1e-4)
    x = xin.reshape(2, 4)
    exp = x / np.sqrt((x ** 2).mean(1, keepdims=True) + 1e-4)
    assert np.all(np.abs(flt(y) - exp.ravel()) <= 3e-2)


def test_greedy_sample_ids():  # tests.h:1472-1497
    l = np.full(20, -10.0, np.float32)
    l[(0 * 2 + 1) * 5 + 1], l[(0 * 2 + 1) * 5 + 2], l[(0 * 2 + 1) * 5 + 3] = 0.5, 2.5, 1.5
    l[(1 * 2 + 1) * 5 + 1], l[(1 * 2 + 1) * 5 + 2], l[(1 * 2 + 1) * 5 + 3] = 3.0, 2.0, 1.0
    out = np.zeros(2, np.uint16)
    oracle.greedy_sample(f16(l), out, 2, 2, 5, 1, 1, 3)
    assert out.tolist() == [2, 1]


def test_embed_rows():  # tests.h:1224-1252
    E = f16(np.arange(1, 13, dtype=np.float32))
    idx = np.array([1, 3], np.uint16)
    out = np.empty(6, np.uint16)
    oracle.embed(E, idx, out, 4, 3)
    assert np.array_equal(flt(out), np.array([4, 5, 6, 10, 11, 12], np.float32))


HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_tests_oracle")


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="reference harness not built (needs the reference checkout)")
def test_reference_tests_h_against_oracle():
    r = subprocess.run([HARNESS], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "[FAIL]" not in r.stdout
    assert "ALL REFERENCE KATS PASSED" in r.stdout
