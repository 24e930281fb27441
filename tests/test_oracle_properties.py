"""CPU checks of the oracle and of the host-side algorithms the kernels use.

* the fp16 / bf16 quantisers against numpy / torch on normal values, plus the
  reference quantiser's half-up subnormal rule (evk_ai.h:113-117);
* matmul / attention / row ops against independent numpy formulas;
* greedy_sample: the CUDA kernel's one-pass 64-bit key (value, bit-reversed
  lane rank) against the reference's literal 256-lane scan + tree, on
  adversarial ties, NaN and -inf (bit-exact ids).
"""
import numpy as np
import pytest

import oracle
from conftest import assert_close

rng = np.random.default_rng(1234)


def test_f16_normals_match_numpy():
    x = rng.standard_normal(200000).astype(np.float32) * 100
    got = oracle.from_float(x, 0)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


def test_f16_subnormal_half_up():
    # 2^-24 * 1.5 is a tie between subnormals 1 and 2 -> half-up gives 2
    # (numpy's round-to-even also gives 2); 2^-24 * 2.5 -> half-up gives 3,
    # round-to-even would give 2; values below 2^-24 flush to zero (the
    # reference tests the exponent before rounding), where RNE would give 1.
    v = np.array([2.0 ** -24 * 1.5, 2.0 ** -24 * 2.5, 2.0 ** -24 * 0.75], np.float32)
    got = oracle.from_float(v, 0)
    assert got.tolist() == [2, 3, 0]


def test_bf16_matches_torch():
    import torch

    x = rng.standard_normal(100000).astype(np.float32) * 1e3
    got = oracle.from_float(x, 1)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("ta,tb,acc", [(0, 0, 0), (1, 0, 0), (0, 1, 1), (1, 1, 0)])
def test_matmul_vs_numpy(ta, tb, acc):
    B, M, K, N = 2, 24, 40, 16
    A = oracle.normal(B * M * K, 1)
    Bm = oracle.normal(B * K * N, 2)
    C0 = oracle.normal(B * M * N, 3)
    C = C0.copy()
    flags = ta | (tb << 1) | (acc << 2)
    oracle.matmul(A, Bm, C, B, M, K, N, M * K, K * N, M * N, flags)
    a = oracle.to_float(A).reshape(B, *((K, M) if ta else (M, K))).astype(np.float64)
    b = oracle.to_float(Bm).reshape(B, *((N, K) if tb else (K, N))).astype(np.float64)
    a = a.transpose(0, 2, 1) if ta else a
    b = b.transpose(0, 2, 1) if tb else b
    ref = a @ b + (oracle.to_float(C0).reshape(B, M, N) if acc else 0)
    assert np.array_equal(C, oracle.from_float(ref.astype(np.float32).ravel()))


def np_attention(q, k, v, B, N, H, Hkv, Dh, causal):
    q = q.reshape(B, N, H, Dh).astype(np.float64)
    k = k.reshape(B, N, Hkv, Dh).astype(np.float64)
    v = v.reshape(B, N, Hkv, Dh).astype(np.float64)
    out = np.zeros((B, N, H, Dh))
    for h in range(H):
        g = h // (H // Hkv)
        s = np.einsum("bid,bjd->bij", q[:, :, h], k[:, :, g]) / np.sqrt(Dh)
        if causal:
            s = np.where(np.tril(np.ones((N, N), bool)), s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        out[:, :, h] = np.einsum("bij,bjd->bid", p, v[:, :, g])
    return out.ravel()


@pytest.mark.parametrize("causal,H,Hkv", [(False, 4, 1), (True, 4, 4), (True, 4, 2)])
def test_flash_vs_numpy(causal, H, Hkv):
    B, N, Dh = 2, 37, 32
    q = oracle.normal(B * N * H * Dh, 5)
    k = oracle.normal(B * N * Hkv * Dh, 6)
    v = oracle.normal(B * N * Hkv * Dh, 7)
    o = np.empty_like(q)
    oracle.flash_attention(q, k, v, o, B, N, H, Hkv, Dh, 0.0, int(causal))
    ref = np_attention(oracle.to_float(q), oracle.to_float(k), oracle.to_float(v), B, N, H, Hkv, Dh, causal)
    # the oracle scales by the fp32 value of 1/sqrt(Dh): at most one fp16 ulp apart
    assert_close(o, oracle.from_float(ref.astype(np.float32)), max_abs=0, rel_l2=1e-4, ulps=1.0)


def test_single_query_equals_last_causal_row():
    B, L, H, Dh = 2, 29, 4, 64
    q = oracle.normal(B * L * H * Dh, 11)
    k = oracle.normal(B * L * H * Dh, 12)
    v = oracle.normal(B * L * H * Dh, 13)
    o = np.empty_like(q)
    oracle.flash_attention(q, k, v, o, B, L, H, H, Dh, 0.0, 1)
    qlast = q.reshape(B, L, H * Dh)[:, -1].copy()
    out = np.empty(B * H * Dh, np.uint16)
    oracle.single_query_attention(qlast, k, v, out, B, H, H, Dh, L, L)
    assert np.array_equal(out, o.reshape(B, L, H * Dh)[:, -1].ravel())


# ------------------------------------------------------------ greedy model --
def bitrev8(x):
    return int(f"{x:08b}"[::-1], 2)


def greedy_key_model(vals, base, count):
    """The CUDA kernel's selection rule (ops_sample.cu) in numpy."""
    best, tok = None, base
    for j in range(count):
        v = vals[base + j]
        if not (v > -np.finfo(np.float32).max):
            continue
        key = (float(v), -(bitrev8(j & 255) * (1 << 24) + (j >> 8)))
        if best is None or key > best:
            best, tok = key, base + j
    return tok


@pytest.mark.parametrize("case", range(12))
def test_greedy_key_rule_matches_reference_tree(case):
    r = np.random.default_rng(case)
    V = int(r.integers(300, 3000))
    base = int(r.integers(0, 50))
    count = int(r.integers(1, V - base))
    # few distinct values -> many ties across lanes and within a lane
    vals = r.integers(-3, 3, size=V).astype(np.float32)
    if case % 3 == 1:
        vals[r.integers(0, V, 20)] = np.nan
    if case % 3 == 2:
        vals[:] = -np.inf
        vals[r.integers(0, V, 5)] = 1.0
    if case == 11:
        vals[:] = np.nan  # nothing selectable -> token_base
    logits = oracle.from_float(vals)
    out = np.zeros(1, np.uint32)
    oracle.greedy_sample(logits, out, 1, 1, V, 0, base, count)
    model = greedy_key_model(oracle.to_float(logits), base, count)
    assert int(out[0]) == model


def test_fill_normal_is_deterministic_and_normal():
    a = oracle.normal(1 << 20, 42)
    b = oracle.normal(1 << 20, 42)
    assert np.array_equal(a, b)
    x = oracle.to_float(a)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
