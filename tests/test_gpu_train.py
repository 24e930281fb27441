"""GPU parity of the training-side kernels (backward passes, losses,
optimisers, flash-attention backward) through the C ABI against the CPU
oracle's restatements of the reference shaders, on seeded inputs in both
storage types.  The oracle side is pinned by the reference's own
example/tests.h (tests/test_oracle_kats.py).

Tolerances: elementwise ops that read and write the same element once are
compared with the usual 2e-2 + 1 ulp / rel-L2 1e-3 bar (fp16; bf16 rel-L2
4e-3); index and order-defined work (embed_backward) bit-exact; the
reductions (softmax / rms_norm backward, losses) and the attention backward,
whose summation order differs from the oracle's fp64 sums, at rel-L2 2e-3
(fp16) / 8e-3 (bf16) with the same elementwise bound.
"""
import numpy as np
import pytest

import oracle
from conftest import assert_close, dcode, dev, u16

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
DTYPES = [torch.float16, torch.bfloat16]


@pytest.fixture(autouse=True, scope="module")
def _init():
    import evk_b200

    evk_b200.init(0)
    yield
    evk_b200.check_device_error()


def ev():
    import evk_b200

    return evk_b200


def rel(dt):
    return 1e-3 if dt == 0 else 4e-3


def rel_red(dt):
    return 2e-3 if dt == 0 else 8e-3


def close(got, ref, dt, what, rel_l2=None):
    assert_close(u16(got).ravel(), ref.ravel(), dt, rel_l2=rel_l2 or rel(dt), what=what)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 1000, 65537])
def test_relu_gelu_backward(dtype, n):
    dt = dcode(dtype)
    x, go, gi = oracle.normal(n, 1, dtype=dt), oracle.normal(n, 2, dtype=dt), oracle.normal(n, 3, dtype=dt)
    out = torch.empty(n, dtype=dtype, device="cuda")
    ev().relu(dev(x, dtype), out)
    r = np.empty_like(x)
    oracle.relu(x, r, dt)
    assert np.array_equal(u16(out).ravel(), r), "relu is exact"
    g = dev(gi, dtype)
    ev().relu_backward(dev(go, dtype), dev(x, dtype), g)
    r = gi.copy()
    oracle.relu_backward(go, x, r, dt)
    assert np.array_equal(u16(g).ravel(), r), "relu_backward is exact"
    g = dev(gi, dtype)
    ev().gelu_backward(dev(go, dtype), dev(x, dtype), g)
    r = gi.copy()
    oracle.gelu_backward(go, x, r, dt)
    close(g, r, dt, "gelu_backward")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,L", [(1, 7), (5, 128), (33, 1000)])
def test_softmax_and_rms_norm_backward(dtype, rows, L):
    dt = dcode(dtype)
    x = oracle.normal(rows * L, 4, dtype=dt)
    p = np.empty_like(x)
    oracle.softmax(x, p, rows, L, 0.5, dt)
    g, gi = oracle.normal(rows * L, 5, dtype=dt), oracle.normal(rows * L, 6, 0.1, dtype=dt)
    t = dev(gi, dtype).view(rows, L)
    ev().softmax_backward(dev(p, dtype).view(rows, L), dev(g, dtype).view(rows, L), t, 0.5)
    r = gi.copy()
    oracle.softmax_backward(p, g, r, rows, L, 0.5, dt)
    close(t, r, dt, "softmax_backward", rel_red(dt))
    t = dev(gi, dtype).view(rows, L)
    ev().rms_norm_backward(dev(x, dtype).view(rows, L), dev(g, dtype).view(rows, L), t, 1e-5)
    r = gi.copy()
    oracle.rms_norm_backward(x, g, r, rows, L, 1e-5, dt)
    close(t, r, dt, "rms_norm_backward", rel_red(dt))


@pytest.mark.parametrize("dtype", DTYPES)
def test_rope_position_sum_batch(dtype):
    dt = dcode(dtype)
    B, S, D = 3, 17, 64
    go, gi = oracle.normal(B * S * D, 7, dtype=dt), oracle.normal(B * S * D, 8, dtype=dt)
    t = dev(gi, dtype)
    ev().rope_backward(dev(go, dtype), t, B, S, D, 10000.0)
    r = gi.copy()
    oracle.rope_backward(go, r, B, S, D, 10000.0, dt)
    close(t, r, dt, "rope_backward")
    x, pos = oracle.normal(B * S * D, 9, dtype=dt), oracle.normal(S * D, 10, dtype=dt)
    out = torch.empty(B * S * D, dtype=dtype, device="cuda")
    ev().position_add(dev(x, dtype), dev(pos, dtype), out, B, S, D)
    r = np.empty_like(x)
    oracle.position_add(x, pos, r, B, S, D, dt)
    assert np.array_equal(u16(out).ravel(), r), "position_add is exact"
    gp0 = oracle.normal(S * D, 11, dtype=dt)
    ti, tp = dev(gi, dtype), dev(gp0, dtype)
    ev().position_add_backward(dev(go, dtype), ti, tp, B, S, D)
    ri, rp = gi.copy(), gp0.copy()
    oracle.position_add_backward(go, ri, rp, B, S, D, dt)
    assert np.array_equal(u16(ti).ravel(), ri)
    close(tp, rp, dt, "position_add_backward(pos)")
    out0 = oracle.normal(S * D, 12, dtype=dt)
    to = dev(out0, dtype)
    ev().sum_batch(dev(go, dtype), to, B, S * D)
    r = out0.copy()
    oracle.sum_batch(go, r, B, S * D, dt)
    close(to, r, dt, "sum_batch")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ib", [2, 4])
def test_embed_backward_exact(dtype, ib):
    dt = dcode(dtype)
    V, D, n = 50, 72, 300  # many repeated ids: order of the rounded adds matters
    ids = oracle.uniform_ids(n, 13, 0, V, ib)
    go, gE = oracle.normal(n * D, 14, dtype=dt), oracle.normal(V * D, 15, dtype=dt)
    t = dev(gE, dtype).view(V, D)
    tids = torch.from_numpy(ids.view(np.int16 if ib == 2 else np.int32)).cuda()
    ev().embed_backward(dev(go, dtype).view(n, D), tids, t)
    r = gE.copy()
    oracle.embed_backward(go, ids, r, V, D, dt)
    assert np.array_equal(u16(t).ravel(), r), "embed_backward keeps the index order of the rounded adds"


@pytest.mark.parametrize("dtype", DTYPES)
def test_sgd_and_adam_steps(dtype):
    dt = dcode(dtype)
    n = 4099
    p0, g = oracle.normal(n, 16, dtype=dt), oracle.normal(n, 17, dtype=dt)
    t = dev(p0, dtype)
    ev().sgd(t, dev(g, dtype), 0.01)
    r = p0.copy()
    oracle.sgd(r, g, 0.01, dt)
    close(t, r, dt, "sgd")
    # three Adam steps on the same state, fresh gradients each step
    tp, tm, tv = dev(p0, dtype), torch.zeros(n, dtype=dtype, device="cuda"), torch.zeros(n, dtype=dtype, device="cuda")
    rp, rm, rv = p0.copy(), np.zeros(n, np.uint16), np.zeros(n, np.uint16)
    for step in range(1, 4):
        gs = oracle.normal(n, 100 + step, dtype=dt)
        ev().adam(tp, dev(gs, dtype), tm, tv, step, 1e-2)
        oracle.adam(rp, gs, rm, rv, step, 1e-2, dtype=dt)
    close(tp, rp, dt, "adam param")
    close(tm, rm, dt, "adam m")
    close(tv, rv, dt, "adam v")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,V,ignored", [(4, 10, 0), (37, 1000, 5), (3, 32000, 1), (2, 64, 2)])
def test_losses(dtype, rows, V, ignored):
    dt = dcode(dtype)
    n = rows * 33
    p, tg = oracle.normal(n, 18, dtype=dt), oracle.normal(n, 19, dtype=dt)
    grad, res = torch.empty(n, dtype=dtype, device="cuda"), torch.empty(1, dtype=dtype, device="cuda")
    ev().mse_loss(dev(p, dtype), dev(tg, dtype), grad, res)
    rg, rr = np.empty_like(p), np.empty(1, np.uint16)
    oracle.mse_loss(p, tg, rg, rr, dt)
    close(grad, rg, dt, "mse grad")
    close(res, rr, dt, "mse loss", rel_red(dt))
    logits = oracle.normal(rows * V, 20, 2.0, dtype=dt)
    tgt = oracle.uniform_ids(rows, 21, 1, V, 4)
    tgt[:ignored] = 0  # ignored positions (all of them when ignored == rows)
    for tb in (2, 4):
        t = tgt.astype(np.uint16 if tb == 2 else np.uint32)
        tt = torch.from_numpy(t.view(np.int16 if tb == 2 else np.int32)).cuda()
        grad = torch.empty(rows, V, dtype=dtype, device="cuda")
        res = torch.empty(1, dtype=dtype, device="cuda")
        ev().cross_entropy_loss(dev(logits, dtype).view(rows, V), tt, grad, res)
        rg, rr = np.empty(rows * V, np.uint16), np.empty(1, np.uint16)
        oracle.cross_entropy_loss(logits, t, rg, rr, rows, V, dt)
        close(grad, rg, dt, "cross-entropy grad", rel_red(dt))
        close(res, rr, dt, "cross-entropy loss", rel_red(dt))
        if ignored:
            assert not torch.any(grad[:ignored].float() != 0), "ignored rows get zero gradient"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,N,H,Hkv,Dh,flags", [
    (1, 16, 2, 1, 16, 0),    # the reference's test shape (MQA, non-causal)
    (2, 48, 4, 1, 32, 0),    # MQA, ragged tile
    (1, 70, 4, 2, 64, 1),    # GQA, causal
    (2, 64, 2, 2, 64, 2),    # MHA, exact (normalised) softmax gradient
    (1, 33, 2, 2, 128, 3),   # Dh 128, causal + normalised
])
def test_flash_attention_bwd(dtype, B, N, H, Hkv, Dh, flags):
    dt = dcode(dtype)
    q, dO = oracle.normal(B * N * H * Dh, 22, dtype=dt), oracle.normal(B * N * H * Dh, 23, dtype=dt)
    k, v = oracle.normal(B * N * Hkv * Dh, 24, dtype=dt), oracle.normal(B * N * Hkv * Dh, 25, dtype=dt)
    tq, tk, tv, tdo = (dev(a, dtype) for a in (q, k, v, dO))
    tq, tdo = tq.view(B, N, H * Dh), tdo.view(B, N, H * Dh)
    tk, tv = tk.view(B, N, Hkv * Dh), tv.view(B, N, Hkv * Dh)
    o = torch.zeros_like(tq)
    dQ, dK, dV = torch.empty_like(tq), torch.empty_like(tk), torch.empty_like(tv)
    ev().flash_attention_bwd(tq, tk, tv, o, tdo, dQ, dK, dV, heads=H, causal=bool(flags & 1),
                             normalized=bool(flags & 2))
    rq, rk, rv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    oracle.flash_attention_bwd(q, k, v, dO, rq, rk, rv, B, N, H, Hkv, Dh, 0.0, flags, dt)
    close(dQ, rq, dt, "dQ", rel_red(dt))
    close(dK, rk, dt, "dK", rel_red(dt))
    close(dV, rv, dt, "dV", rel_red(dt))


def test_flash_attention_bwd_normalized_matches_torch_autograd():
    """With EVKCU_ATTN_BWD_NORMALIZED the gradients are the exact softmax
    attention gradients: compare with torch autograd in fp32."""
    B, N, H, Dh = 2, 96, 4, 64
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v, dO = (torch.randn(B, N, H * Dh, device="cuda", generator=g).half() for _ in range(4))
    dQ, dK, dV = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ev().flash_attention_bwd(q, k, v, torch.zeros_like(q), dO, dQ, dK, dV, heads=H, causal=True, normalized=True)
    qf, kf, vf = (t.float().view(B, N, H, Dh).transpose(1, 2).requires_grad_() for t in (q, k, v))
    out = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True)
    out.backward(dO.float().view(B, N, H, Dh).transpose(1, 2))
    for got, ref in ((dQ, qf.grad), (dK, kf.grad), (dV, vf.grad)):
        ref = ref.transpose(1, 2).reshape(B, N, H * Dh)
        r = ((got.float() - ref).norm() / ref.norm()).item()
        assert r <= 2e-3, r
