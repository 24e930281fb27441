"""GPU parity of the bandwidth-bound ops through the C ABI against the CPU
oracle (seeded inputs, both storage types), plus the reference's own
known-answer vectors (example/tests.h) run on the GPU."""
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


f16 = lambda x: oracle.from_float(np.asarray(x, np.float32))  # noqa: E731


# ------------------------------------------------------- reference KATs ----
def test_kat_add():
    a, b = dev(f16([0, 1, 2, 3]), torch.float16), dev(f16([0, 2, 4, 6]), torch.float16)
    c = torch.empty_like(a)
    ev().add(a, b, c)
    torch.cuda.synchronize()
    assert np.array_equal(u16(c), f16([0, 3, 6, 9]))


def test_kat_softmax_masked():
    m = dev(f16([0.0, -65504.0, 1.0, -65504.0]), torch.float16).view(1, 4)
    o = torch.empty_like(m)
    ev().softmax(m, o, 1e-5)
    p = o.float().cpu().numpy().ravel()
    assert p[1] == 0 and p[3] == 0 and abs(p[0] + p[2] - 1) <= 5e-3 and p[0] > 0.49 and p[2] > 0.49


def test_kat_greedy():
    l = np.full(20, -10.0, np.float32)
    l[6], l[7], l[8] = 0.5, 2.5, 1.5
    l[16], l[17], l[18] = 3.0, 2.0, 1.0
    logits = dev(f16(l), torch.float16).view(2, 2, 5)
    out = torch.zeros(2, dtype=torch.int16, device="cuda")
    ev().greedy_sample(logits, out, 1, 1, 3)
    assert out.cpu().tolist() == [2, 1]


def test_kat_rms_rope_gelu_embed():
    x = dev(f16([3, 4, 0, 0, 1, 2, 3, 4]), torch.float16).view(2, 4)
    y = torch.empty_like(x)
    ev().rms_norm(x, y, 1e-4)
    xr = np.array([[3, 4, 0, 0], [1, 2, 3, 4]], np.float64)
    assert np.all(np.abs(y.float().cpu().numpy() - xr / np.sqrt((xr ** 2).mean(1, keepdims=True) + 1e-4)) <= 3e-2)
    r = dev(f16([1, 2, 3, 4, 5, 6, 7, 8]), torch.float16).view(1, 2, 4)
    ro = torch.empty_like(r)
    ev().rope(r, ro, 1, 2, 4, 10000.0)
    ref = np.empty(8, np.uint16)
    oracle.rope(f16([1, 2, 3, 4, 5, 6, 7, 8]), ref, 1, 2, 4)
    assert_close(u16(ro).ravel(), ref, what="rope kat")
    g = dev(f16([-1, 0, 1]), torch.float16)
    go = torch.empty_like(g)
    ev().gelu(g, go)
    gx = np.array([-1.0, 0, 1])
    assert np.all(np.abs(go.float().cpu().numpy() - 0.5 * gx * (1 + np.tanh(0.7978845608 * (gx + 0.044715 * gx ** 3)))) <= 2e-2)
    E = dev(f16(np.arange(1, 13)), torch.float16).view(4, 3)
    idx = torch.tensor([1, 3], dtype=torch.int16, device="cuda")
    eo = torch.empty(2, 3, dtype=torch.float16, device="cuda")
    ev().embed(E, idx, eo)
    assert eo.float().cpu().numpy().ravel().tolist() == [4, 5, 6, 10, 11, 12]


# ------------------------------------------------------ random parity ----
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [1, 7, 8, 1000, 65536 + 3])
def test_add_gelu_scale(dtype, n):
    dc = dcode(dtype)
    a, b = oracle.normal(n, 1, 2.0, dtype=dc), oracle.normal(n, 2, 2.0, dtype=dc)
    ta, tb = dev(a, dtype), dev(b, dtype)
    tc = torch.empty_like(ta)
    ev().add(ta, tb, tc)
    rc = np.empty_like(a)
    oracle.add(a, b, rc, dc)
    assert np.array_equal(u16(tc), rc), "add must be bit-exact (one fp32 add, one rounding)"
    tg = torch.empty_like(ta)
    ev().gelu(ta, tg)
    rg = np.empty_like(a)
    oracle.gelu(a, rg, dc)
    assert_close(u16(tg), rg, dc, max_abs=2e-3, what="gelu")
    ev().scale(ta, 0.37)
    oracle.scale(a, 0.37, dc)
    assert np.array_equal(u16(ta), a), "scale must be bit-exact"
    ev().zero(tb)
    assert torch.count_nonzero(tb).item() == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,D", [(1, 512), (5, 4), (33, 2048), (7, 100), (4, 4096), (300, 2048), (259, 4096), (256, 24)])
def test_rms_norm(dtype, rows, D):
    dc = dcode(dtype)
    x = oracle.normal(rows * D, 3, 3.0, dtype=dc)
    g = oracle.normal(D, 4, 1.0, 1.0, dtype=dc)
    t = dev(x, dtype).view(rows, D)
    o = torch.empty_like(t)
    ev().rms_norm(t, o, 1e-5)
    r = np.empty_like(x)
    oracle.rms_norm(x, r, rows, D, 1e-5, dtype=dc)
    assert_close(u16(o).ravel(), r, dc, what="rms_norm")
    tg = dev(g, dtype)
    ev().rms_norm(t, o, 1e-5, gamma=tg)
    oracle.rms_norm(x, r, rows, D, 1e-5, gamma=g, dtype=dc)
    assert_close(u16(o).ravel(), r, dc, what="rms_norm gamma")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,L,scale", [(1, 5, 1.0), (6, 128, 0.125), (3, 2049, 0.7), (64, 32000, 1.0)])
def test_softmax(dtype, rows, L, scale):
    dc = dcode(dtype)
    x = oracle.normal(rows * L, 5, 4.0, dtype=dc)
    xf = oracle.to_float(x, dc)
    xf[::7] = -65504.0  # masked entries
    x = oracle.from_float(xf, dc)
    t = dev(x, dtype).view(rows, L)
    o = torch.empty_like(t)
    ev().softmax(t, o, scale)
    r = np.empty_like(x)
    oracle.softmax(x, r, rows, L, scale, dc)
    assert_close(u16(o).ravel(), r, dc, max_abs=1e-4, what="softmax")
    assert np.all(u16(o).ravel()[::7] == 0) or dc == 1 and np.all(oracle.to_float(u16(o).ravel()[::7], dc) == 0)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,S,D,hd,off", [(1, 2, 4, 0, 0), (2, 128, 512, 0, 0), (1, 1, 512, 64, 300), (3, 17, 256, 128, 5), (1, 5, 6, 0, 2)])
def test_rope(dtype, B, S, D, hd, off):
    dc = dcode(dtype)
    x = oracle.normal(B * S * D, 6, 1.0, dtype=dc)
    t = dev(x, dtype).view(B, S, D)
    o = torch.empty_like(t)
    ev().rope(t, o, B, S, D, 10000.0, head_dim=hd, pos_offset=off)
    r = np.empty_like(x)
    oracle.rope(x, r, B, S, D, hd, off, 10000.0, dc)
    assert_close(u16(o).ravel(), r, dc, max_abs=2e-3, what="rope")


@pytest.mark.parametrize("dtype", DTYPES)
def test_causal_mask_and_embed(dtype):
    dc = dcode(dtype)
    B, N = 3, 67
    s = oracle.normal(B * N * N, 7, dtype=dc)
    t = dev(s, dtype).view(B, N, N)
    ev().apply_causal_mask(t)
    oracle.causal_mask(s, B, N, dc)
    assert np.array_equal(u16(t).ravel(), s)
    V, Dm = 1000, 72
    E = oracle.normal(V * Dm, 8, dtype=dc)
    for ib in (2, 4):
        ids = oracle.uniform_ids(257, 9, 0, V, ib)
        tids = torch.from_numpy(ids.view(np.int16 if ib == 2 else np.int32)).cuda()
        out = torch.empty(257, Dm, dtype=dtype, device="cuda")
        ev().embed(dev(E, dtype).view(V, Dm), tids, out)
        r = np.empty(257 * Dm, np.uint16)
        oracle.embed(E, ids, r, V, Dm)
        assert np.array_equal(u16(out).ravel(), r)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,S,V,pos,base,count", [(1, 1, 32000, 0, 0, 32000), (4, 3, 128256, 2, 0, 128256),
                                                  (2, 2, 5000, 1, 3, 4000), (16, 1, 128256, 0, 17, 100000),
                                                  (1, 1, 300, 0, 1, 1)])
@pytest.mark.parametrize("ties", [False, True])
def test_greedy_sample(dtype, B, S, V, pos, base, count, ties):
    dc = dcode(dtype)
    if ties:
        vals = np.random.default_rng(B + V).integers(-4, 4, size=B * S * V).astype(np.float32)
        l = oracle.from_float(vals, dc)
    else:
        l = oracle.normal(B * S * V, 10, 3.0, dtype=dc)
    t = dev(l, dtype).view(B, S, V)
    for ob, tdt, ndt in ((2, torch.int16, np.uint16), (4, torch.int32, np.uint32)):
        if ob == 2 and base + count > 65535:
            continue
        out = torch.zeros(B, dtype=tdt, device="cuda")
        ev().greedy_sample(t, out, pos, base, count)
        ref = np.zeros(B, ndt)
        oracle.greedy_sample(l, ref, B, S, V, pos, base, count, dc)
        got = out.cpu().numpy().view(ndt)
        assert np.array_equal(got, ref), "greedy ids must be bit-exact"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("V", [1000, 128256])
def test_greedy_sample_signed_zero_max(dtype, V):
    """A row whose maximum is 0, held by -0.0 in an earlier lane and +0.0 in a
    later one: the reference's `>` treats the two zeros as equal, so its lane
    tie rule (not the sign) decides the id."""
    dc = dcode(dtype)
    B = 2
    vals = -1.0 - np.abs(np.random.default_rng(V).standard_normal(B * V)).astype(np.float32)
    vals = vals.reshape(B, V)
    vals[0, 3], vals[0, 7] = -0.0, 0.0        # lane 3 (bit-reversed 192) beats lane 7 (224)
    vals[1, 700 % V], vals[1, 12] = 0.0, -0.0  # lane 12 vs lane 700 % 256
    l = oracle.from_float(vals.ravel(), dc)
    assert l.reshape(B, V)[0, 3] in (0x8000,), "quantiser must keep -0.0"
    t = dev(l, dtype).view(B, 1, V)
    out = torch.zeros(B, dtype=torch.int32, device="cuda")
    ev().greedy_sample(t, out, 0, 0, V)
    ref = np.zeros(B, np.uint32)
    oracle.greedy_sample(l, ref, B, 1, V, 0, 0, V, dc)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref), (out, ref)
    assert ref[0] == 3


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B,S,D,hd,off,gamma", [(1, 128, 512, 0, 0, False), (2, 17, 256, 64, 5, True),
                                                (8, 1, 2048, 128, 300, True), (4, 64, 4096, 128, 0, False)])
def test_rms_norm_rope_fused_vs_oracle(dtype, B, S, D, hd, off, gamma):
    """evkcu_rms_norm_rope against the oracle's rms_norm then rope (which
    rounds in between: one storage ulp of slack in the tolerance)."""
    dc = dcode(dtype)
    rows = B * S
    x = oracle.normal(rows * D, 60, 3.0, dtype=dc)
    g = oracle.normal(D, 61, dtype=dc) if gamma else None
    out = torch.empty(rows, D, dtype=dtype, device="cuda")
    ev().rms_norm_rope(dev(x, dtype).view(rows, D), out, S, 1e-5, 10000.0, hd, off,
                       gamma=dev(g, dtype) if gamma else None)
    n = np.empty_like(x)
    oracle.rms_norm(x, n, rows, D, 1e-5, gamma=g, dtype=dc)
    r = np.empty_like(x)
    oracle.rope(n, r, B, S, D, hd, off, 10000.0, dc)
    assert_close(u16(out).ravel(), r, dc, rel_l2=1e-3 if dc == 0 else 4e-3, ulps=2.0, what="rms_norm_rope")
