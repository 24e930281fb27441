"""GPU parity of flash_attention (tcgen05 path for Dh 64/128, CUDA-core path
for other Dh) and single-query decode attention through the C ABI: against
the CPU oracle at small sizes, against a torch fp32 reference at the
benchmark's full size, and the reference's flash-vs-unfused comparison
(example/tests.h:473-563) on the GPU with our own matmul and softmax."""
import numpy as np
import pytest

import oracle
from conftest import assert_close, dcode, dev, u16

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True, scope="module")
def _init():
    import evk_b200

    evk_b200.init(0)
    yield
    evk_b200.check_device_error()


def ev():
    import evk_b200

    return evk_b200


FLASH = [
    # B, N, H, Hkv, Dh, causal
    (1, 128, 1, 1, 64, False),
    (1, 200, 2, 1, 64, False),   # reference MQA semantics, ragged N
    (2, 256, 4, 4, 64, True),
    (1, 333, 4, 2, 64, True),    # GQA, ragged causal
    (2, 130, 2, 2, 128, False),
    (1, 300, 2, 2, 128, True),
    (1, 77, 2, 1, 32, False),    # CUDA-core path
    (1, 65, 3, 3, 80, True),     # CUDA-core path
    (1, 1, 2, 2, 64, True),      # single query
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", FLASH, ids=[str(c) for c in FLASH])
def test_flash_vs_oracle(dtype, case):
    B, N, H, Hkv, Dh, causal = case
    dc = dcode(dtype)
    q = oracle.normal(B * N * H * Dh, 21, dtype=dc)
    k = oracle.normal(B * N * Hkv * Dh, 22, dtype=dc)
    v = oracle.normal(B * N * Hkv * Dh, 23, dtype=dc)
    tq, tk, tv = dev(q, dtype).view(B, N, H * Dh), dev(k, dtype).view(B, N, Hkv * Dh), dev(v, dtype).view(B, N, Hkv * Dh)
    to = torch.empty_like(tq)
    ev().flash_attention(tq, tk, tv, to, heads=H, causal=causal)
    r = np.empty_like(q)
    oracle.flash_attention(q, k, v, r, B, N, H, Hkv, Dh, 0.0, int(causal), dc)
    # P is rounded to the storage type before the PV product (as the
    # reference's fp16 P tile is): fp16 keeps rel-L2 well under 1e-3.
    rel = 1e-3 if dc == 0 else 8e-3
    assert_close(u16(to).ravel(), r, dc, max_abs=2e-2, rel_l2=rel, what=f"flash {case}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_scores_growing_along_the_sequence(dtype, causal):
    """Scores that grow linearly with the key position (k proportional to the
    position): every 128-key block's maximum exceeds the previous one by ~17
    in log2 units, so the lazily kept reference maximum of every row must move
    (and O be rescaled) on every block."""
    B, N, H, Dh = 1, 512, 2, 64
    dc = dcode(dtype)
    pos = np.arange(N, dtype=np.float32)
    qf = np.full((B, N, H, Dh), 0.5, np.float32)
    kf = np.repeat((3.0 * pos / 128.0)[None, :, None, None], H, axis=2) * np.ones((B, N, H, Dh), np.float32)
    q = oracle.from_float(qf.ravel(), dc)
    k = oracle.from_float(kf.ravel(), dc)
    v = oracle.normal(B * N * H * Dh, 71, dtype=dc)
    to = torch.empty(B, N, H * Dh, dtype=dtype, device="cuda")
    ev().flash_attention(dev(q, dtype).view(B, N, H * Dh), dev(k, dtype).view(B, N, H * Dh),
                         dev(v, dtype).view(B, N, H * Dh), to, heads=H, causal=causal)
    r = np.empty_like(q)
    oracle.flash_attention(q, k, v, r, B, N, H, H, Dh, 0.0, int(causal), dc)
    assert bool(torch.isfinite(to.float()).all())
    assert_close(u16(to).ravel(), r, dc, max_abs=2e-2, rel_l2=1e-3 if dc == 0 else 8e-3, what="flash growing scores")


def test_flash_reference_api_default_mqa():
    """evk::ai::flash_attention call shape: K/V (B, N, Dh) shared by all heads."""
    B, N, H, Dh = 2, 256, 4, 64
    q = oracle.normal(B * N * H * Dh, 31)
    k = oracle.normal(B * N * Dh, 32)
    v = oracle.normal(B * N * Dh, 33)
    tq = dev(q, torch.float16).view(B, N, H * Dh)
    to = torch.empty_like(tq)
    ev().flash_attention(tq, dev(k, torch.float16).view(B, N, Dh), dev(v, torch.float16).view(B, N, Dh), to)
    r = np.empty_like(q)
    oracle.flash_attention(q, k, v, r, B, N, H, 1, Dh, 0.0, 0, 0)
    assert_close(u16(to).ravel(), r, 0, what="flash MQA")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_flash_full_size_c2_vs_torch(dtype):
    """Benchmark configuration: B=4, H=16, S=2048, Dh=64, causal (per-head K/V)."""
    B, H, S, Dh = 4, 16, 2048, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(B, S, H * Dh, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, S, H * Dh, device="cuda", generator=g).to(dtype)
    v = torch.randn(B, S, H * Dh, device="cuda", generator=g).to(dtype)
    o = torch.empty_like(q)
    ev().flash_attention(q, k, v, o, heads=H, causal=True)
    qf, kf, vf = (t.float().view(B, S, H, Dh).transpose(1, 2) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True).transpose(1, 2).reshape(B, S, H * Dh)
    err = (o.float() - ref)
    rel = (err.norm() / ref.norm()).item()
    assert rel <= (1e-3 if dtype == torch.float16 else 8e-3), rel
    assert err.abs().max().item() <= (2e-2 if dtype == torch.float16 else 6e-2)


def test_reference_flash_vs_unfused_n32768():
    """example/tests.h:473-563 on the GPU: MQA flash vs matmul->softmax->matmul
    with the reference's deterministic fills, max-abs <= 5e-2."""
    N, Dh = 32768, 64
    i = torch.arange(N, device="cuda").view(N, 1)
    d = torch.arange(Dh, device="cuda").view(1, Dh)
    q = (((i + d) % 13).float() / 13).half().view(1, N, Dh)
    k = (((i * 7 + d) % 11).float() / 11).half().view(1, N, Dh)
    v = (((i + 3 * d) % 17).float() / 17).half().view(1, N, Dh)
    o_flash = torch.empty_like(q)
    ev().flash_attention(q, k, v, o_flash)
    q_scaled = (q.float() * (1.0 / Dh ** 0.5)).half()
    s = torch.empty(1, N, N, dtype=torch.float16, device="cuda")
    ev().matmul(q_scaled, k, s, False, True, False)
    p = torch.empty_like(s)
    ev().softmax(s, p)
    del s
    o_base = torch.empty_like(q)
    ev().matmul(p, v, o_base)
    torch.cuda.synchronize()
    assert (o_flash.float() - o_base.float()).abs().max().item() <= 5e-2


DECODE = [
    # B, H, Hkv, Dh, max_len, cur_len
    (1, 8, 8, 64, 384, 1),
    (1, 8, 8, 64, 384, 200),
    (2, 8, 1, 64, 160, 160),     # the shader's MQA single-head-dim layout, all heads share K/V
    (8, 16, 16, 128, 2560, 2304),
    (2, 32, 8, 128, 1000, 999),  # GQA
    (3, 4, 4, 32, 64, 33),
    (1, 2, 2, 256, 100, 77),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", DECODE, ids=[str(c) for c in DECODE])
def test_single_query_attention_vs_oracle(dtype, case):
    B, H, Hkv, Dh, L, cur = case
    dc = dcode(dtype)
    q = oracle.normal(B * H * Dh, 41, dtype=dc)
    kc = oracle.normal(B * L * Hkv * Dh, 42, dtype=dc)
    vc = oracle.normal(B * L * Hkv * Dh, 43, dtype=dc)
    out = torch.empty(B, H * Dh, dtype=dtype, device="cuda")
    ev().single_query_attention(dev(q, dtype).view(B, H * Dh), dev(kc, dtype).view(B, L, Hkv * Dh),
                                dev(vc, dtype).view(B, L, Hkv * Dh), out, H, cur)
    r = np.empty(B * H * Dh, np.uint16)
    oracle.single_query_attention(q, kc, vc, r, B, H, Hkv, Dh, L, cur, 0.0, dc)
    assert_close(u16(out).ravel(), r, dc, rel_l2=1e-3 if dc == 0 else 4e-3, what=f"decode {case}")


def test_single_query_attention_empty_cache_is_zero():
    out = torch.full((1, 128), 7.0, dtype=torch.float16, device="cuda")
    q = torch.randn(1, 128, device="cuda").half()
    kc = torch.randn(1, 16, 128, device="cuda").half()
    ev().single_query_attention(q, kc, kc, out, 2, 0)
    assert bool((out == 0).all())


def test_single_query_attention_scratch_reuse_across_shapes():
    """Split-reduction scratch is shared by calls of different grid shapes:
    a large call after a small one must not read stale counters."""
    for (B, H, Dh, L, cur) in [(8, 16, 128, 256, 64), (1, 2, 128, 256, 200), (8, 16, 64, 256, 64), (8, 16, 128, 256, 64)]:
        q = oracle.normal(B * H * Dh, 51)
        kc = oracle.normal(B * L * H * Dh, 52)
        vc = oracle.normal(B * L * H * Dh, 53)
        out = torch.empty(B, H * Dh, dtype=torch.float16, device="cuda")
        ev().single_query_attention(dev(q, torch.float16).view(B, H * Dh), dev(kc, torch.float16).view(B, L, H * Dh),
                                    dev(vc, torch.float16).view(B, L, H * Dh), out, H, cur)
        r = np.empty(B * H * Dh, np.uint16)
        oracle.single_query_attention(q, kc, vc, r, B, H, H, Dh, L, cur)
        assert_close(u16(out).ravel(), r, 0, what=f"decode reuse {(B, H, Dh, L, cur)}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_single_query_attention_ignores_cache_rows_past_length(dtype):
    """Rows at and past cur_len (a cache's unwritten tail, or the next
    sequence's rows inside the same 64-row tile) carry weight 0: NaN / Inf
    there must not reach the output (0 * NaN would)."""
    B, H, Dh, L, cur = 2, 4, 64, 160, 131
    dc = dcode(dtype)
    q = oracle.normal(B * H * Dh, 61, dtype=dc)
    kc = oracle.normal(B * L * H * Dh, 62, dtype=dc).reshape(B, L, H * Dh)
    vc = oracle.normal(B * L * H * Dh, 63, dtype=dc).reshape(B, L, H * Dh)
    r = np.empty(B * H * Dh, np.uint16)
    oracle.single_query_attention(q, kc.ravel().copy(), vc.ravel().copy(), r, B, H, H, Dh, L, cur, 0.0, dc)
    nan = 0x7E00 if dc == 0 else 0x7FC0
    kc[:, cur:, :] = nan
    vc[:, cur:, :] = nan
    out = torch.empty(B, H * Dh, dtype=dtype, device="cuda")
    ev().single_query_attention(dev(q, dtype).view(B, H * Dh), dev(kc.ravel(), dtype).view(B, L, H * Dh),
                                dev(vc.ravel(), dtype).view(B, L, H * Dh), out, H, cur)
    assert bool(torch.isfinite(out.float()).all())
    assert_close(u16(out).ravel(), r, dc, rel_l2=1e-3 if dc == 0 else 4e-3, what="decode with NaN tail")


def _flash_random_cases(n=12, seed=1202):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        Dh = int(rng.choice([64, 64, 128, 128, 96]))  # 96: the one-warp-per-row kernel
        Hkv = int(rng.choice([1, 2, 4]))
        H = Hkv * int(rng.choice([1, 2, 4]))
        B = int(rng.integers(1, 4))
        N = int(rng.integers(16, 700 if Dh == 96 else 1500))
        causal = bool(rng.integers(0, 2))
        out.append((B, N, H, Hkv, Dh, causal))
    return out


FLASH_RANDOM = _flash_random_cases()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", FLASH_RANDOM, ids=[str(c) for c in FLASH_RANDOM])
def test_flash_random_shapes_vs_torch(dtype, case):
    """Seeded random shapes (ragged sequence lengths, MQA / GQA / MHA, Dh 64,
    128 and 96, causal or not) against torch fp32 attention, with the bounds
    of the full-size test."""
    B, N, H, Hkv, Dh, causal = case
    g = torch.Generator(device="cuda").manual_seed(N * 131 + H * 7 + Dh)
    q = torch.randn(B, N, H * Dh, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, N, Hkv * Dh, device="cuda", generator=g).to(dtype)
    v = torch.randn(B, N, Hkv * Dh, device="cuda", generator=g).to(dtype)
    o = torch.empty_like(q)
    ev().flash_attention(q, k, v, o, heads=H, causal=causal)
    qf = q.float().view(B, N, H, Dh).transpose(1, 2)
    kf = k.float().view(B, N, Hkv, Dh).transpose(1, 2).repeat_interleave(H // Hkv, dim=1)
    vf = v.float().view(B, N, Hkv, Dh).transpose(1, 2).repeat_interleave(H // Hkv, dim=1)
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=causal)
    ref = ref.transpose(1, 2).reshape(B, N, H * Dh)
    err = o.float() - ref
    rel = (err.norm() / ref.norm()).item()
    assert rel <= (1e-3 if dtype == torch.float16 else 8e-3), rel
    assert err.abs().max().item() <= (2e-2 if dtype == torch.float16 else 6e-2)
