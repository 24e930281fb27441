"""GPU parity of evk::ai::matmul (tcgen05 path and the small-M GEMV path)
through the C ABI: against the CPU oracle at sizes it finishes quickly, against
a torch fp32 reference for the large shapes, and the reference's identity
known-answer tests bit-exactly."""
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


def identity(n, val):
    x = np.zeros(n * n, np.float32)
    x[:: n + 1] = val
    return oracle.from_float(x)


def test_kat_identity_400():  # example/tests.h:163-194
    n = 400
    a, b = dev(identity(n, 2.0), torch.float16).view(n, n), dev(identity(n, 2.0), torch.float16).view(n, n)
    c = torch.empty(n, n, dtype=torch.float16, device="cuda")
    ev().matmul(a, b, c)
    assert np.array_equal(u16(c).ravel(), identity(n, 4.0))


def test_kat_broadcast():  # example/tests.h:196-219
    a = torch.ones(1, 32, 32, dtype=torch.float16, device="cuda")
    b = dev(identity(32, 1.0), torch.float16).view(32, 32)
    c = torch.empty(3, 32, 32, dtype=torch.float16, device="cuda")
    ev().matmul(a, b, c)
    assert bool((c == 1).all())


CASES = [
    # batch, M, K, N, ta, tb, acc, broadcast ('a', 'b' or '')
    (1, 128, 64, 128, 0, 0, 0, ""),
    (1, 1024, 1024, 1024, 0, 0, 0, ""),
    (1, 200, 72, 136, 0, 0, 0, ""),
    (1, 200, 72, 136, 1, 0, 0, ""),
    (1, 200, 72, 136, 0, 1, 0, ""),
    (1, 200, 72, 136, 1, 1, 1, ""),
    (3, 96, 264, 80, 0, 0, 1, ""),
    (3, 96, 264, 80, 0, 0, 0, "b"),
    (3, 96, 264, 80, 0, 1, 0, "a"),
    (2, 384, 512, 520, 1, 0, 0, ""),
    (1, 17, 512, 1024, 0, 0, 0, ""),  # tcgen05 with a ragged M tile
    (1, 1, 512, 2048, 0, 0, 0, ""),   # GEMV
    (1, 4, 2048, 512, 0, 0, 1, ""),   # GEMV split-K + acc
    (1, 16, 1024, 4096, 0, 0, 0, ""),  # GEMV, 16 rows
    (1, 3, 512, 32000, 0, 1, 0, ""),  # GEMV, transposed B (tied LM head)
    (4, 2, 512, 1024, 0, 0, 0, "b"),  # GEMV over a broadcast weight
    # M >= 256: the paired-SM kernel's shapes when it is forced on
    # (tests/test_gpu_gemm_pair.py); ragged M, N and K, every operand layout
    (1, 1000, 72, 776, 0, 0, 1, ""),
    (1, 520, 136, 264, 0, 1, 1, ""),
    (3, 256, 128, 256, 1, 1, 0, "a"),
    (2, 304, 200, 520, 1, 0, 1, "b"),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_matmul_vs_oracle(dtype, case):
    batch, M, K, N, ta, tb, acc, bc = case
    dc = dcode(dtype)
    ba = 1 if bc == "a" else batch
    bb = 1 if bc == "b" else batch
    A = oracle.normal(ba * M * K, 1, dtype=dc)
    B = oracle.normal(bb * K * N, 2, dtype=dc)
    C = oracle.normal(batch * M * N, 3, dtype=dc)
    tA = dev(A, dtype).view(ba, *((K, M) if ta else (M, K)))
    tB = dev(B, dtype).view(bb, *((N, K) if tb else (K, N)))
    tC = dev(C, dtype).view(batch, M, N)
    ev().matmul(tA, tB, tC, bool(ta), bool(tb), bool(acc))
    R = C.copy()
    oracle.matmul(A, B, R, batch, M, K, N, 0 if ba == 1 and batch > 1 else M * K, 0 if bb == 1 and batch > 1 else K * N,
                  M * N, ta | (tb << 1) | (acc << 2), dc)
    assert_close(u16(tC).ravel(), R, dc, what=f"matmul {case}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K,N", [(4096, 4096, 4096), (2048, 8192, 2048), (8192, 2048, 4096)])
def test_matmul_large_vs_torch_fp32(dtype, M, K, N):
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    b = torch.randn(K, N, device="cuda", generator=g).to(dtype)
    c = torch.empty(M, N, dtype=dtype, device="cuda")
    ev().matmul(a, b, c)
    # fp32 reference rounded once to the storage type (as the oracle does):
    # what remains is accumulation order, at most ~1 storage ulp per element.
    ref = (a.float() @ b.float()).to(dtype).float()
    err = (c.float() - ref)
    rel = err.norm() / ref.norm()
    tol_elem = (2e-2 + (2 ** -10 if dtype == torch.float16 else 2 ** -7) * ref.abs())
    assert rel.item() <= (1e-3 if dtype == torch.float16 else 2e-3), f"rel-L2 {rel.item()}"
    assert bool((err.abs() <= tol_elem).all()), f"max abs err {err.abs().max().item()}"


def test_matmul_rejects_bad_rows():
    import evk_b200

    a = torch.randn(64, 12, device="cuda").half()  # K = 12 not a multiple of 8
    b = torch.randn(12, 64, device="cuda").half()
    c = torch.empty(64, 64, device="cuda").half()
    with pytest.raises(evk_b200.EvkcuError):
        ev().matmul(a, b, c)


def _random_cases(n=14, seed=20261202):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        batch = int(rng.choice([1, 1, 2, 3]))
        M = int(rng.integers(1, 1600))
        K = 8 * int(rng.integers(1, 300))
        N = 8 * int(rng.integers(1, 260))
        ta, tb, acc = (int(x) for x in rng.integers(0, 2, 3))
        if ta:
            M = max(8, M - M % 8)  # transpose_a: M is the contiguous dimension
        bc = str(rng.choice(["", "", "a", "b"])) if batch > 1 else ""
        out.append((batch, M, K, N, ta, tb, acc, bc))
    return out


RANDOM_CASES = _random_cases()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", RANDOM_CASES, ids=[str(c) for c in RANDOM_CASES])
def test_matmul_random_shapes_vs_torch_fp32(dtype, case):
    """Seeded random shapes (ragged M, N, K; every operand layout; batch
    broadcast; C +=) against a torch fp32 product rounded once to the storage
    type, with the same bounds as the large-shape test."""
    batch, M, K, N, ta, tb, acc, bc = case
    g = torch.Generator(device="cuda").manual_seed(M * 7919 + N * 31 + K)
    ba = 1 if bc == "a" else batch
    bb = 1 if bc == "b" else batch
    a = torch.randn(ba, *((K, M) if ta else (M, K)), device="cuda", generator=g).to(dtype)
    b = torch.randn(bb, *((N, K) if tb else (K, N)), device="cuda", generator=g).to(dtype)
    c = torch.randn(batch, M, N, device="cuda", generator=g).to(dtype)
    c0 = c.float().clone()
    ev().matmul(a, b, c, bool(ta), bool(tb), bool(acc))
    A = a.float().transpose(1, 2) if ta else a.float()
    B = b.float().transpose(1, 2) if tb else b.float()
    ref = torch.matmul(A.expand(batch, M, K), B.expand(batch, K, N)) + (c0 if acc else 0.0)
    ref = ref.to(dtype).float()
    err = c.float() - ref
    rel = (err.norm() / ref.norm()).item()
    tol_elem = 2e-2 + (2 ** -10 if dtype == torch.float16 else 2 ** -7) * ref.abs()
    assert rel <= (1e-3 if dtype == torch.float16 else 2e-3), f"rel-L2 {rel}"
    assert bool((err.abs() <= tol_elem).all()), f"max abs err {err.abs().max().item()}"
