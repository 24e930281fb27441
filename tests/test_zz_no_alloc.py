"""evkcu_greedy_sample_noalloc: greedy argmax for callers that cannot
allocate GPU memory when they call it (code running during a CUDA stream
capture, serving loops whose HBM is fully reserved up front, hosts that forbid
allocation on the hot path).  Its scratch is a fixed device array inside the
library, so its ids must equal the allocating entry point's, call after call.

The file name makes pytest collect it last, so a failure here never hides the
result of another test; it also passes on its own in a fresh process.
"""
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _call(fn, logits, out, position, base, count):
    import evk_b200

    B, S, V = logits.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(logits.data_ptr(), out.data_ptr(), B, S, V, position, base, count, out.element_size(),
              evk_b200._dtype_code(logits), stream)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_noalloc_matches_allocating_entry_two_calls(dtype):
    import evk_b200

    evk_b200.init(0)
    lib = evk_b200.lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    # Two calls in a row with different shapes: the second reuses the array
    # the first one left behind.  Ids are integers: the bar is bit-exact.
    for (B, S, V, pos, base, count) in [(4, 2, 128256, 1, 0, 128256), (16, 1, 32000, 0, 5, 31000)]:
        logits = (torch.randn(B, S, V, device="cuda", generator=g) * 3).to(dtype)
        logits[:, pos, base + 17] = 50.0  # a tie across lanes exercises the tie rule
        logits[:, pos, base + 17 + 256] = 50.0
        ref = torch.zeros(B, dtype=torch.int32, device="cuda")
        got = torch.full((B,), -1, dtype=torch.int32, device="cuda")
        assert _call(lib.evkcu_greedy_sample, logits, ref, pos, base, count) == 0
        assert _call(lib.evkcu_greedy_sample_noalloc, logits, got, pos, base, count) == 0, \
            lib.evkcu_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (got.cpu().tolist(), ref.cpu().tolist())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import evk_b200

    lib = evk_b200.lib()
    logits = torch.zeros(1100, 1, 8, dtype=torch.float16, device="cuda")  # B = 1100 > 1024
    out = torch.zeros(1100, dtype=torch.int32, device="cuda")
    assert _call(lib.evkcu_greedy_sample_noalloc, logits, out, 0, 0, 8) == 1
    assert b"fixed scratch" in lib.evkcu_last_error()
