"""evk_b200 — B200 (sm_100a) backend for the evk::ai inference operators.

The product is the C ABI in ``include/evkcu.h`` (``libevkcu.so``) and the
C++20 ``evk::ai`` layer above it (``libevk_ai.so``).  This module binds the C
ABI with ctypes so Python callers (tests, ``bench.py``) can drive the kernels
on torch-allocated device memory.  It is a thin binding: no kernel runs
anywhere but in ``libevkcu.so``, and importing it fails loudly when the
library has not been built.

Function names follow the reference's operators (carloshgsilva/evk
``evk_ai.h:489-615``); argument meaning follows ``include/evkcu.h``.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libevkcu.so")
AI_LIB_PATH = os.path.join(_HERE, "libevk_ai.so")

F16 = 0
BF16 = 1
MM_TRANSPOSE_A = 1
MM_TRANSPOSE_B = 2
MM_ACC_C = 4
ATTN_CAUSAL = 1
ATTN_BWD_NORMALIZED = 2

STATUS = {
    0: "OK",
    1: "BAD_SHAPE",
    2: "BAD_ALIGN",
    3: "CUDA_ERROR",
    4: "COMM_ERROR",
    5: "TIMEOUT",
    6: "UNSUPPORTED",
    7: "BAD_ARG",
}


class EvkcuError(RuntimeError):
    def __init__(self, op: str, status: int, msg: str):
        super().__init__(f"{op} failed: {STATUS.get(status, status)}: {msg}")
        self.status = status


_u32, _u64, _f32, _int, _vp = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p

# name -> argtypes (all return int status unless listed in _RET)
SIGNATURES = {
    "evkcu_init": [_int],
    "evkcu_shutdown": [],
    "evkcu_last_error": [],
    "evkcu_version": [],
    "evkcu_check_device_error": [],
    "evkcu_launch_count": [],
    "evkcu_reset_launch_count": [],
    "evkcu_matmul": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u64, _u64, _u64, _u32, _int, _vp],
    "evkcu_flash_attention": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _u32, _int, _vp],
    "evkcu_single_query_attention": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _f32, _int, _vp],
    "evkcu_rms_norm": [_vp, _vp, _vp, _u32, _u32, _f32, _int, _vp],
    "evkcu_rope": [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _int, _vp],
    "evkcu_gelu": [_vp, _vp, _u64, _int, _vp],
    "evkcu_softmax": [_vp, _vp, _u32, _u32, _f32, _int, _vp],
    "evkcu_add": [_vp, _vp, _vp, _u64, _int, _vp],
    "evkcu_scale": [_vp, _u64, _f32, _int, _vp],
    "evkcu_zero": [_vp, _u64, _int, _vp],
    "evkcu_causal_mask": [_vp, _u32, _u32, _int, _vp],
    "evkcu_embed": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _int, _vp],
    "evkcu_greedy_sample": [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _int, _vp],
    "evkcu_greedy_sample_noalloc": [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _int, _vp],
    "evkcu_rms_norm_rope": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _f32, _int, _vp],
    # training side
    "evkcu_relu": [_vp, _vp, _u64, _int, _vp],
    "evkcu_relu_backward": [_vp, _vp, _vp, _u64, _int, _vp],
    "evkcu_gelu_backward": [_vp, _vp, _vp, _u64, _int, _vp],
    "evkcu_softmax_backward": [_vp, _vp, _vp, _u32, _u32, _f32, _int, _vp],
    "evkcu_rms_norm_backward": [_vp, _vp, _vp, _u32, _u32, _f32, _int, _vp],
    "evkcu_rope_backward": [_vp, _vp, _u32, _u32, _u32, _f32, _int, _vp],
    "evkcu_embed_backward": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _int, _vp],
    "evkcu_position_add": [_vp, _vp, _vp, _u32, _u32, _u32, _int, _vp],
    "evkcu_position_add_backward": [_vp, _vp, _vp, _u32, _u32, _u32, _int, _vp],
    "evkcu_sum_batch": [_vp, _vp, _u32, _u64, _int, _vp],
    "evkcu_sgd": [_vp, _vp, _u64, _f32, _int, _vp],
    "evkcu_adam": [_vp, _vp, _vp, _vp, _u64, _u32, _f32, _f32, _f32, _f32, _int, _vp],
    "evkcu_mse_loss": [_vp, _vp, _vp, _vp, _u64, _int, _vp],
    "evkcu_cross_entropy_loss": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _int, _vp],
    "evkcu_flash_attention_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _u32,
                                  _int, _vp],
}
_RET = {
    "evkcu_last_error": ctypes.c_char_p,
    "evkcu_version": ctypes.c_char_p,
    "evkcu_launch_count": ctypes.c_uint64,
    "evkcu_reset_launch_count": None,
}


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libevkcu.so and declares every C-ABI entry point."""
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `make -C evk_b200` (or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RET.get(name, ctypes.c_int)
    return lib


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load_library()
    return _lib


def _check(op: str, status: int) -> None:
    if status != 0:
        raise EvkcuError(op, status, lib().evkcu_last_error().decode())


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {t.dtype}: evk tensors are 2-byte fp16 (or bf16)")


def _ptr(t) -> int:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("evk_b200 ops take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("evk_b200 ops take contiguous (row-major) tensors")
    return t.data_ptr()


def _stream(stream) -> int:
    import torch

    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def init(device: int = -1) -> None:
    _check("evkcu_init", lib().evkcu_init(device))


def launch_count() -> int:
    return int(lib().evkcu_launch_count())


def reset_launch_count() -> None:
    lib().evkcu_reset_launch_count()


def check_device_error() -> None:
    _check("evkcu_check_device_error", lib().evkcu_check_device_error())


# ------------------------------------------------------------------ operators
def matmul(a, b, c, transpose_a=False, transpose_b=False, acc_c=False, stream=None):
    """evk::ai::matmul (evk_ai.cpp:254-330): c = op(a) @ op(b) (+ c).

    Shapes follow the reference: (..., M, K) x (..., K, N) -> (..., M, N); an
    operand whose leading dims multiply to 1 is broadcast over the batch.
    """
    def lead(t):
        n = 1
        for d in t.shape[:-2]:
            n *= d
        return n

    ba, bb, bc = lead(a), lead(b), lead(c)
    batch = max(ba, bb, bc)
    M = a.shape[-1] if transpose_a else a.shape[-2]
    K = a.shape[-2] if transpose_a else a.shape[-1]
    N = b.shape[-2] if transpose_b else b.shape[-1]
    Kb = b.shape[-1] if transpose_b else b.shape[-2]
    if Kb != K or c.shape[-2] != M or c.shape[-1] != N or bc != batch or ba not in (1, batch) or bb not in (1, batch):
        raise EvkcuError("matmul", 1, f"incompatible shapes {tuple(a.shape)} {tuple(b.shape)} {tuple(c.shape)}")
    ea, eb, ec = a.shape[-2] * a.shape[-1], b.shape[-2] * b.shape[-1], c.shape[-2] * c.shape[-1]
    sa = 0 if (ba == 1 and batch > 1) else ea
    sb = 0 if (bb == 1 and batch > 1) else eb
    flags = (MM_TRANSPOSE_A if transpose_a else 0) | (MM_TRANSPOSE_B if transpose_b else 0) | (MM_ACC_C if acc_c else 0)
    _check("evkcu_matmul", lib().evkcu_matmul(_ptr(a), _ptr(b), _ptr(c), batch, M, K, N, sa, sb, ec, flags,
                                              _dtype_code(a), _stream(stream)))
    return c


def flash_attention(q, k, v, o, heads: Optional[int] = None, causal=False, scale: float = 0.0, stream=None):
    """evk::ai::flash_attention (evk_ai.cpp:332-369) plus extensions.

    q, o: (B, N, H*Dh); k, v: (B, N, Hkv*Dh).  Without `heads` the reference's
    multi-query call is assumed (Hkv = 1, Dh = k.shape[-1]).  `heads` gives H
    (Dh = q.shape[-1] // H, Hkv = k.shape[-1] // Dh).
    """
    B, N, D = q.shape
    if heads is None:
        Dh = k.shape[-1]
        H, Hkv = D // Dh, 1
    else:
        H = heads
        Dh = D // H
        Hkv = k.shape[-1] // Dh
    _check("evkcu_flash_attention", lib().evkcu_flash_attention(
        _ptr(q), _ptr(k), _ptr(v), _ptr(o), B, N, H, Hkv, Dh, scale, ATTN_CAUSAL if causal else 0,
        _dtype_code(q), _stream(stream)))
    return o


def single_query_attention(q, kcache, vcache, out, heads: int, cur_len: int, scale: float = 0.0, stream=None):
    """Decode attention over a KV cache (shaders/single_query_attention.comp).

    q, out: (B, H*Dh); kcache, vcache: (B, max_len, Hkv*Dh).
    """
    B = q.shape[0]
    Dh = q.shape[-1] // heads
    max_len = kcache.shape[1]
    Hkv = kcache.shape[-1] // Dh
    _check("evkcu_single_query_attention", lib().evkcu_single_query_attention(
        _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(out), B, heads, Hkv, Dh, max_len, cur_len, scale,
        _dtype_code(q), _stream(stream)))
    return out


def rms_norm(x, out, eps=1e-4, gamma=None, stream=None):
    D = x.shape[-1]
    _check("evkcu_rms_norm", lib().evkcu_rms_norm(_ptr(x), _ptr(out), _ptr(gamma), x.numel() // D, D, eps,
                                                  _dtype_code(x), _stream(stream)))
    return out


def rope(x, out, batch, seq_len, dim, base=10000.0, head_dim=0, pos_offset=0, stream=None):
    _check("evkcu_rope", lib().evkcu_rope(_ptr(x), _ptr(out), batch, seq_len, dim, head_dim, pos_offset, base,
                                          _dtype_code(x), _stream(stream)))
    return out


def rms_norm_rope(x, out, seq_len, eps=1e-5, base=10000.0, head_dim=0, pos_offset=0, gamma=None, stream=None):
    """Fused rms_norm + rope over rows of the last dimension (evkcu_rms_norm_rope)."""
    D = x.shape[-1]
    _check("evkcu_rms_norm_rope", lib().evkcu_rms_norm_rope(
        _ptr(x), _ptr(out), _ptr(gamma), x.numel() // D, seq_len, D, head_dim, pos_offset, eps, base,
        _dtype_code(x), _stream(stream)))
    return out


def gelu(x, out, stream=None):
    _check("evkcu_gelu", lib().evkcu_gelu(_ptr(x), _ptr(out), x.numel(), _dtype_code(x), _stream(stream)))
    return out


def softmax(x, out, scale=1.0, stream=None):
    L = x.shape[-1]
    _check("evkcu_softmax", lib().evkcu_softmax(_ptr(x), _ptr(out), x.numel() // L, L, scale, _dtype_code(x),
                                                _stream(stream)))
    return out


def add(a, b, c, stream=None):
    _check("evkcu_add", lib().evkcu_add(_ptr(a), _ptr(b), _ptr(c), a.numel(), _dtype_code(a), _stream(stream)))
    return c


def scale(x, s, stream=None):
    _check("evkcu_scale", lib().evkcu_scale(_ptr(x), x.numel(), s, _dtype_code(x), _stream(stream)))
    return x


def zero(x, stream=None):
    _check("evkcu_zero", lib().evkcu_zero(_ptr(x), x.numel(), _dtype_code(x), _stream(stream)))
    return x


def apply_causal_mask(s, stream=None):
    N = s.shape[-1]
    _check("evkcu_causal_mask", lib().evkcu_causal_mask(_ptr(s), s.numel() // (N * N), N, _dtype_code(s),
                                                        _stream(stream)))
    return s


def embed(E, idx, out, stream=None):
    """idx: int16/uint16 (reference) or int32 ids, any shape."""
    import torch

    ib = 2 if idx.element_size() == 2 else 4
    _check("evkcu_embed", lib().evkcu_embed(_ptr(E), _ptr(idx), _ptr(out), E.shape[0], E.shape[1], idx.numel(), ib,
                                            _dtype_code(E), _stream(stream)))
    return out


def greedy_sample(logits, out, position, token_base, token_count, stream=None):
    """logits (B, S, V); out (B,) int16/uint16 (reference) or int32 ids."""
    B, S, V = logits.shape
    ob = 2 if out.element_size() == 2 else 4
    _check("evkcu_greedy_sample", lib().evkcu_greedy_sample(
        _ptr(logits), _ptr(out), B, S, V, position, token_base, token_count, ob, _dtype_code(logits),
        _stream(stream)))
    return out


# ------------------------------------------------------------ training side --
def relu(x, out, stream=None):
    _check("evkcu_relu", lib().evkcu_relu(_ptr(x), _ptr(out), x.numel(), _dtype_code(x), _stream(stream)))
    return out


def relu_backward(grad_out, x, grad_in, stream=None):
    _check("evkcu_relu_backward", lib().evkcu_relu_backward(_ptr(grad_out), _ptr(x), _ptr(grad_in), x.numel(),
                                                            _dtype_code(x), _stream(stream)))
    return grad_in


def gelu_backward(grad_out, x, grad_in, stream=None):
    _check("evkcu_gelu_backward", lib().evkcu_gelu_backward(_ptr(grad_out), _ptr(x), _ptr(grad_in), x.numel(),
                                                            _dtype_code(x), _stream(stream)))
    return grad_in


def softmax_backward(probs, grad_out, grad_in, scale=1.0, stream=None):
    L = probs.shape[-1]
    _check("evkcu_softmax_backward", lib().evkcu_softmax_backward(
        _ptr(probs), _ptr(grad_out), _ptr(grad_in), probs.numel() // L, L, scale, _dtype_code(probs),
        _stream(stream)))
    return grad_in


def rms_norm_backward(x, grad_out, grad_in, eps=1e-4, stream=None):
    D = x.shape[-1]
    _check("evkcu_rms_norm_backward", lib().evkcu_rms_norm_backward(
        _ptr(x), _ptr(grad_out), _ptr(grad_in), x.numel() // D, D, eps, _dtype_code(x), _stream(stream)))
    return grad_in


def rope_backward(grad_out, grad_in, batch, seq_len, dim, base=10000.0, stream=None):
    _check("evkcu_rope_backward", lib().evkcu_rope_backward(_ptr(grad_out), _ptr(grad_in), batch, seq_len, dim,
                                                            base, _dtype_code(grad_out), _stream(stream)))
    return grad_in


def embed_backward(grad_out, idx, grad_E, stream=None):
    ib = 2 if idx.element_size() == 2 else 4
    _check("evkcu_embed_backward", lib().evkcu_embed_backward(
        _ptr(grad_out), _ptr(idx), _ptr(grad_E), grad_E.shape[0], grad_E.shape[1], idx.numel(), ib,
        _dtype_code(grad_E), _stream(stream)))
    return grad_E


def position_add(x, pos, out, batch, seq_len, dim, stream=None):
    _check("evkcu_position_add", lib().evkcu_position_add(_ptr(x), _ptr(pos), _ptr(out), batch, seq_len, dim,
                                                          _dtype_code(x), _stream(stream)))
    return out


def position_add_backward(grad_out, grad_in, grad_pos, batch, seq_len, dim, stream=None):
    _check("evkcu_position_add_backward", lib().evkcu_position_add_backward(
        _ptr(grad_out), _ptr(grad_in), _ptr(grad_pos), batch, seq_len, dim, _dtype_code(grad_out),
        _stream(stream)))
    return grad_in, grad_pos


def sum_batch(x, out, batch, size, stream=None):
    _check("evkcu_sum_batch", lib().evkcu_sum_batch(_ptr(x), _ptr(out), batch, size, _dtype_code(x),
                                                    _stream(stream)))
    return out


def sgd(param, grad, lr, stream=None):
    _check("evkcu_sgd", lib().evkcu_sgd(_ptr(param), _ptr(grad), param.numel(), lr, _dtype_code(param),
                                        _stream(stream)))
    return param


def adam(param, grad, m, v, step, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-4, stream=None):
    """m, v: the AdamState buffers (zero-initialised, same dtype/size as param);
    step: the state's timestep after increment (1 on the first call)."""
    _check("evkcu_adam", lib().evkcu_adam(_ptr(param), _ptr(grad), _ptr(m), _ptr(v), param.numel(), step, lr, beta1,
                                          beta2, eps, _dtype_code(param), _stream(stream)))
    return param


def mse_loss(pred, target, grad, result, stream=None):
    _check("evkcu_mse_loss", lib().evkcu_mse_loss(_ptr(pred), _ptr(target), _ptr(grad), _ptr(result), pred.numel(),
                                                  _dtype_code(pred), _stream(stream)))
    return result


def cross_entropy_loss(logits, targets, grad, result, stream=None):
    """logits (rows, V); targets (rows,) int16/uint16 (reference) or int32."""
    V = logits.shape[-1]
    tb = 2 if targets.element_size() == 2 else 4
    _check("evkcu_cross_entropy_loss", lib().evkcu_cross_entropy_loss(
        _ptr(logits), _ptr(targets), _ptr(grad), _ptr(result), logits.numel() // V, V, tb, _dtype_code(logits),
        _stream(stream)))
    return result


def flash_attention_bwd(q, k, v, o, dO, dQ, dK, dV, heads: Optional[int] = None, causal=False, normalized=False,
                        scale: float = 0.0, stream=None):
    """Gradients of flash_attention (evk_ai.cpp:371-473).  Layouts as
    flash_attention; without `heads` the reference's multi-query call."""
    B, N, D = q.shape
    if heads is None:
        Dh = k.shape[-1]
        H, Hkv = D // Dh, 1
    else:
        H = heads
        Dh = D // H
        Hkv = k.shape[-1] // Dh
    flags = (ATTN_CAUSAL if causal else 0) | (ATTN_BWD_NORMALIZED if normalized else 0)
    _check("evkcu_flash_attention_bwd", lib().evkcu_flash_attention_bwd(
        _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(dQ), _ptr(dK), _ptr(dV), B, N, H, Hkv, Dh, scale, flags,
        _dtype_code(q), _stream(stream)))
    return dQ, dK, dV


# ------------------------------------------------------------- LLM driver --
class LlmConfig(ctypes.Structure):
    """evkcu_llm_config (include/evkcu.h)."""

    _fields_ = [(n, ctypes.c_uint32) for n in ("layers", "d_model", "heads", "kv_heads", "hidden", "vocab",
                                                "max_batch", "max_seq")] + \
               [("rope_base", ctypes.c_float), ("eps", ctypes.c_float), ("dtype", ctypes.c_int),
                ("tied_embeddings", ctypes.c_uint32), ("tp_rank", ctypes.c_uint32), ("tp_size", ctypes.c_uint32)]


_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES.update({
    "evkcu_single_query_attention_devlen": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _f32, _int, _vp],
    "evkcu_comm_unique_id": [_vp],
    "evkcu_comm_init": [_vp, _int, _int, _pp],
    "evkcu_comm_destroy": [_vp],
    "evkcu_llm_create": [ctypes.POINTER(LlmConfig), _vp, _pp],
    "evkcu_llm_destroy": [_vp],
    "evkcu_llm_init_random": [_vp, _u64, _f32, _vp],
    "evkcu_llm_set_weight": [_vp, ctypes.c_char_p, _u32, _vp, _vp],
    "evkcu_llm_prefill": [_vp, _vp, _u32, _u32, _vp, _vp, _vp],
    "evkcu_llm_decode": [_vp, _vp, _vp, _vp, _vp],
    "evkcu_llm_length": [_vp],
    "evkcu_llm_fused_allreduce": [_vp],
    "evkcu_llm_load": [_vp, ctypes.c_char_p, _vp],
    "evkcu_llm_save": [_vp, ctypes.c_char_p, _vp],
})
_RET["evkcu_llm_length"] = ctypes.c_uint32
_RET["evkcu_llm_fused_allreduce"] = ctypes.c_uint32


class Comm:
    """NCCL communicator for tensor parallelism (one process per GPU)."""

    def __init__(self, unique_id: bytes, rank: int, world: int):
        self.handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, 128)
        _check("evkcu_comm_init", lib().evkcu_comm_init(buf, rank, world, ctypes.byref(self.handle)))

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check("evkcu_comm_unique_id", lib().evkcu_comm_unique_id(buf))
        return buf.raw

    def close(self):
        if self.handle:
            _check("evkcu_comm_destroy", lib().evkcu_comm_destroy(self.handle))
            self.handle = ctypes.c_void_p()


class Llm:
    """Device-resident decoder (evkcu_llm_*): prefill, CUDA-graph decode,
    optional tensor parallelism.  Token ids are int32 CUDA tensors."""

    def __init__(self, layers, d_model, heads, hidden, vocab, max_batch, max_seq, kv_heads=None, rope_base=10000.0,
                 eps=1e-5, dtype=F16, tied_embeddings=True, tp_rank=0, tp_size=1, comm: Optional[Comm] = None):
        self.cfg = LlmConfig(layers, d_model, heads, kv_heads or heads, hidden, vocab, max_batch, max_seq, rope_base,
                             eps, dtype, int(tied_embeddings), tp_rank, tp_size)
        self.handle = ctypes.c_void_p()
        _check("evkcu_llm_create", lib().evkcu_llm_create(ctypes.byref(self.cfg), comm.handle if comm else None,
                                                          ctypes.byref(self.handle)))

    def close(self):
        if self.handle:
            lib().evkcu_llm_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed=42, std=0.02, stream=None):
        _check("evkcu_llm_init_random", lib().evkcu_llm_init_random(self.handle, seed, std, _stream(stream)))

    def set_weight(self, name: str, tensor, layer: int = 0, stream=None):
        _check("evkcu_llm_set_weight", lib().evkcu_llm_set_weight(self.handle, name.encode(), layer, _ptr(tensor),
                                                                  _stream(stream)))

    def load(self, path: str, stream=None):
        """Loads every weight from a weight blob (see write_weight_blob)."""
        _check("evkcu_llm_load", lib().evkcu_llm_load(self.handle, os.fsencode(path), _stream(stream)))

    def save(self, path: str, stream=None):
        """Writes every weight to a weight blob (single-GPU models)."""
        _check("evkcu_llm_save", lib().evkcu_llm_save(self.handle, os.fsencode(path), _stream(stream)))

    def prefill(self, tokens, next_ids, logits=None, stream=None):
        B, S = tokens.shape
        _check("evkcu_llm_prefill", lib().evkcu_llm_prefill(self.handle, _ptr(tokens), B, S, _ptr(next_ids),
                                                            _ptr(logits), _stream(stream)))
        return next_ids

    def decode(self, ids, next_ids, logits=None, stream=None):
        _check("evkcu_llm_decode", lib().evkcu_llm_decode(self.handle, _ptr(ids), _ptr(next_ids), _ptr(logits),
                                                          _stream(stream)))
        return next_ids

    @property
    def fused_allreduce(self) -> bool:
        """Whether decode all-reduces run fused over peer memory (tensor parallel)."""
        return bool(lib().evkcu_llm_fused_allreduce(self.handle))

    @property
    def length(self) -> int:
        return int(lib().evkcu_llm_length(self.handle))


# ------------------------------------------------------------- weight blob --
BLOB_MAGIC = b"EVKWBLOB"


def blob_layout(layers, d_model, heads, hidden, vocab, kv_heads=None, tied_embeddings=True):
    """(name, layer, shape) of every tensor of a weight blob, in file order
    (include/evkcu.h, evkcu_llm_load)."""
    kv = kv_heads or heads
    dh = d_model // heads
    out = [("embedding", 0, (vocab, d_model))]
    if not tied_embeddings:
        out.append(("lm_head", 0, (d_model, vocab)))
    for l in range(layers):
        out += [("wqkv", l, (d_model, (heads + 2 * kv) * dh)), ("wo", l, (heads * dh, d_model)),
                ("w1", l, (d_model, hidden)), ("w2", l, (hidden, d_model))]
    return out


def write_weight_blob(path, weights, layers, d_model, heads, hidden, vocab, kv_heads=None, tied_embeddings=True,
                      dtype=F16):
    """Writes a weight blob from host arrays of 2-byte storage values.

    weights maps (name, layer) to an array with the blob_layout shape (any
    2-byte dtype: numpy uint16/float16, or torch half/bfloat16 on the CPU)."""
    import numpy as np

    kv = kv_heads or heads
    header = np.zeros(16, np.uint32)
    header[:2] = np.frombuffer(BLOB_MAGIC, np.uint32)
    header[2:11] = [1, dtype, layers, d_model, heads, kv, hidden, vocab, 1 if tied_embeddings else 0]
    with open(path, "wb") as f:
        f.write(header.tobytes())
        for name, layer, shape in blob_layout(layers, d_model, heads, hidden, vocab, kv, tied_embeddings):
            a = weights[(name, layer)]
            if hasattr(a, "numpy"):
                import torch

                a = a.detach().contiguous().cpu().view(torch.int16).numpy()
            a = np.ascontiguousarray(a)
            if a.dtype.itemsize != 2 or a.size != shape[0] * shape[1]:
                raise ValueError(f"{name}[{layer}]: expected {shape} of 2-byte values, got {a.shape} {a.dtype}")
            f.write(a.view(np.uint16).tobytes())
