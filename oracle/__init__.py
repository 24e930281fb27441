"""CPU oracle bindings — TEST INFRASTRUCTURE ONLY.

ctypes binding of ``oracle/liboracle.so`` (the C++ restatement of the
reference's shader math, ``evk_oracle.cpp``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
use it, and only as the checker or the timed CPU baseline; the product
(``evk_b200``) never imports it.

All arrays are numpy ``uint16`` views of 2-byte storage (fp16 = dtype 0,
bf16 = dtype 1).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32, _u64, _f32, _int, _vp = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p

_SIGS = {
    "oracle_matmul": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u64, _u64, _u64, _u32, _int],
    "oracle_flash_attention": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _u32, _int],
    "oracle_single_query_attention": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _f32, _int],
    "oracle_rms_norm": [_vp, _vp, _vp, _u32, _u32, _f32, _int],
    "oracle_rope": [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _int],
    "oracle_gelu": [_vp, _vp, _u64, _int],
    "oracle_softmax": [_vp, _vp, _u32, _u32, _f32, _int],
    "oracle_add": [_vp, _vp, _vp, _u64, _int],
    "oracle_scale": [_vp, _u64, _f32, _int],
    "oracle_causal_mask": [_vp, _u32, _u32, _int],
    "oracle_embed": [_vp, _vp, _vp, _u32, _u32, _u32, _u32],
    "oracle_greedy_sample": [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _u32, _int],
    "oracle_fill_normal": [_vp, _u64, _u64, _f32, _f32, _int],
    "oracle_fill_uniform_ids": [_vp, _u64, _u64, _u32, _u32, _u32],
    "oracle_quantize": [_vp, _vp, _u64, _int],
    "oracle_dequantize": [_vp, _vp, _u64, _int],
    "oracle_num_threads": [],
    "oracle_relu": [_vp, _vp, _u64, _int],
    "oracle_relu_backward": [_vp, _vp, _vp, _u64, _int],
    "oracle_gelu_backward": [_vp, _vp, _vp, _u64, _int],
    "oracle_softmax_backward": [_vp, _vp, _vp, _u32, _u32, _f32, _int],
    "oracle_rms_norm_backward": [_vp, _vp, _vp, _u32, _u32, _f32, _int],
    "oracle_rope_backward": [_vp, _vp, _u32, _u32, _u32, _f32, _int],
    "oracle_embed_backward": [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _int],
    "oracle_position_add": [_vp, _vp, _vp, _u32, _u32, _u32, _int],
    "oracle_position_add_backward": [_vp, _vp, _vp, _u32, _u32, _u32, _int],
    "oracle_sum_batch": [_vp, _vp, _u32, _u64, _int],
    "oracle_sgd": [_vp, _vp, _u64, _f32, _int],
    "oracle_adam": [_vp, _vp, _vp, _vp, _u64, _u32, _f32, _f32, _f32, _f32, _int],
    "oracle_mse_loss": [_vp, _vp, _vp, _vp, _u64, _int],
    "oracle_cross_entropy_loss": [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _int],
    "oracle_flash_attention_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _u32, _int],
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: build with `make -C oracle`")
        L = ctypes.CDLL(LIB_PATH)
        for n, a in _SIGS.items():
            f = getattr(L, n)
            f.argtypes = a
            f.restype = ctypes.c_int if n == "oracle_num_threads" else None
        _lib = L
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def normal(n, seed, std=1.0, mean=0.0, dtype=0):
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_fill_normal(_p(out), n, seed, mean, std, dtype)
    return out


def uniform_ids(n, seed, lo, hi, id_bytes=2):
    out = np.empty(n, dtype=np.uint16 if id_bytes == 2 else np.uint32)
    lib().oracle_fill_uniform_ids(_p(out), n, seed, lo, hi, id_bytes)
    return out


def to_float(a, dtype=0):
    out = np.empty(a.shape, dtype=np.float32)
    lib().oracle_dequantize(_p(np.ascontiguousarray(a)), _p(out), a.size, dtype)
    return out


def from_float(a, dtype=0):
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_quantize(_p(a), _p(out), a.size, dtype)
    return out


def num_threads():
    return lib().oracle_num_threads()


def matmul(A, B, C, batch, M, K, N, sa, sb, sc, flags, dtype=0):
    lib().oracle_matmul(_p(A), _p(B), _p(C), batch, M, K, N, sa, sb, sc, flags, dtype)
    return C


def flash_attention(q, k, v, o, B, N, H, Hkv, Dh, scale=0.0, flags=0, dtype=0):
    lib().oracle_flash_attention(_p(q), _p(k), _p(v), _p(o), B, N, H, Hkv, Dh, scale, flags, dtype)
    return o


def single_query_attention(q, kc, vc, out, B, H, Hkv, Dh, max_len, cur_len, scale=0.0, dtype=0):
    lib().oracle_single_query_attention(_p(q), _p(kc), _p(vc), _p(out), B, H, Hkv, Dh, max_len, cur_len, scale, dtype)
    return out


def rms_norm(x, out, rows, D, eps, gamma=None, dtype=0):
    lib().oracle_rms_norm(_p(x), _p(out), _p(gamma), rows, D, eps, dtype)
    return out


def rope(x, out, batch, seq, dim, head_dim=0, pos_offset=0, base=10000.0, dtype=0):
    lib().oracle_rope(_p(x), _p(out), batch, seq, dim, head_dim, pos_offset, base, dtype)
    return out


def gelu(x, out, dtype=0):
    lib().oracle_gelu(_p(x), _p(out), x.size, dtype)
    return out


def softmax(x, out, rows, L, scale=1.0, dtype=0):
    lib().oracle_softmax(_p(x), _p(out), rows, L, scale, dtype)
    return out


def add(a, b, c, dtype=0):
    lib().oracle_add(_p(a), _p(b), _p(c), a.size, dtype)
    return c


def scale(x, s, dtype=0):
    lib().oracle_scale(_p(x), x.size, s, dtype)
    return x


def causal_mask(s, batch, N, dtype=0):
    lib().oracle_causal_mask(_p(s), batch, N, dtype)
    return s


def embed(E, idx, out, vocab, dim):
    lib().oracle_embed(_p(E), _p(idx), _p(out), vocab, dim, idx.size, idx.dtype.itemsize)
    return out


def greedy_sample(logits, out, B, S, V, position, token_base, token_count, dtype=0):
    lib().oracle_greedy_sample(_p(logits), _p(out), B, S, V, position, token_base, token_count, out.dtype.itemsize,
                               dtype)
    return out


# ------------------------------------------------------------ training side --
def relu(x, out, dtype=0):
    lib().oracle_relu(_p(x), _p(out), x.size, dtype)
    return out


def relu_backward(go, x, gi, dtype=0):
    lib().oracle_relu_backward(_p(go), _p(x), _p(gi), x.size, dtype)
    return gi


def gelu_backward(go, x, gi, dtype=0):
    lib().oracle_gelu_backward(_p(go), _p(x), _p(gi), x.size, dtype)
    return gi


def softmax_backward(p, g, gi, rows, L, scale=1.0, dtype=0):
    lib().oracle_softmax_backward(_p(p), _p(g), _p(gi), rows, L, scale, dtype)
    return gi


def rms_norm_backward(x, g, gi, rows, D, eps, dtype=0):
    lib().oracle_rms_norm_backward(_p(x), _p(g), _p(gi), rows, D, eps, dtype)
    return gi


def rope_backward(go, gi, batch, seq, dim, base=10000.0, dtype=0):
    lib().oracle_rope_backward(_p(go), _p(gi), batch, seq, dim, base, dtype)
    return gi


def embed_backward(go, idx, gE, vocab, dim, dtype=0):
    lib().oracle_embed_backward(_p(go), _p(idx), _p(gE), vocab, dim, idx.size, idx.dtype.itemsize, dtype)
    return gE


def position_add(x, pos, out, batch, seq, dim, dtype=0):
    lib().oracle_position_add(_p(x), _p(pos), _p(out), batch, seq, dim, dtype)
    return out


def position_add_backward(go, gi, gp, batch, seq, dim, dtype=0):
    lib().oracle_position_add_backward(_p(go), _p(gi), _p(gp), batch, seq, dim, dtype)
    return gi, gp


def sum_batch(x, out, batch, size, dtype=0):
    lib().oracle_sum_batch(_p(x), _p(out), batch, size, dtype)
    return out


def sgd(p, g, lr, dtype=0):
    lib().oracle_sgd(_p(p), _p(g), p.size, lr, dtype)
    return p


def adam(p, g, m, v, step, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-4, dtype=0):
    lib().oracle_adam(_p(p), _p(g), _p(m), _p(v), p.size, step, lr, beta1, beta2, eps, dtype)
    return p


def mse_loss(pred, tgt, grad, result, dtype=0):
    lib().oracle_mse_loss(_p(pred), _p(tgt), _p(grad), _p(result), pred.size, dtype)
    return result


def cross_entropy_loss(logits, tgt, grad, result, rows, V, dtype=0):
    lib().oracle_cross_entropy_loss(_p(logits), _p(tgt), _p(grad), _p(result), rows, V, tgt.dtype.itemsize, dtype)
    return result


def flash_attention_bwd(q, k, v, dO, dQ, dK, dV, B, N, H, Hkv, Dh, scale=0.0, flags=0, dtype=0):
    lib().oracle_flash_attention_bwd(_p(q), _p(k), _p(v), _p(dO), _p(dQ), _p(dK), _p(dV), B, N, H, Hkv, Dh, scale,
                                     flags, dtype)
    return dQ, dK, dV
