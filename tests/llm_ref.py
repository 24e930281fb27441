"""Reference decoder for the LLM-driver parity tests, composed from the CPU
oracle's op restatements (test infrastructure).

Same block as the driver (evk_b200/csrc/llm.cu) and example/main_llm.cpp's
CausalAttentionBlock: x += Wo(attn(rope(q), rope(k), v)) on rms_norm(x);
x += W2(gelu(W1 rms_norm(x))); logits = rms_norm(x) . LM head; greedy ids.
Every intermediate is rounded to the storage type at the same points as the
GPU path; the full sequence is recomputed for each position (the reference's
own decode strategy, example/main_llm.cpp:633-649).
"""
import numpy as np

import oracle


class RefModel:
    def __init__(self, layers, d_model, heads, hidden, vocab, tied, dtype=0, seed=5, std=0.02, rope_base=10000.0,
                 eps=1e-5):
        self.L, self.D, self.H, self.F, self.V = layers, d_model, heads, hidden, vocab
        self.Dh = d_model // heads
        self.tied, self.dt, self.base, self.eps = tied, dtype, rope_base, eps
        s = seed
        self.emb = oracle.normal(vocab * d_model, s, std, dtype=dtype)
        self.lm_head = None if tied else oracle.normal(d_model * vocab, s + 1, std, dtype=dtype)
        self.w = []
        for l in range(layers):
            b = s + 10 * (l + 1)
            self.w.append({
                "wqkv": oracle.normal(d_model * 3 * d_model, b, std, dtype=dtype),
                "wo": oracle.normal(d_model * d_model, b + 1, std, dtype=dtype),
                "w1": oracle.normal(d_model * hidden, b + 2, std, dtype=dtype),
                "w2": oracle.normal(hidden * d_model, b + 3, std, dtype=dtype),
            })

    def _mm(self, a, b, M, K, N, acc=None, tb=False):
        c = acc.copy() if acc is not None else np.empty(M * N, np.uint16)
        flags = (2 if tb else 0) | (4 if acc is not None else 0)
        oracle.matmul(a, b, c, 1, M, K, N, M * K, K * N, M * N, flags, self.dt)
        return c

    def forward_last_logits(self, tokens):
        """tokens [B, S] -> logits [B, V] (uint16) of the last position."""
        B, S = tokens.shape
        D, H, Dh, F, dt = self.D, self.H, self.Dh, self.F, self.dt
        R = B * S
        ids = np.ascontiguousarray(tokens.reshape(-1).astype(np.uint32))
        x = np.empty(R * D, np.uint16)
        oracle.embed(self.emb, ids, x, self.V, D)
        for w in self.w:
            xn = np.empty_like(x)
            oracle.rms_norm(x, xn, R, D, self.eps, dtype=dt)
            qkv = self._mm(xn, w["wqkv"], R, D, 3 * D).reshape(R, 3 * D)
            q = np.ascontiguousarray(qkv[:, :D])
            k = np.ascontiguousarray(qkv[:, D:2 * D])
            v = np.ascontiguousarray(qkv[:, 2 * D:])
            qr, kr = np.empty_like(q), np.empty_like(k)
            oracle.rope(q, qr, B, S, D, Dh, 0, self.base, dt)
            oracle.rope(k, kr, B, S, D, Dh, 0, self.base, dt)
            att = np.empty(R * D, np.uint16)
            oracle.flash_attention(qr, kr, v, att, B, S, H, H, Dh, 0.0, 1, dt)
            x = self._mm(att, w["wo"], R, D, D, acc=x)
            oracle.rms_norm(x, xn, R, D, self.eps, dtype=dt)
            h = self._mm(xn, w["w1"], R, D, F)
            hg = np.empty_like(h)
            oracle.gelu(h, hg, dt)
            x = self._mm(hg, w["w2"], R, F, D, acc=x)
        xl = np.ascontiguousarray(x.reshape(B, S, D)[:, -1, :]).reshape(-1)
        xln = np.empty_like(xl)
        oracle.rms_norm(xl, xln, B, D, self.eps, dtype=dt)
        if self.tied:
            return self._mm(xln, self.emb, B, D, self.V, tb=True).reshape(B, self.V)
        return self._mm(xln, self.lm_head, B, D, self.V).reshape(B, self.V)

    def greedy(self, logits):
        B, V = logits.shape
        out = np.zeros(B, np.uint32)
        oracle.greedy_sample(np.ascontiguousarray(logits).reshape(-1), out, B, 1, V, 0, 0, V, self.dt)
        return out
