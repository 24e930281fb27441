"""Reference decoder for the LLM-driver parity tests, composed from the CPU
oracle's op restatements (test infrastructure).

Same block as the driver (evk_b200/csrc/llm.cu) and example/main_llm.cpp's
CausalAttentionBlock: x += Wo(attn(rope(q), rope(k), v)) on rms_norm(x);
x += W2(gelu(W1 rms_norm(x))); logits = rms_norm(x) . LM head; greedy ids.
Every intermediate is rounded to the storage type at the same points as the
GPU path.  Two ways to run it:
- forward_last_logits recomputes the full sequence for each position (the
  reference's own decode strategy, example/main_llm.cpp:633-649);
- start / step keep per-layer K and V caches (rotated, rounded rows, as the
  driver stores them) and run single-query attention for each new token, so
  long greedy runs at the benchmark sizes finish in seconds.  The two agree
  up to the attention's summation order.
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

    def _head(self, xl, B):
        xln = np.empty_like(xl)
        oracle.rms_norm(xl, xln, B, self.D, self.eps, dtype=self.dt)
        if self.tied:
            return self._mm(xln, self.emb, B, self.D, self.V, tb=True).reshape(B, self.V)
        return self._mm(xln, self.lm_head, B, self.D, self.V).reshape(B, self.V)

    def _blocks(self, x, B, S, pos):
        """Runs every block on x [B*S, D] at positions pos..pos+S-1, appending
        the rotated K and V rows to the caches."""
        D, H, Dh, F, dt, Lm = self.D, self.H, self.Dh, self.F, self.dt, self.max_len
        R = B * S
        for l, w in enumerate(self.w):
            xn = np.empty_like(x)
            oracle.rms_norm(x, xn, R, D, self.eps, dtype=dt)
            qkv = self._mm(xn, w["wqkv"], R, D, 3 * D).reshape(R, 3 * D)
            q = np.ascontiguousarray(qkv[:, :D])
            k = np.ascontiguousarray(qkv[:, D:2 * D])
            v = np.ascontiguousarray(qkv[:, 2 * D:])
            qr, kr = np.empty_like(q), np.empty_like(k)
            oracle.rope(q, qr, B, S, D, Dh, pos, self.base, dt)
            oracle.rope(k, kr, B, S, D, Dh, pos, self.base, dt)
            kc = self.kc[l].reshape(B, Lm, D)
            vc = self.vc[l].reshape(B, Lm, D)
            kc[:, pos:pos + S] = kr.reshape(B, S, D)
            vc[:, pos:pos + S] = v.reshape(B, S, D)
            att = np.empty(R * D, np.uint16)
            if S == 1:
                oracle.single_query_attention(np.ascontiguousarray(qr.reshape(-1)), self.kc[l], self.vc[l], att, B, H,
                                              H, Dh, Lm, pos + 1, 0.0, dt)
            else:
                assert pos == 0, "multi-token chunks only at the start"
                oracle.flash_attention(qr, kr, v, att, B, S, H, H, Dh, 0.0, 1, dt)
            x = self._mm(att, w["wo"], R, D, D, acc=x)
            oracle.rms_norm(x, xn, R, D, self.eps, dtype=dt)
            h = self._mm(xn, w["w1"], R, D, F)
            hg = np.empty_like(h)
            oracle.gelu(h, hg, dt)
            x = self._mm(hg, w["w2"], R, F, D, acc=x)
        return x

    def start(self, tokens, max_len):
        """Prefill of tokens [B, S] with fresh caches of max_len positions;
        returns the last position's logits [B, V] (uint16)."""
        B, S = tokens.shape
        self.B, self.max_len, self.len = B, max_len, S
        self.kc = [np.zeros(B * max_len * self.D, np.uint16) for _ in self.w]
        self.vc = [np.zeros(B * max_len * self.D, np.uint16) for _ in self.w]
        ids = np.ascontiguousarray(tokens.reshape(-1).astype(np.uint32))
        x = np.empty(B * S * self.D, np.uint16)
        oracle.embed(self.emb, ids, x, self.V, self.D)
        x = self._blocks(x, B, S, 0)
        xl = np.ascontiguousarray(x.reshape(B, S, self.D)[:, -1, :]).reshape(-1)
        return self._head(xl, B)

    def step(self, ids):
        """One decode step: ids [B] appended at the current length; returns
        the new position's logits [B, V]."""
        B = self.B
        assert self.len < self.max_len
        x = np.empty(B * self.D, np.uint16)
        oracle.embed(self.emb, np.ascontiguousarray(np.asarray(ids, np.uint32)), x, self.V, self.D)
        x = self._blocks(x, B, 1, self.len)
        self.len += 1
        return self._head(x, B)

    def greedy(self, logits):
        B, V = logits.shape
        out = np.zeros(B, np.uint32)
        oracle.greedy_sample(np.ascontiguousarray(logits).reshape(-1), out, B, 1, V, 0, 0, V, self.dt)
        return out
