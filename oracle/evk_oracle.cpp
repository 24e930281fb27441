// evk_oracle.cpp — CPU restatement of the reference's evk::ai shader math.
// TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline); see
// evk_oracle.h.  Citations are paths within carloshgsilva/evk.
#include "evk_oracle.h"

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// Dynamic parallel-for over [0, n) on all hardware threads (or
// EVK_ORACLE_THREADS), in chunks of `grain` indices.
int n_threads() {
    static int n = [] {
        const char* e = std::getenv("EVK_ORACLE_THREADS");
        int v = e ? std::atoi(e) : 0;
        if (v <= 0) v = (int)std::thread::hardware_concurrency();
        return v > 0 ? v : 1;
    }();
    return n;
}
template <class F>
void par_for(int64_t n, F fn, int64_t grain = 1) {
    if (n <= 0) return;
    const int nt = (int)std::min<int64_t>(n_threads(), (n + grain - 1) / grain);
    if (nt <= 1) {
        for (int64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::atomic<int64_t> next{0};
    auto worker = [&] {
        for (;;) {
            const int64_t b = next.fetch_add(grain);
            if (b >= n) return;
            const int64_t e = std::min(n, b + grain);
            for (int64_t i = b; i < e; ++i) fn(i);
        }
    };
    std::vector<std::thread> ts;
    for (int t = 1; t < nt; ++t) ts.emplace_back(worker);
    worker();
    for (auto& t : ts) t.join();
}


// ---- 2-byte float formats ---------------------------------------------------
// fp32 -> fp16 following float16_t::float_to_float16 (evk_ai.h:52-121):
// Inf/NaN keep their class (NaN payload's top bits, forced non-zero), values
// above the fp16 range overflow to Inf, normals round to nearest-even, values
// below 2^-24 flush to a signed zero and subnormals round half-up.
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t bexp = (x >> 23) & 0xFFu;
    uint32_t frac = x & 0x7FFFFFu;
    if (bexp == 0xFFu) {
        if (frac == 0) return sign | 0x7C00u;
        uint16_t pl = (uint16_t)((frac >> 13) & 0x3FFu);
        return sign | 0x7C00u | (pl ? pl : 1u);
    }
    const int e = (int)bexp - 127;
    if (e > 15) return sign | 0x7C00u;
    if (e >= -14) {
        uint32_t he = (uint32_t)(e + 15);
        uint32_t m = frac >> 13;
        const uint32_t rest = frac & 0x1FFFu;
        if (rest > 0x1000u || (rest == 0x1000u && (m & 1u))) {
            if (++m == 0x400u) {
                m = 0;
                if (++he == 0x1Fu) return sign | 0x7C00u;
            }
        }
        return sign | (uint16_t)(he << 10) | (uint16_t)m;
    }
    if (e < -24) return sign;
    frac |= 0x800000u;
    const int sh = -14 - e;  // 1..10
    uint32_t m = frac >> (13 + sh);
    if ((frac >> (12 + sh)) & 1u) ++m;
    return sign | (uint16_t)(m & 0x3FFu);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    float out;
    if (e == 0) {
        out = std::ldexp((float)m, -24);
        return sign ? -out : out;
    }
    uint32_t bits;
    if (e == 0x1Fu)
        bits = sign | 0x7F800000u | (m << 13);
    else
        bits = sign | ((e + 112u) << 23) | (m << 13);
    std::memcpy(&out, &bits, 4);
    return out;
}

// bf16: the upper half of fp32, round-to-nearest-even; NaN stays quiet NaN.
uint16_t f32_to_bf16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    const uint32_t lsb = (x >> 16) & 1u;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}
float bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline float ld(const uint16_t* p, uint64_t i, int dt) { return dt ? bf16_to_f32(p[i]) : f16_to_f32(p[i]); }
inline uint16_t st(float f, int dt) { return dt ? f32_to_bf16(f) : f32_to_f16(f); }

inline uint64_t splitmix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

}  // namespace

extern "C" {

uint16_t oracle_f32_to_f16(float f) { return f32_to_f16(f); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
float oracle_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }

void oracle_quantize(const float* in, uint16_t* out, uint64_t n, int dtype) {
    par_for((int64_t)n, [&](int64_t i) { out[i] = st(in[i], dtype); }, 1 << 16);
}
void oracle_dequantize(const uint16_t* in, float* out, uint64_t n, int dtype) {
    par_for((int64_t)n, [&](int64_t i) { out[i] = ld(in, i, dtype); }, 1 << 16);
}

int oracle_num_threads(void) { return n_threads(); }

// shaders/matmul.comp:44-140 with evk_ai.cpp:254-330: C[b] = op(A[b]) op(B[b])
// (+C[b]); A read column-major when transposed (matmul.comp:71-82); stride 0
// broadcasts an operand over the batch (evk_ai.cpp:299-304).
void oracle_matmul(const uint16_t* A, const uint16_t* B, uint16_t* C, uint32_t batch, uint32_t M, uint32_t K,
                   uint32_t N, uint64_t stride_a, uint64_t stride_b, uint64_t stride_c, uint32_t flags, int dt) {
    const bool ta = flags & 1u, tb = flags & 2u, acc = flags & 4u;
    // Rows are independent; with few rows (decode shapes) each row is also
    // split into column chunks so every thread has work.  The chunking does
    // not change any element's summation order.
    const int64_t rows = (int64_t)batch * M;
    int64_t chunks = 1;
    if (rows < 4 * n_threads()) chunks = std::min<int64_t>((4 * n_threads() + rows - 1) / rows, (N + 255) / 256);
    if (chunks < 1) chunks = 1;
    const uint32_t cw = (uint32_t)((N + chunks - 1) / chunks);
    par_for(rows * chunks, [&](int64_t task) {
        {
            const int64_t bm = task / chunks, ch = task % chunks;
            const int64_t b = bm / M, m = bm % M;
            const uint32_t n0 = (uint32_t)std::min<int64_t>((int64_t)ch * cw, N);
            const uint32_t n1 = (uint32_t)std::min<int64_t>((int64_t)n0 + cw, N);
            if (n0 >= n1) return;
            const uint16_t* a = A + b * stride_a;
            const uint16_t* bb = B + b * stride_b;
            uint16_t* c = C + b * stride_c;
            std::vector<float> arow(K);
            for (uint32_t k = 0; k < K; ++k) arow[k] = ld(a, ta ? (uint64_t)k * M + m : (uint64_t)m * K + k, dt);
            std::vector<double> acc_row(n1 - n0, 0.0);
            if (!tb) {
                for (uint32_t k = 0; k < K; ++k) {
                    const double av = arow[k];
                    if (av == 0.0) continue;
                    const uint16_t* brow = bb + (uint64_t)k * N;
                    for (uint32_t n = n0; n < n1; ++n) acc_row[n - n0] += av * (double)ld(brow, n, dt);
                }
            } else {
                for (uint32_t n = n0; n < n1; ++n) {
                    const uint16_t* brow = bb + (uint64_t)n * K;
                    double s = 0.0;
                    for (uint32_t k = 0; k < K; ++k) s += (double)arow[k] * (double)ld(brow, k, dt);
                    acc_row[n - n0] = s;
                }
            }
            for (uint32_t n = n0; n < n1; ++n) {
                double v = acc_row[n - n0];
                if (acc) v += (double)ld(c, (uint64_t)m * N + n, dt);
                c[(uint64_t)m * N + n] = st((float)v, dt);
            }
        }
    });
}

// shaders/flash_attention.comp:53-185: per head, O = softmax(Q K^T * scale) V
// with the final 1/l (0 when l = 0, :166).  K/V head g = h / (H / Hkv); the
// reference is Hkv = 1 and non-causal; flag bit 0 adds the causal mask j <= i.
void oracle_flash_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, uint32_t B,
                            uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dt) {
    const bool causal = flags & 1u;
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)Dh);
    const uint64_t qp = (uint64_t)H * Dh, kp = (uint64_t)Hkv * Dh;
    par_for((int64_t)B * H * N, [&](int64_t bhi) {
            const int64_t i = bhi % N, h = (bhi / N) % H, b = bhi / ((int64_t)N * H);
            {
                const uint32_t g = (uint32_t)h / (H / Hkv);
                std::vector<float> qv(Dh);
                for (uint32_t d = 0; d < Dh; ++d) qv[d] = ld(q, (b * N + i) * qp + h * Dh + d, dt);
                const uint32_t jend = causal ? (uint32_t)i + 1 : N;
                std::vector<double> s(jend);
                double mx = -INFINITY;
                for (uint32_t j = 0; j < jend; ++j) {
                    const uint64_t kb = (b * N + j) * kp + (uint64_t)g * Dh;
                    double acc = 0.0;
                    for (uint32_t d = 0; d < Dh; ++d) acc += (double)qv[d] * (double)ld(k, kb + d, dt);
                    s[j] = acc * (double)scale;
                    mx = std::max(mx, s[j]);
                }
                std::vector<double> out(Dh, 0.0);
                double l = 0.0;
                for (uint32_t j = 0; j < jend; ++j) {
                    const double p = std::exp(s[j] - mx);
                    l += p;
                    const uint64_t vb = (b * N + j) * kp + (uint64_t)g * Dh;
                    for (uint32_t d = 0; d < Dh; ++d) out[d] += p * (double)ld(v, vb + d, dt);
                }
                const double inv = l > 0.0 ? 1.0 / l : 0.0;
                for (uint32_t d = 0; d < Dh; ++d) o[(b * N + i) * qp + h * Dh + d] = st((float)(out[d] * inv), dt);
            }
    }, 16);
}

// shaders/single_query_attention.comp:27-71: o = softmax(q K^T * dim^-1/2) V
// over the first cur_len positions, 0 when the weight sum is 0.  Generalised
// to B sequences and H query heads over Hkv cached heads.
void oracle_single_query_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* out,
                                   uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t max_len,
                                   uint32_t cur_len, float scale, int dt) {
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)Dh);
    const uint64_t kp = (uint64_t)Hkv * Dh;
    par_for((int64_t)B * H, [&](int64_t bh) {
        const int64_t b = bh / H, h = bh % H;
        {
            const uint32_t g = (uint32_t)h / (H / Hkv);
            std::vector<double> s(cur_len);
            double mx = -INFINITY;
            for (uint32_t p = 0; p < cur_len; ++p) {
                const uint64_t kb = ((uint64_t)b * max_len + p) * kp + (uint64_t)g * Dh;
                double acc = 0.0;
                for (uint32_t d = 0; d < Dh; ++d)
                    acc += (double)ld(q, ((uint64_t)b * H + h) * Dh + d, dt) * (double)ld(kc, kb + d, dt);
                s[p] = acc * scale;
                mx = std::max(mx, s[p]);
            }
            double l = 0.0;
            std::vector<double> o(Dh, 0.0);
            for (uint32_t p = 0; p < cur_len; ++p) {
                const double w = std::exp(s[p] - mx);
                l += w;
                const uint64_t vb = ((uint64_t)b * max_len + p) * kp + (uint64_t)g * Dh;
                for (uint32_t d = 0; d < Dh; ++d) o[d] += w * (double)ld(vc, vb + d, dt);
            }
            const double inv = l > 0.0 ? 1.0 / l : 0.0;
            for (uint32_t d = 0; d < Dh; ++d) out[((uint64_t)b * H + h) * Dh + d] = st((float)(o[d] * inv), dt);
        }
    });
}

// shaders/rms_norm.comp:21-48 — clamp to +-65504, fp32 sum of squares,
// inversesqrt(mean + eps); gamma (extension) multiplies after normalising.
void oracle_rms_norm(const uint16_t* in, uint16_t* out, const uint16_t* gamma, uint32_t rows, uint32_t D, float eps,
                     int dt) {
    par_for((int64_t)rows, [&](int64_t r) {
        const uint64_t base = (uint64_t)r * D;
        float ss = 0.0f;
        for (uint32_t j = 0; j < D; ++j) {
            float x = std::fmin(std::fmax(ld(in, base + j, dt), -65504.0f), 65504.0f);
            ss += x * x;
        }
        const float inv = 1.0f / std::sqrt(ss / (float)D + eps);
        for (uint32_t j = 0; j < D; ++j) {
            float x = std::fmin(std::fmax(ld(in, base + j, dt), -65504.0f), 65504.0f) * inv;
            if (gamma) x *= ld(gamma, j, dt);
            out[base + j] = st(x, dt);
        }
    }, 64);
}

// shaders/rope.comp:18-40 — pair p of each rot_dim slice at position t:
// angle = t * base^(-2p/rot_dim); (x0, x1) -> (x0 c - x1 s, x0 s + x1 c).
void oracle_rope(const uint16_t* in, uint16_t* out, uint32_t batch, uint32_t seq_len, uint32_t dim, uint32_t head_dim,
                 uint32_t pos_offset, float base, int dt) {
    if (head_dim == 0) head_dim = dim;
    const uint64_t rows = (uint64_t)batch * seq_len;
    par_for((int64_t)rows, [&](int64_t r) {
        const float t = (float)((uint32_t)(r % seq_len) + pos_offset);
        for (uint32_t c = 0; c < dim; c += 2) {
            const uint32_t p = (c % head_dim) / 2;
            const float inv_freq = std::pow(base, -2.0f * (float)p / (float)head_dim);
            const float ang = t * inv_freq;
            const float cs = std::cos(ang), sn = std::sin(ang);
            const float x0 = ld(in, r * dim + c, dt), x1 = ld(in, r * dim + c + 1, dt);
            out[r * dim + c] = st(x0 * cs - x1 * sn, dt);
            out[r * dim + c + 1] = st(x0 * sn + x1 * cs, dt);
        }
    }, 64);
}

// shaders/gelu.comp:15-21 — tanh approximation in fp32.
void oracle_gelu(const uint16_t* in, uint16_t* out, uint64_t n, int dt) {
    par_for((int64_t)n, [&](int64_t i) {
        const float x = ld(in, i, dt);
        const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
        out[i] = st(0.5f * x * (1.0f + std::tanh(u)), dt);
    }, 64);
}

// shaders/softmax.comp:23-66 — masked (raw <= -65504) entries are skipped and
// written 0; row max and exp-sum in fp32; sum clamped to >= 1e-20.
void oracle_softmax(const uint16_t* in, uint16_t* out, uint32_t rows, uint32_t L, float scale, int dt) {
    par_for((int64_t)rows, [&](int64_t r) {
        const uint64_t base = (uint64_t)r * L;
        float mx = -FLT_MAX;
        for (uint32_t j = 0; j < L; ++j) {
            float raw = ld(in, base + j, dt);
            if (raw <= -65504.0f) continue;
            mx = std::fmax(mx, raw * scale);
        }
        float sum = 0.0f;
        for (uint32_t j = 0; j < L; ++j) {
            float raw = ld(in, base + j, dt);
            if (raw <= -65504.0f) continue;
            sum += std::exp(raw * scale - mx);
        }
        const float inv = 1.0f / std::fmax(sum, 1e-20f);
        for (uint32_t j = 0; j < L; ++j) {
            float raw = ld(in, base + j, dt);
            out[base + j] = raw <= -65504.0f ? st(0.0f, dt) : st(std::exp(raw * scale - mx) * inv, dt);
        }
    }, 64);
}

// shaders/add.comp:18-26
void oracle_add(const uint16_t* a, const uint16_t* b, uint16_t* c, uint64_t n, int dt) {
    par_for((int64_t)n, [&](int64_t i) { c[i] = st(ld(a, i, dt) + ld(b, i, dt), dt); }, 1 << 14);
}

// shaders/scale.comp (in place)
void oracle_scale(uint16_t* x, uint64_t n, float s, int dt) {
    par_for((int64_t)n, [&](int64_t i) { x[i] = st(ld(x, i, dt) * s, dt); }, 1 << 14);
}

// shaders/causal_mask.comp:29-32 — j > i set to -65504.
void oracle_causal_mask(uint16_t* s, uint32_t batch, uint32_t N, int dt) {
    const uint16_t sent = st(-65504.0f, dt);
    par_for((int64_t)batch * N, [&](int64_t r) {
        const uint32_t i = (uint32_t)(r % N);
        for (uint32_t j = i + 1; j < N; ++j) s[(uint64_t)r * N + j] = sent;
    }, 64);
}

// shaders/embed.comp:18-28 — out[i,:] = E[idx[i],:] (index clamped to the
// vocabulary, as the CUDA backend does, instead of reading out of bounds).
void oracle_embed(const uint16_t* E, const void* idx, uint16_t* out, uint32_t vocab, uint32_t dim, uint32_t n_idx,
                  uint32_t idx_bytes) {
    par_for((int64_t)n_idx, [&](int64_t i) {
        uint32_t t = idx_bytes == 2 ? ((const uint16_t*)idx)[i] : ((const uint32_t*)idx)[i];
        if (t >= vocab) t = vocab - 1;
        std::memcpy(out + (uint64_t)i * dim, E + (uint64_t)t * dim, (size_t)dim * 2);
    }, 64);
}

// shaders/greedy_sample.comp:24-64, literally: 256 lanes scan j = lane,
// lane+256, ... keeping the first strict maximum (start -FLT_MAX / token_base),
// then the shared-memory tree at strides 128..1 taking the partner only when
// strictly greater.
void oracle_greedy_sample(const uint16_t* logits, void* out, uint32_t B, uint32_t S, uint32_t V, uint32_t position,
                          uint32_t token_base, uint32_t token_count, uint32_t out_bytes, int dt) {
    for (uint32_t b = 0; b < B; ++b) {
        const uint64_t row = ((uint64_t)b * S + position) * V;
        float bv[256];
        uint32_t bt[256];
        for (uint32_t lid = 0; lid < 256; ++lid) {
            bv[lid] = -FLT_MAX;
            bt[lid] = token_base;
            for (uint32_t j = lid; j < token_count; j += 256) {
                const uint32_t tok = token_base + j;
                const float v = ld(logits, row + tok, dt);
                if (v > bv[lid]) {
                    bv[lid] = v;
                    bt[lid] = tok;
                }
            }
        }
        for (uint32_t s = 128; s > 0; s >>= 1)
            for (uint32_t lid = 0; lid < s; ++lid)
                if (bv[lid + s] > bv[lid]) {
                    bv[lid] = bv[lid + s];
                    bt[lid] = bt[lid + s];
                }
        if (out_bytes == 2)
            ((uint16_t*)out)[b] = (uint16_t)bt[0];
        else
            ((uint32_t*)out)[b] = bt[0];
    }
}

// ---- training side -------------------------------------------------------
// shaders/relu.comp: out = max(0, x)
void oracle_relu(const uint16_t* in, uint16_t* out, uint64_t n, int dt) {
    par_for((int64_t)n, [&](int64_t i) { out[i] = st(std::max(0.0f, ld(in, i, dt)), dt); }, 4096);
}
// shaders/relu_bwd.comp: gi += x > 0 ? go : 0
void oracle_relu_backward(const uint16_t* go, const uint16_t* in, uint16_t* gi, uint64_t n, int dt) {
    par_for((int64_t)n, [&](int64_t i) {
        gi[i] = st(ld(gi, i, dt) + (ld(in, i, dt) > 0.0f ? ld(go, i, dt) : 0.0f), dt);
    }, 4096);
}
// shaders/gelu_bwd.comp:16-37: gi += go * gelu'(x), tanh form
void oracle_gelu_backward(const uint16_t* go, const uint16_t* in, uint16_t* gi, uint64_t n, int dt) {
    par_for((int64_t)n, [&](int64_t i) {
        const double x = ld(in, i, dt);
        const double kA = 0.7978845608028654, kB = 0.044715;
        const double t = std::tanh(kA * (x + kB * x * x * x));
        const double g = 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * kA * (1.0 + 3.0 * kB * x * x);
        gi[i] = st((float)(ld(gi, i, dt) + ld(go, i, dt) * g), dt);
    }, 4096);
}
// shaders/softmax_bwd.comp: gi += p (g - dot(g, p)) scale per row
void oracle_softmax_backward(const uint16_t* p, const uint16_t* g, uint16_t* gi, uint32_t rows, uint32_t L,
                             float scale, int dt) {
    par_for((int64_t)rows, [&](int64_t r) {
        const uint64_t b = (uint64_t)r * L;
        double dot = 0.0;
        for (uint32_t j = 0; j < L; ++j) dot += (double)ld(p, b + j, dt) * ld(g, b + j, dt);
        for (uint32_t j = 0; j < L; ++j)
            gi[b + j] = st((float)(ld(gi, b + j, dt) + ld(p, b + j, dt) * (ld(g, b + j, dt) - dot) * scale), dt);
    });
}
// shaders/rms_norm_bwd.comp:21-74: x clamped to +-65504, rms = sqrt(mean x^2 + eps),
// gi += g / rms - x / rms^2 * dot(g, x / rms) / D
void oracle_rms_norm_backward(const uint16_t* x, const uint16_t* g, uint16_t* gi, uint32_t rows, uint32_t D,
                              float eps, int dt) {
    par_for((int64_t)rows, [&](int64_t r) {
        const uint64_t b = (uint64_t)r * D;
        auto xv = [&](uint32_t j) { return (double)std::min(std::max(ld(x, b + j, dt), -65504.0f), 65504.0f); };
        double ss = 0.0;
        for (uint32_t j = 0; j < D; ++j) ss += xv(j) * xv(j);
        const double inv = 1.0 / std::sqrt(ss / D + (double)eps);
        double dot = 0.0;
        for (uint32_t j = 0; j < D; ++j) dot += ld(g, b + j, dt) * xv(j) * inv;
        const double sc = dot / D;
        for (uint32_t j = 0; j < D; ++j)
            gi[b + j] = st((float)(ld(gi, b + j, dt) + ld(g, b + j, dt) * inv - xv(j) * inv * inv * sc), dt);
    });
}
// shaders/rope_bwd.comp: transpose rotation (angle t * base^(-2p/D)), accumulated
void oracle_rope_backward(const uint16_t* go, uint16_t* gi, uint32_t batch, uint32_t seq_len, uint32_t dim,
                          float base, int dt) {
    const uint64_t rows = (uint64_t)batch * seq_len;
    par_for((int64_t)rows, [&](int64_t r) {
        const float t = (float)(uint32_t)(r % seq_len);
        for (uint32_t c = 0; c < dim; c += 2) {
            const float inv_freq = std::pow(base, -2.0f * (float)(c / 2) / (float)dim);
            const float ang = t * inv_freq;
            const float cs = std::cos(ang), sn = std::sin(ang);
            const uint64_t i0 = r * dim + c;
            const float g0 = ld(go, i0, dt), g1 = ld(go, i0 + 1, dt);
            gi[i0] = st(ld(gi, i0, dt) + g0 * cs + g1 * sn, dt);
            gi[i0 + 1] = st(ld(gi, i0 + 1, dt) - g0 * sn + g1 * cs, dt);
        }
    }, 64);
}
// shaders/embed_bwd.comp: gE[idx[i], d] += go[i, d] over i in order, rounding after each add
void oracle_embed_backward(const uint16_t* go, const void* idx, uint16_t* gE, uint32_t vocab, uint32_t dim,
                           uint32_t n_idx, uint32_t idx_bytes, int dt) {
    par_for((int64_t)dim, [&](int64_t d) {
        for (uint32_t i = 0; i < n_idx; ++i) {
            const uint32_t tok = idx_bytes == 2 ? ((const uint16_t*)idx)[i] : ((const uint32_t*)idx)[i];
            if (tok >= vocab) continue;
            const uint64_t o = (uint64_t)tok * dim + d;
            gE[o] = st(ld(gE, o, dt) + ld(go, (uint64_t)i * dim + d, dt), dt);
        }
    });
}
// shaders/position_add.comp: out[b,t,d] = in[b,t,d] + pos[t,d]
void oracle_position_add(const uint16_t* in, const uint16_t* pos, uint16_t* out, uint32_t batch, uint32_t seq_len,
                         uint32_t dim, int dt) {
    const uint64_t n = (uint64_t)batch * seq_len * dim, per = (uint64_t)seq_len * dim;
    par_for((int64_t)n, [&](int64_t i) { out[i] = st(ld(in, i, dt) + ld(pos, i % per, dt), dt); }, 4096);
}
// shaders/sum_batch.comp: out[i] += sum_b in[b * size + i] (fp32, rounded once)
void oracle_sum_batch(const uint16_t* in, uint16_t* out, uint32_t batch, uint64_t size, int dt) {
    par_for((int64_t)size, [&](int64_t i) {
        float s = ld(out, i, dt);
        for (uint32_t b = 0; b < batch; ++b) s += ld(in, (uint64_t)b * size + i, dt);
        out[i] = st(s, dt);
    }, 4096);
}
// shaders/position_add_bwd.comp: mode 0 gi += go; mode 1 gp += sum_b go
void oracle_position_add_backward(const uint16_t* go, uint16_t* gi, uint16_t* gp, uint32_t batch, uint32_t seq_len,
                                  uint32_t dim, int dt) {
    const uint64_t n = (uint64_t)batch * seq_len * dim;
    par_for((int64_t)n, [&](int64_t i) { gi[i] = st(ld(gi, i, dt) + ld(go, i, dt), dt); }, 4096);
    oracle_sum_batch(go, gp, batch, (uint64_t)seq_len * dim, dt);
}
// shaders/sgd.comp
void oracle_sgd(uint16_t* p, const uint16_t* g, uint64_t n, float lr, int dt) {
    par_for((int64_t)n, [&](int64_t i) { p[i] = st(ld(p, i, dt) - lr * ld(g, i, dt), dt); }, 4096);
}
// shaders/adam.comp with evk_ai.cpp:525-566 (bias corrections from the step)
void oracle_adam(uint16_t* p, const uint16_t* g, uint16_t* mb, uint16_t* vb, uint64_t n, uint32_t step, float lr,
                 float b1, float b2, float eps, int dt) {
    const float c1 = 1.0f / (1.0f - std::pow(b1, (float)step));
    const float c2 = 1.0f / (1.0f - std::pow(b2, (float)step));
    par_for((int64_t)n, [&](int64_t i) {
        const float grad = ld(g, i, dt);
        if (std::isnan(grad) || std::isinf(grad)) return;
        const float stored = ld(vb, i, dt);
        float rms = stored > 0.0f ? std::exp2(stored - 41.0f) : 0.0f;
        float m = ld(mb, i, dt) * rms;
        float v = rms * rms;
        m = b1 * m + (1.0f - b1) * grad;
        v = b2 * v + (1.0f - b2) * grad * grad;
        rms = std::sqrt(std::max(v, 0.0f));
        const float mn = m / std::max(rms, 1.0e-8f);
        if (!std::isnan(mn) && !std::isinf(mn)) mb[i] = st(mn, dt);
        const float lg = std::log2(std::max(rms, 1.0e-12f)) + 41.0f;
        if (!std::isnan(lg) && !std::isinf(lg)) vb[i] = st(lg, dt);
        const float upd = lr * (m * c1) / (rms * std::sqrt(c2) + eps);
        if (!std::isnan(upd) && !std::isinf(upd))
            p[i] = st(std::min(std::max(ld(p, i, dt) - upd, -65504.0f), 65504.0f), dt);
    }, 4096);
}
// shaders/mse_loss.comp: grad = 2 (p - t) / n; result = mean (p - t)^2
void oracle_mse_loss(const uint16_t* pred, const uint16_t* tgt, uint16_t* grad, uint16_t* result, uint64_t n,
                     int dt) {
    double s = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        const float d = ld(pred, i, dt) - ld(tgt, i, dt);
        s += (double)d * d;
        grad[i] = st(2.0f / (float)n * d, dt);
    }
    result[0] = st((float)(s / (double)n), dt);
}
// shaders/cross_entropy_count.comp, cross_entropy.comp, cross_entropy_scale.comp:
// logits clamped to +-65000; valid rows (0 < t < V) get
// grad = (softmax - onehot(t)) / count and loss (max + ln sum e^(l - max) - l_t) / count;
// other rows zero gradient.  Result = sum of row losses (0 if none / not finite).
void oracle_cross_entropy_loss(const uint16_t* logits, const void* tgt, uint16_t* grad, uint16_t* result,
                               uint32_t rows, uint32_t V, uint32_t target_bytes, int dt) {
    auto target = [&](uint32_t r) {
        return target_bytes == 2 ? (uint32_t)((const uint16_t*)tgt)[r] : ((const uint32_t*)tgt)[r];
    };
    double count = 0.0;
    for (uint32_t r = 0; r < rows; ++r) count += (target(r) != 0 && target(r) < V) ? 1.0 : 0.0;
    std::vector<double> loss(rows, 0.0);
    par_for((int64_t)rows, [&](int64_t r) {
        const uint64_t b = (uint64_t)r * V;
        const uint32_t t = target((uint32_t)r);
        if (!(t != 0 && t < V && count > 0.0)) {
            for (uint32_t j = 0; j < V; ++j) grad[b + j] = st(0.0f, dt);
            return;
        }
        auto lv = [&](uint32_t j) { return (double)std::min(std::max(ld(logits, b + j, dt), -65000.0f), 65000.0f); };
        double mx = -1e300;
        for (uint32_t j = 0; j < V; ++j) mx = std::max(mx, lv(j));
        double den = 0.0;
        for (uint32_t j = 0; j < V; ++j) den += std::exp(lv(j) - mx);
        den = std::max(den, 1e-20);
        for (uint32_t j = 0; j < V; ++j) {
            double gv = std::exp(lv(j) - mx) / den / count;
            if (j == t) gv -= 1.0 / count;
            grad[b + j] = st((float)gv, dt);
        }
        loss[r] = (mx + std::log(den) - lv(t)) / count;
    });
    double s = 0.0;
    for (uint32_t r = 0; r < rows; ++r) s += loss[r];
    if (!(count > 0.0) || std::isnan(s) || std::isinf(s)) s = 0.0;
    result[0] = st((float)s, dt);
}
// shaders/flash_attention_bwd.comp (modes 0 and 1), restated per element:
// s_ij = q_i.k_j * scale, m_i / l_i / t_i the row max, exp-sum and
// sum_j e^(s_ij - m_i) (dO_i.v_j); p_ij = e^(s_ij - m_i) / l_i;
// a_ij = (dO_i.v_j - c_i) p_ij scale with c_i = t_i (the shader) or t_i / l_i
// (flag 2, exact gradient); dQ_i = sum_j a_ij k_j, dK_j = sum_{h,i} a_ij q_i,
// dV_j = sum_{h,i} p_ij dO_i.  K/V head g serves heads g*H/Hkv ...; flag 1 causal.
void oracle_flash_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* dO,
                                uint16_t* dQ, uint16_t* dK, uint16_t* dV, uint32_t B, uint32_t N, uint32_t H,
                                uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dt) {
    const bool causal = flags & 1u, normalized = flags & 2u;
    if (!(scale > 0.0f)) scale = 1.0f / std::sqrt((float)Dh);
    const uint64_t qp = (uint64_t)H * Dh, kp = (uint64_t)Hkv * Dh;
    const uint32_t hg = H / Hkv;
    // per (b, h, i): m, l, c
    std::vector<double> mm((uint64_t)B * H * N), ll(mm.size()), cc(mm.size());
    auto S = [&](uint32_t b, uint32_t h, uint32_t i, uint32_t j) {
        double s = 0.0;
        const uint32_t g = h / hg;
        for (uint32_t d = 0; d < Dh; ++d)
            s += (double)ld(q, (b * (uint64_t)N + i) * qp + h * Dh + d, dt) * ld(k, (b * (uint64_t)N + j) * kp + g * Dh + d, dt);
        return s * scale;
    };
    auto DP = [&](uint32_t b, uint32_t h, uint32_t i, uint32_t j) {
        double s = 0.0;
        const uint32_t g = h / hg;
        for (uint32_t d = 0; d < Dh; ++d)
            s += (double)ld(dO, (b * (uint64_t)N + i) * qp + h * Dh + d, dt) * ld(v, (b * (uint64_t)N + j) * kp + g * Dh + d, dt);
        return s;
    };
    par_for((int64_t)B * H * N, [&](int64_t x) {
        const uint32_t i = (uint32_t)(x % N), h = (uint32_t)((x / N) % H), b = (uint32_t)(x / ((int64_t)N * H));
        const uint32_t je = causal ? i + 1 : N;
        double m = -1e300;
        for (uint32_t j = 0; j < je; ++j) m = std::max(m, S(b, h, i, j));
        double l = 0.0, t = 0.0;
        for (uint32_t j = 0; j < je; ++j) {
            const double w = std::exp(S(b, h, i, j) - m);
            l += w;
            t += w * DP(b, h, i, j);
        }
        mm[x] = m;
        ll[x] = l;
        cc[x] = normalized ? t / std::max(l, 1e-20) : t;
        // dQ
        for (uint32_t d = 0; d < Dh; ++d) {
            double acc = 0.0;
            for (uint32_t j = 0; j < je; ++j) {
                const double p = std::exp(S(b, h, i, j) - m) / std::max(l, 1e-20);
                const double a = (DP(b, h, i, j) - cc[x]) * p * scale;
                acc += a * ld(k, (b * (uint64_t)N + j) * kp + (h / hg) * Dh + d, dt);
            }
            dQ[(b * (uint64_t)N + i) * qp + h * Dh + d] = st((float)acc, dt);
        }
    });
    par_for((int64_t)B * Hkv * N, [&](int64_t x) {
        const uint32_t j = (uint32_t)(x % N), g = (uint32_t)((x / N) % Hkv), b = (uint32_t)(x / ((int64_t)N * Hkv));
        std::vector<double> ak(Dh, 0.0), av(Dh, 0.0);
        for (uint32_t hh = 0; hh < hg; ++hh) {
            const uint32_t h = g * hg + hh;
            for (uint32_t i = causal ? j : 0; i < N; ++i) {
                const uint64_t si = ((uint64_t)b * H + h) * N + i;
                const double p = std::exp(S(b, h, i, j) - mm[si]) / std::max(ll[si], 1e-20);
                const double a = (DP(b, h, i, j) - cc[si]) * p * scale;
                for (uint32_t d = 0; d < Dh; ++d) {
                    ak[d] += a * ld(q, (b * (uint64_t)N + i) * qp + h * Dh + d, dt);
                    av[d] += p * ld(dO, (b * (uint64_t)N + i) * qp + h * Dh + d, dt);
                }
            }
        }
        for (uint32_t d = 0; d < Dh; ++d) {
            dK[(b * (uint64_t)N + j) * kp + g * Dh + d] = st((float)ak[d], dt);
            dV[(b * (uint64_t)N + j) * kp + g * Dh + d] = st((float)av[d], dt);
        }
    });
}

void oracle_fill_normal(uint16_t* out, uint64_t n, uint64_t seed, float mean, float stddev, int dt) {
    const uint64_t s0 = splitmix(seed);
    par_for((int64_t)n, [&](int64_t i) {
        const uint64_t z1 = splitmix(s0 ^ (2ull * i)), z2 = splitmix(s0 ^ (2ull * i + 1));
        const double u1 = ((z1 >> 11) + 1) * (1.0 / 9007199254740992.0);  // (0, 1]
        const double u2 = (z2 >> 11) * (1.0 / 9007199254740992.0);        // [0, 1)
        const double r = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
        out[i] = st((float)(mean + stddev * r), dt);
    }, 64);
}

void oracle_fill_uniform_ids(void* out, uint64_t n, uint64_t seed, uint32_t lo, uint32_t hi, uint32_t id_bytes) {
    const uint64_t s0 = splitmix(seed ^ 0x5bd1e995ull);
    const uint64_t span = hi > lo ? (uint64_t)(hi - lo) : 1;
    for (uint64_t i = 0; i < n; ++i) {
        const uint32_t v = lo + (uint32_t)(splitmix(s0 ^ i) % span);
        if (id_bytes == 2)
            ((uint16_t*)out)[i] = (uint16_t)v;
        else
            ((uint32_t*)out)[i] = v;
    }
}

}  // extern "C"
