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
