// train.cu — the training side of evk::ai on sm_100a: activation and
// normalisation backward passes, losses, optimisers, and the flash-attention
// backward pass.
//
// Reference: evk_ai.cpp:371-566, 614-660, 700-806, 839-1000, 1045-1094 (host)
// and the shaders cited per kernel.  Semantics kept from the shaders: fp32
// arithmetic with one rounding to the storage type per output element, and
// the backward passes ACCUMULATE into their gradient tensor (grad_in +=
// ...), except flash_attention_bwd, mse_loss and cross_entropy_loss, which
// overwrite.  Where a shader reduces with float atomics (cross-entropy) or a
// single workgroup (mse), the kernels here reduce in a fixed order, so
// results are reproducible run to run.
//
// These are HBM-bound elementwise / row kernels (grid-stride, rows per block);
// flash_attention_bwd is a CUDA-core kernel (one warp per query or key row,
// K/V or Q/dO rows staged per block) that keeps no N x N intermediate.
#include <float.h>

#include <algorithm>

#include "common.cuh"

namespace evkcu {
namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(uint64_t work_items, unsigned per_sm = 8) {
    DeviceState* s = state();
    const int sms = s ? s->sm_count : 148;
    uint64_t want = (work_items + kThreads - 1) / kThreads;
    const uint64_t cap = (uint64_t)sms * per_sm;
    if (want < 1) want = 1;
    return (unsigned)(want < cap ? want : cap);
}

#define GRID_STRIDE(i, n)                                                                      \
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n);                 \
         i += (uint64_t)gridDim.x * blockDim.x)

template <typename T>
__device__ __forceinline__ float ld(const T* p, uint64_t i) {
    return Elem<T>::to_f(p[i]);
}
template <typename T>
__device__ __forceinline__ void st(T* p, uint64_t i, float v) {
    p[i] = Elem<T>::from_f(v);
}

// Block-wide sum of one float per thread (blockDim.x a multiple of 32, <= 1024);
// the result is returned to every thread, summed in a fixed order.
__device__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[w] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < nw; ++i) r += sh[i];
    return r;
}
__device__ float block_max(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[w] = v;
    __syncthreads();
    float r = -FLT_MAX;
    for (int i = 0; i < nw; ++i) r = fmaxf(r, sh[i]);
    return r;
}

// ------------------------------------------------------------ elementwise --
// shaders/relu.comp: out = max(0, x)
template <typename T>
__global__ void relu_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t n) {
    GRID_STRIDE(i, n) st(out, i, fmaxf(0.0f, ld(in, i)));
}
// shaders/relu_bwd.comp: gi += x > 0 ? go : 0
template <typename T>
__global__ void relu_bwd_kernel(const T* __restrict__ go, const T* __restrict__ in, T* gi, uint64_t n) {
    GRID_STRIDE(i, n) st(gi, i, ld(gi, i) + (ld(in, i) > 0.0f ? ld(go, i) : 0.0f));
}
// shaders/gelu_bwd.comp:16-37: gi += go * d/dx[0.5 x (1 + tanh(u))],
// u = 0.79788456 (x + 0.044715 x^3)
template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ go, const T* __restrict__ in, T* gi, uint64_t n) {
    GRID_STRIDE(i, n) {
        const float x = ld(in, i);
        const float kA = 0.7978845608028654f, kB = 0.044715f;
        const float x2 = x * x;
        const float t = tanhf(kA * (x + kB * x2 * x));
        const float du = kA * (1.0f + 3.0f * kB * x2);
        const float g = 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * du;
        st(gi, i, ld(gi, i) + ld(go, i) * g);
    }
}
// shaders/sgd.comp: p = p - lr * g
template <typename T>
__global__ void sgd_kernel(T* p, const T* __restrict__ g, uint64_t n, float lr) {
    GRID_STRIDE(i, n) st(p, i, ld(p, i) - lr * ld(g, i));
}
// shaders/adam.comp: moments stored in 2-byte form: m as m / rms(v) and v as
// log2(rms(v)) + 41 (0 meaning "no history"), so small second moments
// survive fp16.  Non-finite gradients leave the element untouched; a
// non-finite stored value or update is skipped.
template <typename T>
__global__ void adam_kernel(T* p, const T* __restrict__ g, T* mbuf, T* vbuf, uint64_t n, float lr, float b1,
                            float b2, float c1inv, float c2inv, float eps) {
    const float kLogOff = 41.0f, kMinRms = 1.0e-12f;
    GRID_STRIDE(i, n) {
        const float grad = ld(g, i);
        if (isnan(grad) || isinf(grad)) continue;
        float param = ld(p, i);
        const float stored = ld(vbuf, i);
        float rms = stored > 0.0f ? exp2f(stored - kLogOff) : 0.0f;
        float m = ld(mbuf, i) * rms;
        float v = rms * rms;
        m = b1 * m + (1.0f - b1) * grad;
        v = b2 * v + (1.0f - b2) * grad * grad;
        rms = sqrtf(fmaxf(v, 0.0f));
        const float mn = m / fmaxf(rms, 1.0e-8f);
        if (!isnan(mn) && !isinf(mn)) st(mbuf, i, mn);
        const float lr2 = log2f(fmaxf(rms, kMinRms)) + kLogOff;
        if (!isnan(lr2) && !isinf(lr2)) st(vbuf, i, lr2);
        const float upd = lr * (m * c1inv) / (rms * sqrtf(c2inv) + eps);
        if (!isnan(upd) && !isinf(upd)) st(p, i, fminf(fmaxf(param - upd, -65504.0f), 65504.0f));
    }
}
// shaders/position_add.comp: out[b, t, d] = in[b, t, d] + pos[t, d]
template <typename T>
__global__ void position_add_kernel(const T* __restrict__ in, const T* __restrict__ pos, T* __restrict__ out,
                                    uint64_t n, uint32_t S, uint32_t D) {
    GRID_STRIDE(i, n) {
        const uint64_t td = i % ((uint64_t)S * D);
        st(out, i, ld(in, i) + ld(pos, td));
    }
}
// shaders/position_add_bwd.comp mode 1: gp[t, d] += sum_b go[b, t, d]
// (summed in fp32 in batch order, rounded once); mode 0 (gi += go) is
// add_kernel-shaped and done by grad_acc_kernel.
template <typename T>
__global__ void grad_acc_kernel(const T* __restrict__ go, T* gi, uint64_t n) {
    GRID_STRIDE(i, n) st(gi, i, ld(gi, i) + ld(go, i));
}
// shaders/sum_batch.comp (and position_add_bwd mode 1): out[i] += sum_b in[b * size + i]
template <typename T>
__global__ void sum_batch_kernel(const T* __restrict__ in, T* out, uint32_t batch, uint64_t size) {
    GRID_STRIDE(i, size) {
        float s = ld(out, i);
        for (uint32_t b = 0; b < batch; ++b) s += ld(in, (uint64_t)b * size + i);
        st(out, i, s);
    }
}
// shaders/rope_bwd.comp: the transpose rotation of rope (angle t * base^(-2p/D),
// same expression as the forward kernel), accumulated into gi.
template <typename T>
__global__ void rope_bwd_kernel(const T* __restrict__ go, T* gi, uint64_t pairs, uint32_t S, uint32_t D,
                                float base) {
    const uint32_t half = D / 2;
    GRID_STRIDE(w, pairs) {
        const uint32_t p = (uint32_t)(w % half);
        const uint64_t row = w / half;
        const float t = (float)(uint32_t)(row % S);
        const float inv_freq = powf(base, -2.0f * (float)p / (float)D);
        float sn, cs;
        sincosf(t * inv_freq, &sn, &cs);
        const uint64_t i0 = row * D + 2 * p;
        const float g0 = ld(go, i0), g1 = ld(go, i0 + 1);
        st(gi, i0, ld(gi, i0) + g0 * cs + g1 * sn);
        st(gi, i0 + 1, ld(gi, i0 + 1) - g0 * sn + g1 * cs);
    }
}
// shaders/embed_bwd.comp: gE[idx[i], d] += go[i, d], indices in order with a
// rounding after every addition (as the shader), one thread per column d.
template <typename T, typename I>
__global__ void embed_bwd_kernel(const T* __restrict__ go, const I* __restrict__ idx, T* gE, uint32_t vocab,
                                 uint32_t D, uint32_t n_idx) {
    for (uint32_t d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x) {
        for (uint32_t i = 0; i < n_idx; ++i) {
            const uint32_t tok = (uint32_t)idx[i];
            if (tok >= vocab) continue;
            const uint64_t o = (uint64_t)tok * D + d;
            st(gE, o, ld(gE, o) + ld(go, (uint64_t)i * D + d));
        }
    }
}

// ------------------------------------------------------------ row kernels --
// shaders/softmax_bwd.comp: gi += p * (g - sum(g * p)) * scale, one block per row.
template <typename T>
__global__ void softmax_bwd_kernel(const T* __restrict__ p, const T* __restrict__ g, T* gi, uint32_t rows,
                                   uint32_t L, float scale) {
    __shared__ float sh[32];
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint64_t base = (uint64_t)r * L;
        float d = 0.0f;
        for (uint32_t j = threadIdx.x; j < L; j += blockDim.x) d += ld(p, base + j) * ld(g, base + j);
        const float dot = block_sum(d, sh);
        for (uint32_t j = threadIdx.x; j < L; j += blockDim.x)
            st(gi, base + j, ld(gi, base + j) + ld(p, base + j) * (ld(g, base + j) - dot) * scale);
        __syncthreads();
    }
}
// shaders/rms_norm_bwd.comp:21-74: with x clamped to +-65504, rms =
// sqrt(mean(x^2) + eps), y = x / rms: gi += g / rms - x / rms^2 * dot(g, y) / D.
template <typename T>
__global__ void rms_norm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ g, T* gi, uint32_t rows,
                                    uint32_t D, float eps) {
    __shared__ float sh[32];
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint64_t base = (uint64_t)r * D;
        float ss = 0.0f;
        for (uint32_t j = threadIdx.x; j < D; j += blockDim.x) {
            const float v = fminf(fmaxf(ld(x, base + j), -65504.0f), 65504.0f);
            ss += v * v;
        }
        const float sum_sq = block_sum(ss, sh);
        const float inv = 1.0f / sqrtf(sum_sq / (float)D + eps);
        float dp = 0.0f;
        for (uint32_t j = threadIdx.x; j < D; j += blockDim.x) {
            const float v = fminf(fmaxf(ld(x, base + j), -65504.0f), 65504.0f);
            dp += ld(g, base + j) * (v * inv);
        }
        const float sc = block_sum(dp, sh) / (float)D;
        for (uint32_t j = threadIdx.x; j < D; j += blockDim.x) {
            const float v = fminf(fmaxf(ld(x, base + j), -65504.0f), 65504.0f);
            st(gi, base + j, ld(gi, base + j) + ld(g, base + j) * inv - v * inv * inv * sc);
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ losses --
// shaders/mse_loss.comp: grad = 2 (pred - target) / N per element; the loss
// mean((pred - target)^2) is reduced as per-block partials (fixed order) and
// then one block sums the partials in block order.
template <typename T>
__global__ void mse_partial_kernel(const T* __restrict__ pred, const T* __restrict__ tgt, T* __restrict__ grad,
                                   float* partial, uint64_t n) {
    __shared__ float sh[32];
    const float gs = 2.0f / (float)n;
    float acc = 0.0f;
    GRID_STRIDE(i, n) {
        const float d = ld(pred, i) - ld(tgt, i);
        acc += d * d;
        st(grad, i, gs * d);
    }
    const float s = block_sum(acc, sh);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
}
template <typename T>
__global__ void mse_final_kernel(const float* partial, uint32_t nparts, T* result, uint64_t n) {
    __shared__ float sh[32];
    float a = 0.0f;
    for (uint32_t i = threadIdx.x; i < nparts; i += blockDim.x) a += partial[i];
    const float s = block_sum(a, sh);
    if (threadIdx.x == 0) st(result, 0, s / (float)n);
}

// shaders/cross_entropy_count.comp: number of valid targets (0 < t < V).
template <typename I>
__global__ void ce_count_kernel(const I* __restrict__ tgt, uint32_t rows, uint32_t V, float* count) {
    __shared__ float sh[32];
    float c = 0.0f;
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) {
        const uint32_t t = (uint32_t)tgt[r];
        c += (t != 0u && t < V) ? 1.0f : 0.0f;
    }
    const float s = block_sum(c, sh);
    if (threadIdx.x == 0) *count = s;
}
// shaders/cross_entropy.comp: per row, with logits clamped to +-65000:
//   grad = softmax(logits) / count, minus 1 / count at the target;
//   loss_row = (max + ln(sum exp(l - max)) - l[target]) / count;
// rows whose target is 0 (the ignore token) or out of range get zero
// gradient and no loss.
template <typename T, typename I>
__global__ void ce_row_kernel(const T* __restrict__ logits, const I* __restrict__ tgt, T* __restrict__ grad,
                              const float* count, float* row_loss, uint32_t rows, uint32_t V) {
    __shared__ float sh[32];
    const float kL2E = 1.4426950408889634f;
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint64_t base = (uint64_t)r * V;
        const uint32_t t = (uint32_t)tgt[r];
        const float cnt = *count;
        const bool valid = t != 0u && t < V && cnt > 0.0f;
        if (!valid) {
            for (uint32_t j = threadIdx.x; j < V; j += blockDim.x) st(grad, base + j, 0.0f);
            if (threadIdx.x == 0) row_loss[r] = 0.0f;
            continue;
        }
        const float inv_valid = 1.0f / cnt;
        float mx = -FLT_MAX;
        for (uint32_t j = threadIdx.x; j < V; j += blockDim.x)
            mx = fmaxf(mx, fminf(fmaxf(ld(logits, base + j), -65000.0f), 65000.0f));
        mx = block_max(mx, sh);
        float se = 0.0f;
        for (uint32_t j = threadIdx.x; j < V; j += blockDim.x)
            se += exp2f((fminf(fmaxf(ld(logits, base + j), -65000.0f), 65000.0f) - mx) * kL2E);
        const float denom = fmaxf(block_sum(se, sh), 1e-20f);
        const float inv_denom = 1.0f / denom;
        for (uint32_t j = threadIdx.x; j < V; j += blockDim.x) {
            const float l = fminf(fmaxf(ld(logits, base + j), -65000.0f), 65000.0f);
            float gv = exp2f((l - mx) * kL2E) * inv_denom * inv_valid;
            if (j == t) {
                gv -= inv_valid;
                row_loss[r] = (mx + logf(denom) - l) * inv_valid;
            }
            st(grad, base + j, gv);
        }
        __syncthreads();
    }
}
// shaders/cross_entropy_scale.comp: the mean loss (0 without valid rows or
// when not finite), rows summed in order.
template <typename T>
__global__ void ce_final_kernel(const float* row_loss, const float* count, uint32_t rows, T* result) {
    __shared__ float sh[32];
    float a = 0.0f;
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) a += row_loss[r];
    float loss = block_sum(a, sh);
    if (!(*count > 0.0f) || isnan(loss) || isinf(loss)) loss = 0.0f;
    if (threadIdx.x == 0) st(result, 0, loss);
}

// ------------------------------------------------- flash attention backward --
// shaders/flash_attention_bwd.comp, restated without the N x N tiles.
// Per query row i of head h (K/V head g = h / (H / Hkv)), with s_ij = q_i . k_j,
// dp_ij = dO_i . v_j:
//   pass 1: m_i = max_j s_ij * scale, l_i = sum_j e^(s_ij scale - m_i),
//           t_i = sum_j e^(s_ij scale - m_i) dp_ij;
//   p_ij = e^(s_ij scale - m_i) / l_i,  a_ij = (dp_ij - c_i) p_ij scale,
//   dQ_i = sum_j a_ij k_j,  dK_j = sum_{h in g, i} a_ij q_i,  dV_j = sum_{h in g, i} p_ij dO_i.
// c_i is t_i in the reference's shader (its `tRow`, not divided by l_i);
// with EVKCU_ATTN_BWD_NORMALIZED it is t_i / l_i = sum_j p_ij dp_ij, the
// exact softmax gradient.  O is not read (the shader recomputes instead).
// One warp per row; a lane holds Dh / 32 (<= 8) elements.

constexpr int kBwdWarps = 8;  // rows per block
constexpr int kBwdTile = 32;  // partner rows staged in shared memory per step

template <typename T>
__device__ __forceinline__ void load_row(const T* src, uint32_t Dh, float (&r)[8]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t d = lane + 32u * e;
        r[e] = d < Dh ? Elem<T>::to_f(src[d]) : 0.0f;
    }
}
__device__ __forceinline__ float warp_dot(const float (&a)[8], const float* b, uint32_t Dh) {
    const int lane = threadIdx.x & 31;
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t d = lane + 32u * e;
        if (d < Dh) s += a[e] * b[d];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// Pass 1 (stats) and the dQ pass share the walk over the keys of one query row.
template <typename T, bool DQ>
__global__ void __launch_bounds__(kBwdWarps * 32) attn_bwd_query_kernel(
    const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V, const T* __restrict__ dO,
    T* __restrict__ dQ, float* __restrict__ stats, uint32_t B, uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh,
    float scale, int causal, int normalized) {
    extern __shared__ float sm[];
    float* sK = sm;                              // [kBwdTile][Dh]
    float* sV = sm + (size_t)kBwdTile * Dh;      // [kBwdTile][Dh]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rows_per_bh = (N + kBwdWarps - 1) / kBwdWarps;
    const uint64_t blk = blockIdx.x;
    const uint32_t bh = (uint32_t)(blk / rows_per_bh);
    const uint32_t b = bh / H, h = bh % H, g = h / (H / Hkv);
    const uint32_t i = (uint32_t)(blk % rows_per_bh) * kBwdWarps + warp;
    const bool live = i < N;
    const uint64_t qo = ((uint64_t)b * N + (live ? i : 0)) * H * Dh + (uint64_t)h * Dh;
    float q[8], go[8], acc[8];
    load_row(Q + qo, Dh, q);
    load_row(dO + qo, Dh, go);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    float m = -INFINITY, l = 0.0f, t = 0.0f, c = 0.0f;
    const uint64_t so = ((uint64_t)bh * N + (live ? i : 0)) * 3;
    if (DQ && live) {
        m = stats[so];
        l = stats[so + 1];
        c = normalized ? stats[so + 2] / fmaxf(l, 1e-20f) : stats[so + 2];
    }
    const float inv_l = 1.0f / fmaxf(l, 1e-20f);
    // keys a block of rows can see
    const uint32_t i_last = min(N, (uint32_t)(blk % rows_per_bh) * kBwdWarps + kBwdWarps) - 1;
    const uint32_t jend = causal ? i_last + 1 : N;
    for (uint32_t j0 = 0; j0 < jend; j0 += kBwdTile) {
        __syncthreads();
        for (uint32_t x = threadIdx.x; x < kBwdTile * Dh; x += blockDim.x) {
            const uint32_t jj = x / Dh, d = x % Dh;
            const uint32_t j = j0 + jj;
            const uint64_t ko = ((uint64_t)b * N + j) * Hkv * Dh + (uint64_t)g * Dh + d;
            sK[x] = j < N ? Elem<T>::to_f(K[ko]) : 0.0f;
            sV[x] = j < N ? Elem<T>::to_f(V[ko]) : 0.0f;
        }
        __syncthreads();
        if (!live) continue;
        const uint32_t jn = min(kBwdTile, (causal ? i + 1 : N) > j0 ? (causal ? i + 1 : N) - j0 : 0u);
        for (uint32_t jj = 0; jj < jn; ++jj) {
            const float s = warp_dot(q, sK + (size_t)jj * Dh, Dh) * scale;
            const float dp = warp_dot(go, sV + (size_t)jj * Dh, Dh);
            if (!DQ) {
                const float mn = fmaxf(m, s);
                const float a = expf(m - mn), w = expf(s - mn);
                l = l * a + w;
                t = t * a + w * dp;
                m = mn;
            } else {
                const float p = expf(s - m) * inv_l;
                const float a = (dp - c) * p * scale;
                const float* kr = sK + (size_t)jj * Dh;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t d = lane + 32u * e;
                    if (d < Dh) acc[e] += a * kr[d];
                }
            }
        }
    }
    if (!live) return;
    if (!DQ) {
        if (lane == 0) {
            stats[so] = m;
            stats[so + 1] = l;
            stats[so + 2] = t;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t d = lane + 32u * e;
            if (d < Dh) dQ[qo + d] = Elem<T>::from_f(acc[e]);
        }
    }
}

// dK / dV: one warp per key row j of K/V head g; walks every query row of every
// head in the group (queries i >= j when causal).
template <typename T>
__global__ void __launch_bounds__(kBwdWarps * 32) attn_bwd_key_kernel(
    const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V, const T* __restrict__ dO,
    T* __restrict__ dK, T* __restrict__ dV, const float* __restrict__ stats, uint32_t B, uint32_t N, uint32_t H,
    uint32_t Hkv, uint32_t Dh, float scale, int causal, int normalized) {
    extern __shared__ float sm[];
    float* sQ = sm;                          // [kBwdTile][Dh]
    float* sO = sm + (size_t)kBwdTile * Dh;  // [kBwdTile][Dh] (dO rows)
    float* sS = sm + (size_t)2 * kBwdTile * Dh;  // [kBwdTile][3] stats
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rows_per_bg = (N + kBwdWarps - 1) / kBwdWarps;
    const uint64_t blk = blockIdx.x;
    const uint32_t bg = (uint32_t)(blk / rows_per_bg);
    const uint32_t b = bg / Hkv, g = bg % Hkv;
    const uint32_t j_first = (uint32_t)(blk % rows_per_bg) * kBwdWarps;
    const uint32_t j = j_first + warp;
    const bool live = j < N;
    const uint64_t ko = ((uint64_t)b * N + (live ? j : 0)) * Hkv * Dh + (uint64_t)g * Dh;
    float k[8], v[8], ak[8], av[8];
    load_row(K + ko, Dh, k);
    load_row(V + ko, Dh, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ak[e] = av[e] = 0.0f;
    const uint32_t hg = H / Hkv;
    const uint32_t i_begin = causal ? j_first : 0;
    for (uint32_t hh = 0; hh < hg; ++hh) {
        const uint32_t h = g * hg + hh;
        for (uint32_t i0 = i_begin; i0 < N; i0 += kBwdTile) {
            __syncthreads();
            for (uint32_t x = threadIdx.x; x < kBwdTile * Dh; x += blockDim.x) {
                const uint32_t ii = x / Dh, d = x % Dh;
                const uint32_t i = i0 + ii;
                const uint64_t qo = ((uint64_t)b * N + i) * H * Dh + (uint64_t)h * Dh + d;
                sQ[x] = i < N ? Elem<T>::to_f(Q[qo]) : 0.0f;
                sO[x] = i < N ? Elem<T>::to_f(dO[qo]) : 0.0f;
            }
            for (uint32_t x = threadIdx.x; x < kBwdTile; x += blockDim.x) {
                const uint32_t i = i0 + x;
                const uint64_t so = ((uint64_t)(b * H + h) * N + (i < N ? i : 0)) * 3;
                const float l = stats[so + 1];
                sS[3 * x] = stats[so];
                sS[3 * x + 1] = 1.0f / fmaxf(l, 1e-20f);
                sS[3 * x + 2] = normalized ? stats[so + 2] / fmaxf(l, 1e-20f) : stats[so + 2];
            }
            __syncthreads();
            if (!live) continue;
            const uint32_t ib = causal ? max(i0, j) : i0;
            const uint32_t ie = min(N, i0 + kBwdTile);
            for (uint32_t i = ib; i < ie; ++i) {
                const uint32_t ii = i - i0;
                const float* qr = sQ + (size_t)ii * Dh;
                const float* orow = sO + (size_t)ii * Dh;
                const float s = warp_dot(k, qr, Dh) * scale;
                const float dp = warp_dot(v, orow, Dh);
                const float p = expf(s - sS[3 * ii]) * sS[3 * ii + 1];
                const float a = (dp - sS[3 * ii + 2]) * p * scale;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t d = lane + 32u * e;
                    if (d < Dh) {
                        ak[e] += a * qr[d];
                        av[e] += p * orow[d];
                    }
                }
            }
        }
    }
    if (!live) return;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t d = lane + 32u * e;
        if (d < Dh) {
            dK[ko + d] = Elem<T>::from_f(ak[e]);
            dV[ko + d] = Elem<T>::from_f(av[e]);
        }
    }
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

#define TRAIN_DTYPE_CHECK(dtype, name) \
    EVKCU_CHECK_ARG((dtype) == EVKCU_F16 || (dtype) == EVKCU_BF16, EVKCU_BAD_ARG, name ": unknown dtype")

extern "C" int evkcu_relu(const void* in, void* out, uint64_t n, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_relu");
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_relu: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        relu_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((const T*)in, (T*)out, n);
        return after_launch("evkcu_relu");
    });
}

extern "C" int evkcu_relu_backward(const void* grad_out, const void* in, void* grad_in, uint64_t n, int dtype,
                                   void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_relu_backward");
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(grad_out && in && grad_in, EVKCU_BAD_ARG, "evkcu_relu_backward: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        relu_bwd_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((const T*)grad_out, (const T*)in,
                                                                            (T*)grad_in, n);
        return after_launch("evkcu_relu_backward");
    });
}

extern "C" int evkcu_gelu_backward(const void* grad_out, const void* in, void* grad_in, uint64_t n, int dtype,
                                   void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_gelu_backward");
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(grad_out && in && grad_in, EVKCU_BAD_ARG, "evkcu_gelu_backward: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        gelu_bwd_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((const T*)grad_out, (const T*)in,
                                                                            (T*)grad_in, n);
        return after_launch("evkcu_gelu_backward");
    });
}

extern "C" int evkcu_softmax_backward(const void* probs, const void* grad_out, void* grad_in, uint32_t rows,
                                      uint32_t L, float scale, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_softmax_backward");
    if (rows == 0 || L == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(probs && grad_out && grad_in, EVKCU_BAD_ARG, "evkcu_softmax_backward: null pointer");
    const unsigned grid = std::min<uint32_t>(rows, (uint32_t)state()->sm_count * 8);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        softmax_bwd_kernel<T><<<grid, kThreads, 0, as_stream(stream)>>>((const T*)probs, (const T*)grad_out,
                                                                        (T*)grad_in, rows, L, scale);
        return after_launch("evkcu_softmax_backward");
    });
}

extern "C" int evkcu_rms_norm_backward(const void* in, const void* grad_out, void* grad_in, uint32_t rows,
                                       uint32_t D, float eps, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_rms_norm_backward");
    if (rows == 0 || D == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && grad_out && grad_in, EVKCU_BAD_ARG, "evkcu_rms_norm_backward: null pointer");
    const unsigned grid = std::min<uint32_t>(rows, (uint32_t)state()->sm_count * 8);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        rms_norm_bwd_kernel<T><<<grid, kThreads, 0, as_stream(stream)>>>((const T*)in, (const T*)grad_out,
                                                                         (T*)grad_in, rows, D, eps);
        return after_launch("evkcu_rms_norm_backward");
    });
}

extern "C" int evkcu_rope_backward(const void* grad_out, void* grad_in, uint32_t batch, uint32_t seq_len,
                                   uint32_t dim, float base, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_rope_backward");
    EVKCU_CHECK_ARG(dim % 2 == 0, EVKCU_BAD_SHAPE, "evkcu_rope_backward: dim must be even");
    const uint64_t pairs = (uint64_t)batch * seq_len * (dim / 2);
    if (pairs == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(grad_out && grad_in, EVKCU_BAD_ARG, "evkcu_rope_backward: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        rope_bwd_kernel<T><<<grid_for(pairs), kThreads, 0, as_stream(stream)>>>((const T*)grad_out, (T*)grad_in,
                                                                                pairs, seq_len, dim, base);
        return after_launch("evkcu_rope_backward");
    });
}

extern "C" int evkcu_embed_backward(const void* grad_out, const void* idx, void* grad_E, uint32_t vocab,
                                    uint32_t dim, uint32_t n_idx, uint32_t idx_bytes, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_embed_backward");
    EVKCU_CHECK_ARG(idx_bytes == 2 || idx_bytes == 4, EVKCU_BAD_ARG, "evkcu_embed_backward: idx_bytes must be 2 or 4");
    if (n_idx == 0 || dim == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(grad_out && idx && grad_E, EVKCU_BAD_ARG, "evkcu_embed_backward: null pointer");
    const unsigned grid = (dim + 127) / 128;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (idx_bytes == 2)
            embed_bwd_kernel<T, uint16_t><<<grid, 128, 0, as_stream(stream)>>>((const T*)grad_out,
                                                                               (const uint16_t*)idx, (T*)grad_E,
                                                                               vocab, dim, n_idx);
        else
            embed_bwd_kernel<T, uint32_t><<<grid, 128, 0, as_stream(stream)>>>((const T*)grad_out,
                                                                               (const uint32_t*)idx, (T*)grad_E,
                                                                               vocab, dim, n_idx);
        return after_launch("evkcu_embed_backward");
    });
}

extern "C" int evkcu_position_add(const void* in, const void* pos, void* out, uint32_t batch, uint32_t seq_len,
                                  uint32_t dim, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_position_add");
    const uint64_t n = (uint64_t)batch * seq_len * dim;
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && pos && out, EVKCU_BAD_ARG, "evkcu_position_add: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        position_add_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((const T*)in, (const T*)pos,
                                                                                (T*)out, n, seq_len, dim);
        return after_launch("evkcu_position_add");
    });
}

extern "C" int evkcu_position_add_backward(const void* grad_out, void* grad_in, void* grad_pos, uint32_t batch,
                                           uint32_t seq_len, uint32_t dim, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_position_add_backward");
    const uint64_t n = (uint64_t)batch * seq_len * dim, np = (uint64_t)seq_len * dim;
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(grad_out && grad_in && grad_pos, EVKCU_BAD_ARG, "evkcu_position_add_backward: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        grad_acc_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((const T*)grad_out, (T*)grad_in, n);
        int r = after_launch("evkcu_position_add_backward(input)");
        if (r) return r;
        sum_batch_kernel<T><<<grid_for(np), kThreads, 0, as_stream(stream)>>>((const T*)grad_out, (T*)grad_pos,
                                                                               batch, np);
        return after_launch("evkcu_position_add_backward(position)");
    });
}

extern "C" int evkcu_sum_batch(const void* in, void* out, uint32_t batch, uint64_t size, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_sum_batch");
    if (size == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_sum_batch: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        sum_batch_kernel<T><<<grid_for(size), kThreads, 0, as_stream(stream)>>>((const T*)in, (T*)out, batch, size);
        return after_launch("evkcu_sum_batch");
    });
}

extern "C" int evkcu_sgd(void* param, const void* grad, uint64_t n, float lr, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_sgd");
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(param && grad, EVKCU_BAD_ARG, "evkcu_sgd: null pointer");
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        sgd_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((T*)param, (const T*)grad, n, lr);
        return after_launch("evkcu_sgd");
    });
}

extern "C" int evkcu_adam(void* param, const void* grad, void* m, void* v, uint64_t n, uint32_t step, float lr,
                          float beta1, float beta2, float eps, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_adam");
    EVKCU_CHECK_ARG(step >= 1, EVKCU_BAD_ARG, "evkcu_adam: step counts from 1");
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(param && grad && m && v, EVKCU_BAD_ARG, "evkcu_adam: null pointer");
    // Bias corrections on the host, as evk_ai.cpp:545-548 does.
    const float c1 = 1.0f / (1.0f - powf(beta1, (float)step));
    const float c2 = 1.0f / (1.0f - powf(beta2, (float)step));
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        adam_kernel<T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>((T*)param, (const T*)grad, (T*)m, (T*)v, n,
                                                                        lr, beta1, beta2, c1, c2, eps);
        return after_launch("evkcu_adam");
    });
}

extern "C" int evkcu_mse_loss(const void* pred, const void* target, void* grad, void* result, uint64_t n, int dtype,
                              void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_mse_loss");
    EVKCU_CHECK_ARG(n > 0, EVKCU_BAD_SHAPE, "evkcu_mse_loss: empty input");
    EVKCU_CHECK_ARG(pred && target && grad && result, EVKCU_BAD_ARG, "evkcu_mse_loss: null pointer");
    const unsigned grid = grid_for(n, 2);
    float* part = (float*)workspace(WS_TRAIN, kTicketBytes + (size_t)grid * sizeof(float));
    EVKCU_CHECK_ARG(part, EVKCU_CUDA_ERROR, "evkcu_mse_loss: workspace");
    part = (float*)((char*)part + kTicketBytes);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        mse_partial_kernel<T><<<grid, kThreads, 0, as_stream(stream)>>>((const T*)pred, (const T*)target, (T*)grad,
                                                                        part, n);
        int r = after_launch("evkcu_mse_loss(partials)");
        if (r) return r;
        mse_final_kernel<T><<<1, kThreads, 0, as_stream(stream)>>>(part, grid, (T*)result, n);
        return after_launch("evkcu_mse_loss(mean)");
    });
}

extern "C" int evkcu_cross_entropy_loss(const void* logits, const void* targets, void* grad, void* result,
                                        uint32_t rows, uint32_t V, uint32_t target_bytes, int dtype, void* stream) {
    TRAIN_DTYPE_CHECK(dtype, "evkcu_cross_entropy_loss");
    EVKCU_CHECK_ARG(target_bytes == 2 || target_bytes == 4, EVKCU_BAD_ARG,
                    "evkcu_cross_entropy_loss: target_bytes must be 2 or 4");
    EVKCU_CHECK_ARG(rows > 0 && V > 0, EVKCU_BAD_SHAPE, "evkcu_cross_entropy_loss: empty input");
    EVKCU_CHECK_ARG(logits && targets && grad && result, EVKCU_BAD_ARG, "evkcu_cross_entropy_loss: null pointer");
    float* ws = (float*)workspace(WS_TRAIN, kTicketBytes + ((size_t)rows + 4) * sizeof(float));
    EVKCU_CHECK_ARG(ws, EVKCU_CUDA_ERROR, "evkcu_cross_entropy_loss: workspace");
    ws = (float*)((char*)ws + kTicketBytes);
    float* count = ws;
    float* row_loss = ws + 4;
    cudaStream_t st = as_stream(stream);
    const unsigned grid = std::min<uint32_t>(rows, (uint32_t)state()->sm_count * 8);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (target_bytes == 2) {
            ce_count_kernel<uint16_t><<<1, 1024, 0, st>>>((const uint16_t*)targets, rows, V, count);
            int r = after_launch("evkcu_cross_entropy_loss(count)");
            if (r) return r;
            ce_row_kernel<T, uint16_t><<<grid, kThreads, 0, st>>>((const T*)logits, (const uint16_t*)targets,
                                                                 (T*)grad, count, row_loss, rows, V);
        } else {
            ce_count_kernel<uint32_t><<<1, 1024, 0, st>>>((const uint32_t*)targets, rows, V, count);
            int r = after_launch("evkcu_cross_entropy_loss(count)");
            if (r) return r;
            ce_row_kernel<T, uint32_t><<<grid, kThreads, 0, st>>>((const T*)logits, (const uint32_t*)targets,
                                                                 (T*)grad, count, row_loss, rows, V);
        }
        int r = after_launch("evkcu_cross_entropy_loss(rows)");
        if (r) return r;
        ce_final_kernel<T><<<1, 1024, 0, st>>>(row_loss, count, rows, (T*)result);
        return after_launch("evkcu_cross_entropy_loss(mean)");
    });
}

extern "C" int evkcu_flash_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                         void* dQ, void* dK, void* dV, uint32_t B, uint32_t N, uint32_t H,
                                         uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype,
                                         void* stream) {
    (void)o;  // the reference recomputes the forward instead of reading O
    TRAIN_DTYPE_CHECK(dtype, "evkcu_flash_attention_bwd");
    if (B == 0 || N == 0 || H == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(q && k && v && dO && dQ && dK && dV, EVKCU_BAD_ARG, "evkcu_flash_attention_bwd: null pointer");
    EVKCU_CHECK_ARG(Hkv >= 1 && H % Hkv == 0, EVKCU_BAD_SHAPE, "evkcu_flash_attention_bwd: H must be a multiple of Hkv");
    EVKCU_CHECK_ARG(Dh >= 1 && Dh <= 256, EVKCU_BAD_SHAPE, "evkcu_flash_attention_bwd: Dh must be in [1, 256]");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)Dh);
    const int causal = (flags & EVKCU_ATTN_CAUSAL) ? 1 : 0;
    const int normalized = (flags & EVKCU_ATTN_BWD_NORMALIZED) ? 1 : 0;
    const size_t stat_bytes = (size_t)B * H * N * 3 * sizeof(float);
    char* ws = (char*)workspace(WS_TRAIN, kTicketBytes + stat_bytes);
    EVKCU_CHECK_ARG(ws, EVKCU_CUDA_ERROR, "evkcu_flash_attention_bwd: workspace");
    float* stats = (float*)(ws + kTicketBytes);
    cudaStream_t st = as_stream(stream);
    const uint32_t rpb = (N + kBwdWarps - 1) / kBwdWarps;
    const uint64_t qblocks = (uint64_t)B * H * rpb, kblocks = (uint64_t)B * Hkv * rpb;
    EVKCU_CHECK_ARG(qblocks <= 0x7fffffffu, EVKCU_BAD_SHAPE, "evkcu_flash_attention_bwd: grid too large");
    const size_t smq = (size_t)2 * kBwdTile * Dh * sizeof(float);
    const size_t smk = smq + (size_t)3 * kBwdTile * sizeof(float);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        static bool attr = false;
        if (!attr) {
            EVKCU_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_query_kernel<T, false>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 80 * 1024));
            EVKCU_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_query_kernel<T, true>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 80 * 1024));
            EVKCU_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_key_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                80 * 1024));
            attr = true;
        }
        const T *Q = (const T*)q, *K = (const T*)k, *Vv = (const T*)v, *GO = (const T*)dO;
        attn_bwd_query_kernel<T, false><<<(unsigned)qblocks, kBwdWarps * 32, smq, st>>>(
            Q, K, Vv, GO, nullptr, stats, B, N, H, Hkv, Dh, scale, causal, normalized);
        int r = after_launch("evkcu_flash_attention_bwd(stats)");
        if (r) return r;
        attn_bwd_query_kernel<T, true><<<(unsigned)qblocks, kBwdWarps * 32, smq, st>>>(
            Q, K, Vv, GO, (T*)dQ, stats, B, N, H, Hkv, Dh, scale, causal, normalized);
        if ((r = after_launch("evkcu_flash_attention_bwd(dQ)"))) return r;
        attn_bwd_key_kernel<T><<<(unsigned)kblocks, kBwdWarps * 32, smk, st>>>(
            Q, K, Vv, GO, (T*)dK, (T*)dV, stats, B, N, H, Hkv, Dh, scale, causal, normalized);
        return after_launch("evkcu_flash_attention_bwd(dK, dV)");
    });
}
