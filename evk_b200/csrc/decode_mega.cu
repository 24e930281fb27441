// decode_mega.cu — one decode step of the LLM driver as ONE persistent kernel.
//
// The step is the same computation as the per-op chain of llm.cu (embed ->
// per layer [RMSNorm -> QKV projection with RoPE into the KV cache ->
// single-query attention -> Wo + residual -> RMSNorm -> W1 + GELU -> W2 +
// residual] -> RMSNorm -> LM head -> greedy ids), for small models where that
// chain is bound by per-kernel fixed costs rather than by HBM: at the C3 shape
// (6 layers, d_model 512, batch 1) about 45 kernels move 70 MB per token.
// Reference: example/main_llm.cpp:622-654 (the decode loop),
// CausalAttentionBlock::forward :528-546.
//
// Structure: a cooperative grid of one CTA per SM (all resident, checked by
// the cooperative launch).  Phases are separated by a grid barrier (a counter
// and a generation word in global memory; every wait is bounded and gives up
// with an error status).  Within a phase, work items are strided over the
// CTAs:
//   GEMV phases  item = 256 output columns x a range of K rows; each lane
//                owns 8 columns (one 16-byte load per weight row), the eight
//                warps split the rows, the CTA reduces in shared memory.  With
//                several K ranges per column chunk the partials go to scratch
//                and the last CTA of the chunk (ticket) sums them in range
//                order, so results are deterministic, then applies the
//                epilogue (RoPE + cache write, GELU, or residual add).
//   attention    item = (sequence, head, range of 32 cached positions): one
//                warp per position stream, online softmax, partial (m, l, o)
//                per item; the last item of a (sequence, head) merges in range
//                order.
//   LM head      item = 64 vocabulary rows (tied embedding) or 256 columns
//                (separate head); each CTA keeps its best 64-bit greedy key per
//                sequence (greedy_key.cuh: the reference's tie rule), CTA 0
//                merges them after the last barrier.
// Every activation another CTA wrote is read with L2 loads (__ldcg): L1 is not
// coherent across SMs.  Rounding to the storage type happens where the per-op
// chain stores a tensor (normalised x, q / k / v, attention output, h1, x,
// logits), so the step matches it up to fp32 summation order.
#include <float.h>

#include <algorithm>

#include "decode_mega.cuh"
#include "greedy_key.cuh"

namespace evkcu {

namespace {

constexpr int kMT = 256;              // threads per CTA
constexpr int kMW = kMT / 32;         // warps per CTA
constexpr int kMCols = 256;           // output columns per GEMV item (8 per lane)
constexpr int kMaxB = 4;              // sequences per step
constexpr uint32_t kMegaTimeout = 0x501;

// Per-matrix split of the K rows: kc rows per item, ks items per chunk.
struct MegaSplit {
    uint32_t kc, ks;
};

struct MegaArgs {
    uint32_t B, D, H, Hkv, Dh, F, V, layers, max_seq, tied;
    float eps, scale_log2;
    const void* emb;
    const void* lm_head;
    const MegaLayer* layer;  // [layers], device memory
    void *x, *q, *attn, *h1;  // activations
    void* logits;             // optional [B, V]
    const float2* rope_cs;    // [max_seq, Dh / 2] (cos, sin)
    uint32_t *d_pos, *d_len;  // d_pos[2]: decode-step counter
    const uint32_t* ids_in;
    uint32_t* ids_out;
    float* partial;                // split-K / attention partials
    unsigned int* tickets;         // per chunk / per (b, h); left at zero
    unsigned long long* keys;      // [grid, B]
    unsigned int* bar;             // [0] arrivals, [1] generation, [2] abort
    unsigned int* err;
    MegaSplit s_qkv, s_wo, s_w1, s_w2;
    uint32_t att_tickets;          // ticket offset of the attention merge
};

// ------------------------------------------------------------ grid barrier --
// All CTAs arrive; the last one resets the counter and bumps the generation.
// Waits are bounded (about 2 s of clock) and honour the abort word, so a CTA
// that gives up makes every other one leave at its next barrier.
__device__ bool grid_sync(const MegaArgs& a) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned int* gen = a.bar + 1;
        volatile unsigned int* abort = a.bar + 2;
        const unsigned int g0 = *gen;
        __threadfence();
        const unsigned int arrived = atomicAdd(a.bar, 1u);
        int ok = 1;
        if (arrived == gridDim.x - 1) {
            atomicExch(a.bar, 0u);
            __threadfence();
            atomicAdd(a.bar + 1, 1u);
        } else {
            const long long t0 = clock64();
            while (*gen == g0) {
                if (*abort || clock64() - t0 > kSpinLimitCycles) {
                    atomicExch(a.bar + 2, 1u);
                    atomicCAS(a.err, 0u, kMegaTimeout);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
        s_ok = ok && !*abort;
    }
    __syncthreads();
    return s_ok != 0;
}

template <typename T>
__device__ __forceinline__ float ldg_f(const T* p) {
    return Elem<T>::to_f(__ldcg(p));
}

// xs[b][k] (fp32) = the B rows of `src` ([B, K], storage type), optionally
// RMS-normalised (shaders/rms_norm.comp:21-48) and rounded to the storage type
// as the per-op chain stores it.
template <typename T>
__device__ void load_rows(const T* src, uint32_t B, uint32_t K, bool norm, float eps, float* xs) {
    __shared__ float s_red[kMaxB][kMW];
    for (uint32_t b = 0; b < B; ++b) {
        float ss = 0.0f;
        for (uint32_t k = threadIdx.x; k < K; k += kMT) {
            const float v = ldg_f(src + (uint64_t)b * K + k);
            xs[b * K + k] = v;
            const float c = fminf(fmaxf(v, -65504.0f), 65504.0f);
            ss += c * c;
        }
        if (!norm) continue;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) s_red[b][threadIdx.x >> 5] = ss;
    }
    __syncthreads();
    if (!norm) return;
    for (uint32_t b = 0; b < B; ++b) {
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kMW; ++w) tot += s_red[b][w];
        const float inv = rsqrtf(tot / (float)K + eps);
        for (uint32_t k = threadIdx.x; k < K; k += kMT) {
            const float c = fminf(fmaxf(xs[b * K + k], -65504.0f), 65504.0f);
            xs[b * K + k] = Elem<T>::to_f(Elem<T>::from_f(c * inv));
        }
    }
    __syncthreads();
}

enum class Epi { Qkv, Gelu, Residual };

// One GEMV phase: out[b, n] = sum_k xs[b, k] W[k, n] over N columns (N a
// multiple of 256), W row-major [K, N], split as `sp`, then the epilogue.
template <typename T, Epi EPI>
__device__ void gemv_phase(const MegaArgs& a, const float* xs, const T* __restrict__ W, uint32_t K, uint32_t N,
                           MegaSplit sp, T* out, const MegaLayer* L, float* red) {
    const uint32_t B = a.B;
    const uint32_t chunks = N / kMCols;
    const uint32_t items = chunks * sp.ks;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ int s_last;
    for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
        const uint32_t c = it / sp.ks, si = it % sp.ks;
        const uint32_t k0 = si * sp.kc, k1 = min(K, k0 + sp.kc);
        const uint32_t n0 = c * kMCols + lane * 8;
        float acc[kMaxB][8];
#pragma unroll
        for (int b = 0; b < kMaxB; ++b)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[b][e] = 0.0f;
        uint32_t k = k0 + warp;
        // four rows in flight per warp
        for (; k + 3 * kMW < k1; k += 4 * kMW) {
            Vec8 w4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                w4[u] = *reinterpret_cast<const Vec8*>(W + (uint64_t)(k + u * kMW) * N + n0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float f[8];
                unpack8<T>(w4[u], f);
#pragma unroll
                for (int b = 0; b < kMaxB; ++b) {
                    if (b >= (int)B) break;
                    const float xv = xs[b * K + k + u * kMW];
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[b][e] = fmaf(xv, f[e], acc[b][e]);
                }
            }
        }
        for (; k < k1; k += kMW) {
            float f[8];
            unpack8<T>(*reinterpret_cast<const Vec8*>(W + (uint64_t)k * N + n0), f);
#pragma unroll
            for (int b = 0; b < kMaxB; ++b) {
                if (b >= (int)B) break;
                const float xv = xs[b * K + k];
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[b][e] = fmaf(xv, f[e], acc[b][e]);
            }
        }
        // reduce the eight warps: red[warp][b][256]
        for (uint32_t b = 0; b < B; ++b)
#pragma unroll
            for (int e = 0; e < 8; ++e) red[(warp * kMaxB + b) * kMCols + lane * 8 + e] = acc[b][e];
        __syncthreads();
        const uint32_t nout = B * kMCols;
        float* part = a.partial + (uint64_t)it * kMaxB * kMCols;
        for (uint32_t o = threadIdx.x; o < nout; o += kMT) {
            const uint32_t b = o / kMCols, col = o % kMCols;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kMW; ++w) s += red[(w * kMaxB + b) * kMCols + col];
            red[(kMW * kMaxB + b) * kMCols + col] = s;  // the item's sum, after the warp slots
            if (sp.ks > 1) __stcg(part + b * kMCols + col, s);
        }
        __syncthreads();
        if (sp.ks > 1) {
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const unsigned int t = atomicAdd(&a.tickets[c], 1u);
                s_last = t == sp.ks - 1;
                if (s_last) a.tickets[c] = 0;  // every split arrived: ready for the next use
            }
            __syncthreads();
            if (!s_last) continue;
            __threadfence();
            for (uint32_t o = threadIdx.x; o < nout; o += kMT) {
                const uint32_t b = o / kMCols, col = o % kMCols;
                float s = 0.0f;
                for (uint32_t j = 0; j < sp.ks; ++j)
                    s += __ldcg(a.partial + ((uint64_t)(c * sp.ks + j) * kMaxB + b) * kMCols + col);
                red[(kMW * kMaxB + b) * kMCols + col] = s;
            }
            __syncthreads();
        }
        // epilogue over column pairs (RoPE rotates adjacent pairs)
        const float* sum = red + (uint64_t)kMW * kMaxB * kMCols;
        for (uint32_t o = threadIdx.x; o < B * (kMCols / 2); o += kMT) {
            const uint32_t b = o / (kMCols / 2), pcol = (o % (kMCols / 2)) * 2;
            const uint32_t n = c * kMCols + pcol;
            float v0 = sum[b * kMCols + pcol], v1 = sum[b * kMCols + pcol + 1];
            if constexpr (EPI == Epi::Gelu) {
                out[(uint64_t)b * N + n] = Elem<T>::from_f(gelu_f(v0));
                out[(uint64_t)b * N + n + 1] = Elem<T>::from_f(gelu_f(v1));
            } else if constexpr (EPI == Epi::Residual) {
                T* y = out + (uint64_t)b * N + n;
                y[0] = Elem<T>::from_f(ldg_f(y) + v0);
                y[1] = Elem<T>::from_f(ldg_f(y + 1) + v1);
            } else {
                // columns [q heads | k heads | v heads]; RoPE on q and k at
                // position *d_pos, (cos, sin) from the model's table; q to
                // a.q, k and v to row b * max_seq + pos of the layer's cache.
                const uint32_t Dh = a.Dh, hq = a.H * Dh, hk = a.Hkv * Dh;
                const uint32_t pos = *a.d_pos;
                if (n < hq + hk) {
                    const uint32_t p = (n % Dh) / 2;
                    const float2 cs = a.rope_cs[(uint64_t)pos * (Dh / 2) + p];
                    const float r0 = v0 * cs.x - v1 * cs.y, r1 = v0 * cs.y + v1 * cs.x;
                    v0 = r0;
                    v1 = r1;
                }
                T* dst;
                if (n < hq)
                    dst = reinterpret_cast<T*>(a.q) + (uint64_t)b * hq + n;
                else if (n < hq + hk)
                    dst = reinterpret_cast<T*>(L->kc) + ((uint64_t)b * a.max_seq + pos) * hk + (n - hq);
                else
                    dst = reinterpret_cast<T*>(L->vc) + ((uint64_t)b * a.max_seq + pos) * hk + (n - hq - hk);
                dst[0] = Elem<T>::from_f(v0);
                dst[1] = Elem<T>::from_f(v1);
            }
        }
        __syncthreads();
    }
}

// Single-query attention of every (sequence, head) over positions [0, len)
// of the layer's cache: items of 32 positions, one warp per position stream.
template <typename T>
__device__ void attention_phase(const MegaArgs& a, const MegaLayer* L, float* red) {
    const uint32_t B = a.B, H = a.H, Dh = a.Dh, G = H / a.Hkv, hk = a.Hkv * Dh;
    const uint32_t len = *a.d_len;
    const uint32_t per = 32;
    const uint32_t nsplit = (len + per - 1) / per;
    const uint32_t items = B * H * nsplit;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ne = Dh / 32;  // q / o elements per lane (2 or 4)
    __shared__ int s_last;
    for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
        const uint32_t s = it % nsplit, bh = it / nsplit, h = bh % H, b = bh / H, g = h / G;
        float q[4], o[4];
        const T* qp = reinterpret_cast<const T*>(a.q) + (uint64_t)b * H * Dh + (uint64_t)h * Dh;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            q[e] = e < (int)ne ? ldg_f(qp + lane + 32 * e) : 0.0f;
            o[e] = 0.0f;
        }
        float m = -INFINITY, l = 0.0f;
        const uint32_t p0 = s * per, p1 = min(len, p0 + per);
        const T* kb = reinterpret_cast<const T*>(L->kc) + (uint64_t)b * a.max_seq * hk + (uint64_t)g * Dh;
        const T* vb = reinterpret_cast<const T*>(L->vc) + (uint64_t)b * a.max_seq * hk + (uint64_t)g * Dh;
        for (uint32_t p = p0 + warp; p < p1; p += kMW) {
            float d = 0.0f;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < (int)ne) d += q[e] * ldg_f(kb + (uint64_t)p * hk + lane + 32 * e);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            const float sc = d * a.scale_log2;
            const float mn = fmaxf(m, sc);
            const float al = exp2f(m - mn), w = exp2f(sc - mn);
            l = l * al + w;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < (int)ne) o[e] = o[e] * al + w * ldg_f(vb + (uint64_t)p * hk + lane + 32 * e);
            m = mn;
        }
        // merge the warps: red[warp][2 + Dh]
        float* rw = red + warp * (2 + 128);
        if (lane == 0) {
            rw[0] = m;
            rw[1] = l;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (e < (int)ne) rw[2 + lane + 32 * e] = o[e];
        __syncthreads();
        float* part = a.partial + (uint64_t)it * (2 + 128);
        if (threadIdx.x < 32) {
            float mm = -INFINITY;
            for (int w = 0; w < kMW; ++w) mm = fmaxf(mm, red[w * 130]);
            float ll = 0.0f, oo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int w = 0; w < kMW; ++w) {
                const float mw = red[w * 130];
                const float f = mw == -INFINITY ? 0.0f : exp2f(mw - mm);
                ll += red[w * 130 + 1] * f;
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (e < (int)ne) oo[e] += red[w * 130 + 2 + lane + 32 * e] * f;
            }
            if (lane == 0) {
                __stcg(part, mm);
                __stcg(part + 1, ll);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < (int)ne) __stcg(part + 2 + lane + 32 * e, oo[e]);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned int* tk = &a.tickets[a.att_tickets + bh];
            const unsigned int t = atomicAdd(tk, 1u);
            s_last = t == nsplit - 1;
            if (s_last) *tk = 0;
        }
        __syncthreads();
        if (s_last && threadIdx.x < 32) {
            __threadfence();
            const float* base = a.partial + (uint64_t)bh * nsplit * (2 + 128);
            float mm = -INFINITY;
            for (uint32_t j = 0; j < nsplit; ++j) mm = fmaxf(mm, __ldcg(base + j * 130));
            float ll = 0.0f, oo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (uint32_t j = 0; j < nsplit; ++j) {
                const float mj = __ldcg(base + j * 130);
                const float f = mj == -INFINITY ? 0.0f : exp2f(mj - mm);
                ll += __ldcg(base + j * 130 + 1) * f;
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (e < (int)ne) oo[e] += __ldcg(base + j * 130 + 2 + lane + 32 * e) * f;
            }
            const float inv = ll > 0.0f ? 1.0f / ll : 0.0f;
            T* op = reinterpret_cast<T*>(a.attn) + (uint64_t)b * H * Dh + (uint64_t)h * Dh;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < (int)ne) op[lane + 32 * e] = Elem<T>::from_f(oo[e] * inv);
        }
        __syncthreads();
    }
}

// LM head over the normalised rows xs [B, D]: per CTA the best greedy key of
// each sequence, optionally the rounded logits.
template <typename T>
__device__ void head_phase(const MegaArgs& a, const float* xs, float* red) {
    const uint32_t B = a.B, D = a.D, V = a.V;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long best[kMaxB];
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) best[b] = 0ull;
    T* logits = reinterpret_cast<T*>(a.logits);
    if (a.tied) {
        // logits[b, v] = xs[b] . E[v]: E rows are contiguous; a warp per row.
        const T* E = reinterpret_cast<const T*>(a.emb);
        const uint32_t rows_per_item = 64, items = (V + rows_per_item - 1) / rows_per_item;
        for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
            for (uint32_t r = warp; r < rows_per_item; r += kMW) {
                const uint32_t v = it * rows_per_item + r;
                if (v >= V) break;
                float acc[kMaxB] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (uint32_t k = lane * 8; k < D; k += 256) {
                    float f[8];
                    unpack8<T>(*reinterpret_cast<const Vec8*>(E + (uint64_t)v * D + k), f);
#pragma unroll
                    for (int b = 0; b < kMaxB; ++b) {
                        if (b >= (int)B) break;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[b] = fmaf(xs[b * D + k + e], f[e], acc[b]);
                    }
                }
#pragma unroll
                for (int b = 0; b < kMaxB; ++b) {
                    if (b >= (int)B) break;
                    float sv = acc[b];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, off);
                    const T rounded = Elem<T>::from_f(sv);
                    if (lane == 0 && logits) logits[(uint64_t)b * V + v] = rounded;
                    const unsigned long long key = elem_key(Elem<T>::to_f(rounded), v);
                    best[b] = key > best[b] ? key : best[b];
                }
            }
        }
    } else {
        // logits = xs . lm_head [D, V]: 256-column items over all D rows.
        const T* W = reinterpret_cast<const T*>(a.lm_head);
        const uint32_t items = V / kMCols;
        for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
            const uint32_t n0 = it * kMCols + lane * 8;
            float acc[kMaxB][8];
#pragma unroll
            for (int b = 0; b < kMaxB; ++b)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[b][e] = 0.0f;
            for (uint32_t k = warp; k < D; k += kMW) {
                float f[8];
                unpack8<T>(*reinterpret_cast<const Vec8*>(W + (uint64_t)k * V + n0), f);
#pragma unroll
                for (int b = 0; b < kMaxB; ++b) {
                    if (b >= (int)B) break;
                    const float xv = xs[b * D + k];
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[b][e] = fmaf(xv, f[e], acc[b][e]);
                }
            }
            for (uint32_t b = 0; b < B; ++b)
#pragma unroll
                for (int e = 0; e < 8; ++e) red[(warp * kMaxB + b) * kMCols + lane * 8 + e] = acc[b][e];
            __syncthreads();
            for (uint32_t o = threadIdx.x; o < B * kMCols; o += kMT) {
                const uint32_t b = o / kMCols, col = o % kMCols, v = it * kMCols + col;
                float sv = 0.0f;
#pragma unroll
                for (int w = 0; w < kMW; ++w) sv += red[(w * kMaxB + b) * kMCols + col];
                const T rounded = Elem<T>::from_f(sv);
                if (logits) logits[(uint64_t)b * V + v] = rounded;
                const unsigned long long key = elem_key(Elem<T>::to_f(rounded), v);
                best[b] = key > best[b] ? key : best[b];
            }
            __syncthreads();
        }
    }
    // CTA-wide maximum per sequence
    __shared__ unsigned long long s_best[kMaxB][kMW];
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
        unsigned long long k = best[b];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, off);
            k = t > k ? t : k;
        }
        if (lane == 0) s_best[b][warp] = k;
    }
    __syncthreads();
    if (threadIdx.x < B) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kMW; ++w) k = s_best[threadIdx.x][w] > k ? s_best[threadIdx.x][w] : k;
        __stcg(&a.keys[(uint64_t)blockIdx.x * kMaxB + threadIdx.x], k);
    }
}

template <typename T>
__global__ void __launch_bounds__(kMT, 1) decode_mega_kernel(const MegaArgs a) {
    extern __shared__ float sm[];
    const uint32_t B = a.B, D = a.D;
    const uint32_t kmax = max(max(D, a.F), a.H * a.Dh);
    float* xs = sm;                           // [B][kmax]
    float* red = sm + (uint64_t)kMaxB * kmax;  // [(kMW + 1) * kMaxB * 256]
    // embed: x[b] = E[ids[b]]
    {
        const T* E = reinterpret_cast<const T*>(a.emb);
        T* x = reinterpret_cast<T*>(a.x);
        for (uint32_t e = blockIdx.x * kMT + threadIdx.x; e < B * D; e += gridDim.x * kMT) {
            const uint32_t b = e / D, d = e % D;
            uint32_t tok = __ldcg(a.ids_in + b);
            if (tok >= a.V) tok = a.V - 1;
            x[e] = E[(uint64_t)tok * D + d];
        }
    }
    if (!grid_sync(a)) return;
    const uint32_t hq = a.H * a.Dh, C = (a.H + 2 * a.Hkv) * a.Dh;
    for (uint32_t l = 0; l < a.layers; ++l) {
        const MegaLayer* L = a.layer + l;
        load_rows<T>(reinterpret_cast<const T*>(a.x), B, D, true, a.eps, xs);
        gemv_phase<T, Epi::Qkv>(a, xs, reinterpret_cast<const T*>(L->wqkv), D, C, a.s_qkv, nullptr, L, red);
        if (!grid_sync(a)) return;
        attention_phase<T>(a, L, red);
        if (!grid_sync(a)) return;
        load_rows<T>(reinterpret_cast<const T*>(a.attn), B, hq, false, a.eps, xs);
        gemv_phase<T, Epi::Residual>(a, xs, reinterpret_cast<const T*>(L->wo), hq, D, a.s_wo,
                                     reinterpret_cast<T*>(a.x), L, red);
        if (!grid_sync(a)) return;
        load_rows<T>(reinterpret_cast<const T*>(a.x), B, D, true, a.eps, xs);
        gemv_phase<T, Epi::Gelu>(a, xs, reinterpret_cast<const T*>(L->w1), D, a.F, a.s_w1,
                                 reinterpret_cast<T*>(a.h1), L, red);
        if (!grid_sync(a)) return;
        load_rows<T>(reinterpret_cast<const T*>(a.h1), B, a.F, false, a.eps, xs);
        gemv_phase<T, Epi::Residual>(a, xs, reinterpret_cast<const T*>(L->w2), a.F, D, a.s_w2,
                                     reinterpret_cast<T*>(a.x), L, red);
        if (!grid_sync(a)) return;
    }
    load_rows<T>(reinterpret_cast<const T*>(a.x), B, D, true, a.eps, xs);
    head_phase<T>(a, xs, red);
    if (!grid_sync(a)) return;
    if (blockIdx.x == 0) {
        if (threadIdx.x < B) {
            unsigned long long k = 0ull;
            for (uint32_t c = 0; c < gridDim.x; ++c) {
                const unsigned long long t = __ldcg(&a.keys[(uint64_t)c * kMaxB + threadIdx.x]);
                k = t > k ? t : k;
            }
            a.ids_out[threadIdx.x] = k ? key_to_offset(k) : 0u;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // one more cached position (advance_kernel of the per-op chain)
            const uint32_t p = *a.d_pos + 1;
            a.d_pos[0] = p;
            a.d_pos[2] += 1;
            *a.d_len = p + 1;
        }
    }
}

MegaSplit split_for(uint32_t K, uint32_t N, int grid) {
    const uint32_t chunks = N / kMCols;
    uint32_t ks = std::max<uint32_t>(1, (uint32_t)grid / std::max<uint32_t>(1, chunks));
    static const uint32_t ks_cap = [] {
        const char* e = getenv("EVKCU_MEGA_KSMAX");
        return e ? (uint32_t)atoi(e) : 0u;
    }();
    if (ks_cap) ks = std::min(ks, ks_cap);
    ks = std::min<uint32_t>(ks, std::max<uint32_t>(1, K / 16));  // at least 16 rows per item
    uint32_t kc = (K + ks - 1) / ks;
    kc = (kc + 7) / 8 * 8;
    ks = (K + kc - 1) / kc;
    return {kc, ks};
}

}  // namespace

// Whether the persistent step handles a model of this shape (see llm.cu).
bool decode_mega_supported(uint32_t B, uint32_t D, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t F, uint32_t V,
                           bool tied) {
    const uint32_t C = (H + 2 * Hkv) * Dh;
    const uint32_t kmax = std::max(std::max(D, F), H * Dh);
    return B >= 1 && B <= (uint32_t)kMaxB && (Dh == 64 || Dh == 128) && D % kMCols == 0 && C % kMCols == 0 &&
           F % kMCols == 0 && (H * Dh) % kMCols == 0 && (tied ? V % 8 == 0 && D % 256 == 0 : V % kMCols == 0) &&
           (uint64_t)kMaxB * kmax * 4 <= 64 * 1024;
}

// Scratch the step needs (bytes): partials, tickets, keys, barrier words.
size_t decode_mega_scratch_bytes(uint32_t B, uint32_t D, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t F,
                                 uint32_t max_seq, int grid) {
    const uint32_t C = (H + 2 * Hkv) * Dh;
    uint64_t items = 0;
    for (auto kn : {std::make_pair(D, C), std::make_pair(H * Dh, D), std::make_pair(D, F), std::make_pair(F, D)}) {
        const MegaSplit s = split_for(kn.first, kn.second, grid);
        items = std::max<uint64_t>(items, (uint64_t)(kn.second / kMCols) * s.ks * kMaxB * kMCols);
    }
    const uint64_t att = (uint64_t)kMaxB * H * ((max_seq + 31) / 32) * 130;
    const uint64_t partial = std::max(items, att) * 4;
    const uint64_t tickets = 4096 * 4;
    const uint64_t keys = (uint64_t)grid * kMaxB * 8;
    (void)B;
    return partial + tickets + keys + 64;
}

int decode_mega_step(const MegaHost& h, int dtype, cudaStream_t st) {
    DeviceState* ds = state();
    const int grid = ds->sm_count;
    MegaArgs a{};
    a.B = h.B;
    a.D = h.D;
    a.H = h.H;
    a.Hkv = h.Hkv;
    a.Dh = h.Dh;
    a.F = h.F;
    a.V = h.V;
    a.layers = h.layers;
    a.max_seq = h.max_seq;
    a.tied = h.tied;
    a.eps = h.eps;
    a.scale_log2 = 1.4426950408889634f / sqrtf((float)h.Dh);
    a.emb = h.emb;
    a.lm_head = h.lm_head;
    a.layer = reinterpret_cast<const MegaLayer*>(h.layer_table);
    a.x = h.x;
    a.q = h.q;
    a.attn = h.attn;
    a.h1 = h.h1;
    a.logits = h.logits;
    a.rope_cs = h.rope_cs;
    a.d_pos = h.d_pos;
    a.d_len = h.d_len;
    a.ids_in = h.ids_in;
    a.ids_out = h.ids_out;
    const uint32_t C = (h.H + 2 * h.Hkv) * h.Dh;
    a.s_qkv = split_for(h.D, C, grid);
    a.s_wo = split_for(h.H * h.Dh, h.D, grid);
    a.s_w1 = split_for(h.D, h.F, grid);
    a.s_w2 = split_for(h.F, h.D, grid);
    const size_t sbytes = decode_mega_scratch_bytes(h.B, h.D, h.H, h.Hkv, h.Dh, h.F, h.max_seq, grid);
    char* s = reinterpret_cast<char*>(h.scratch);
    const size_t tickets_off = sbytes - 64 - (size_t)grid * kMaxB * 8 - 4096 * 4;
    a.partial = reinterpret_cast<float*>(s);
    a.tickets = reinterpret_cast<unsigned int*>(s + tickets_off);
    a.keys = reinterpret_cast<unsigned long long*>(s + tickets_off + 4096 * 4);
    a.bar = reinterpret_cast<unsigned int*>(s + sbytes - 64);
    a.err = ds->d_error;
    a.att_tickets = 2048;  // chunks use [0, 2048), attention merges [2048, 4096)
    if (C / kMCols > 2048 || h.F / kMCols > 2048 || (uint64_t)h.B * h.H > 2048)
        return fail(EVKCU_BAD_SHAPE, "decode_mega: too many column chunks");
    const uint32_t kmax = std::max(std::max(h.D, h.F), h.H * h.Dh);
    const size_t smem = ((size_t)kMaxB * kmax + (size_t)(kMW + 1) * kMaxB * kMCols) * sizeof(float);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        auto kern = decode_mega_kernel<T>;
        static bool attr = false;
        if (!attr) {
            EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
            attr = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kMT);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attrs[1];
        attrs[0].id = cudaLaunchAttributeCooperative;
        attrs[0].val.cooperative = 1;
        cfg.attrs = attrs;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
        if (e != cudaSuccess) return cuda_fail(e, "decode_mega (cooperative launch)");
        return after_launch("decode_mega");
    });
}

}  // namespace evkcu
