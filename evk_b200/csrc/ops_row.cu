// ops_row.cu — row-wise HBM-bound ops: rms_norm, softmax, rope.
// One CTA per row with 16-byte vector loads; block-wide reductions with warp
// shuffles and a 32-slot shared buffer.  The row is re-read for the output
// pass, which hits L1/L2 (rows are at most a few tens of KB), so DRAM traffic
// stays one read + one write per element.
#include <float.h>

#include "common.cuh"

namespace evkcu {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum; every thread receives the result.
__device__ float block_sum(float v, float* sh) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[wid] = v;
    __syncthreads();
    float t = lane < nw ? sh[lane] : 0.0f;
    return warp_sum(t);
}

// Online (max, sum-of-exp) pair merge.
__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
    float mn = fmaxf(m, m2);
    s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
    m = mn;
}

__device__ void block_max_sum(float& m, float& s, float* shm, float* shs) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        ms_merge(m, s, m2, s2);
    }
    __syncthreads();
    if (lane == 0) { shm[wid] = m; shs[wid] = s; }
    __syncthreads();
    m = lane < nw ? shm[lane] : -FLT_MAX;
    s = lane < nw ? shs[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        ms_merge(m, s, m2, s2);
    }
}

// ---------------------------------------------------------------- rms_norm --
// shaders/rms_norm.comp:21-48: v = clamp(x, +-65504); y = v * rsqrt(sum(v^2)/D + eps)
template <typename T, bool VEC>
__global__ void rms_norm_kernel(const T* __restrict__ in, T* __restrict__ out, const T* __restrict__ gamma,
                                uint32_t D, float eps) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    __shared__ float sh[32];
    const uint64_t row = blockIdx.x;
    const T* x = in + row * D;
    T* y = out + row * D;
    float ss = 0.0f;
    if (VEC) {
        const Vec8* xv = reinterpret_cast<const Vec8*>(x);
        for (uint32_t c = threadIdx.x; c < D / 8; c += blockDim.x) {
            float f[8];
            unpack8<T>(xv[c], f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                float v = fminf(fmaxf(f[k], -65504.0f), 65504.0f);
                ss += v * v;
            }
        }
    } else {
        for (uint32_t c = threadIdx.x; c < D; c += blockDim.x) {
            float v = fminf(fmaxf(Elem<T>::to_f(x[c]), -65504.0f), 65504.0f);
            ss += v * v;
        }
    }
    float total = block_sum(ss, sh);
    float inv = rsqrtf(total / (float)D + eps);
    if (VEC) {
        const Vec8* xv = reinterpret_cast<const Vec8*>(x);
        const Vec8* gv = reinterpret_cast<const Vec8*>(gamma);
        Vec8* yv = reinterpret_cast<Vec8*>(y);
        for (uint32_t c = threadIdx.x; c < D / 8; c += blockDim.x) {
            float f[8];
            unpack8<T>(xv[c], f);
            float g[8];
            if (gamma) unpack8<T>(gv[c], g);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                float v = fminf(fmaxf(f[k], -65504.0f), 65504.0f) * inv;
                f[k] = gamma ? v * g[k] : v;
            }
            yv[c] = pack8<T>(f);
        }
    } else {
        for (uint32_t c = threadIdx.x; c < D; c += blockDim.x) {
            float v = fminf(fmaxf(Elem<T>::to_f(x[c]), -65504.0f), 65504.0f) * inv;
            if (gamma) v *= Elem<T>::to_f(gamma[c]);
            y[c] = Elem<T>::from_f(v);
        }
    }
}

// One warp per row (up to 8 * 32 * NV elements): the row stays in registers
// as packed 16-byte vectors between the sum of squares and the output, so it
// is read once and the reduction is warp shuffles only.  Eight rows per
// 256-thread CTA; used for many rows (prefill), where it streams faster than
// one CTA per row.
template <typename T, int NV>
__global__ void __launch_bounds__(256) rms_norm_warp_kernel(const T* __restrict__ in, T* __restrict__ out,
                                                            const T* __restrict__ gamma, uint32_t rows, uint32_t D,
                                                            float eps) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (row >= rows) return;
    const Vec8* xv = reinterpret_cast<const Vec8*>(in + (uint64_t)row * D);
    const uint32_t nv = D / 8;
    Vec8 v[NV];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < nv) {
            v[i] = xv[c];
            float f[8];
            unpack8<T>(v[i], f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float x = fminf(fmaxf(f[k], -65504.0f), 65504.0f);
                ss += x * x;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)D + eps);
    const Vec8* gv = reinterpret_cast<const Vec8*>(gamma);
    Vec8* yv = reinterpret_cast<Vec8*>(out + (uint64_t)row * D);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < nv) {
            float f[8], g[8];
            unpack8<T>(v[i], f);
            if (gamma) unpack8<T>(gv[c], g);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float x = fminf(fmaxf(f[k], -65504.0f), 65504.0f) * inv;
                f[k] = gamma ? x * g[k] : x;
            }
            yv[c] = pack8<T>(f);
        }
    }
}

// ----------------------------------------------------------------- softmax --
// shaders/softmax.comp:23-66: entries with raw <= -65504 are masked (skipped
// in max and sum, written as 0); sum clamped to >= 1e-20; outputs computed
// from the raw logits so they are quantised once.
constexpr float kMaskSentinel = -65504.0f;

template <typename T>
__global__ void softmax_kernel(const T* __restrict__ in, T* __restrict__ out, uint32_t L, float scale, bool vec) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    __shared__ float shm[32], shs[32];
    const uint64_t row = blockIdx.x;
    const T* x = in + row * L;
    T* y = out + row * L;
    float m = -FLT_MAX, s = 0.0f;
    auto acc = [&](float raw) {
        if (raw <= kMaskSentinel) return;
        float v = raw * scale;
        if (v > m) {
            s = s * __expf(m - v) + 1.0f;
            m = v;
        } else {
            s += __expf(v - m);
        }
    };
    if (vec) {
        const Vec8* xv = reinterpret_cast<const Vec8*>(x);
        for (uint32_t c = threadIdx.x; c < L / 8; c += blockDim.x) {
            float f[8];
            unpack8<T>(xv[c], f);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc(f[k]);
        }
    } else {
        for (uint32_t c = threadIdx.x; c < L; c += blockDim.x) acc(Elem<T>::to_f(x[c]));
    }
    block_max_sum(m, s, shm, shs);
    float inv = 1.0f / fmaxf(s, 1e-20f);
    auto val = [&](float raw) { return raw <= kMaskSentinel ? 0.0f : __expf(raw * scale - m) * inv; };
    if (vec) {
        const Vec8* xv = reinterpret_cast<const Vec8*>(x);
        Vec8* yv = reinterpret_cast<Vec8*>(y);
        for (uint32_t c = threadIdx.x; c < L / 8; c += blockDim.x) {
            float f[8];
            unpack8<T>(xv[c], f);
#pragma unroll
            for (int k = 0; k < 8; ++k) f[k] = val(f[k]);
            yv[c] = pack8<T>(f);
        }
    } else {
        for (uint32_t c = threadIdx.x; c < L; c += blockDim.x) y[c] = Elem<T>::from_f(val(Elem<T>::to_f(x[c])));
    }
}

// -------------------------------------------------------------------- rope --
// shaders/rope.comp:18-40: pair p of a rot_dim slice at position t rotates by
// t * base^(-2p/rot_dim).  One thread per 4 pairs (16 bytes) when possible.
template <typename T>
__global__ void rope_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t rows, uint32_t seq_len,
                            uint32_t dim, uint32_t head_dim, uint32_t pos_offset, float base, bool vec) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    const uint32_t per_row = vec ? dim / 8 : dim / 2;  // work items per row
    const uint64_t total = rows * per_row;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t w = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += stride) {
        uint64_t row = w / per_row;
        uint32_t item = (uint32_t)(w % per_row);
        float t = (float)((uint32_t)(row % seq_len) + pos_offset);
        if (vec) {
            uint32_t c0 = item * 8;
            const Vec8* src = reinterpret_cast<const Vec8*>(in + row * dim + c0);
            float f[8];
            unpack8<T>(*src, f);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t p = ((c0 % head_dim) >> 1) + k;
                float inv_freq = powf(base, -2.0f * (float)p / (float)head_dim);
                float sn, cs;
                sincosf(t * inv_freq, &sn, &cs);
                float x0 = f[2 * k], x1 = f[2 * k + 1];
                f[2 * k] = x0 * cs - x1 * sn;
                f[2 * k + 1] = x0 * sn + x1 * cs;
            }
            *reinterpret_cast<Vec8*>(out + row * dim + c0) = pack8<T>(f);
        } else {
            uint32_t c0 = item * 2;
            uint32_t p = (c0 % head_dim) >> 1;
            float inv_freq = powf(base, -2.0f * (float)p / (float)head_dim);
            float sn, cs;
            sincosf(t * inv_freq, &sn, &cs);
            float x0 = Elem<T>::to_f(in[row * dim + c0]);
            float x1 = Elem<T>::to_f(in[row * dim + c0 + 1]);
            out[row * dim + c0] = Elem<T>::from_f(x0 * cs - x1 * sn);
            out[row * dim + c0 + 1] = Elem<T>::from_f(x0 * sn + x1 * cs);
        }
    }
}

inline unsigned row_threads(uint32_t items) {
    unsigned t = (items + 31) / 32 * 32;
    if (t < 32) t = 32;
    if (t > 512) t = 512;
    return t;
}

// --------------------------------------------------------- rms_norm + rope --
// The two bandwidth ops fused (rows of `dim`): y = rope(rms_norm(x) [* gamma])
// with rms_norm as above (shaders/rms_norm.comp:21-48) and rope as
// rope_kernel (shaders/rope.comp:18-40, per head_dim slice, position
// row % seq_len + pos_offset), without the intermediate rounding to storage:
// one read and one write per element instead of two of each.
template <typename T>
__global__ void rms_norm_rope_kernel(const T* __restrict__ in, T* __restrict__ out, const T* __restrict__ gamma,
                                     uint32_t D, uint32_t seq_len, uint32_t head_dim, uint32_t pos_offset, float eps,
                                     float base) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sh[32];
    const uint64_t row = blockIdx.x;
    const Vec8* xv = reinterpret_cast<const Vec8*>(in + row * D);
    const Vec8* gv = reinterpret_cast<const Vec8*>(gamma);
    Vec8* yv = reinterpret_cast<Vec8*>(out + row * D);
    float ss = 0.0f;
    for (uint32_t c = threadIdx.x; c < D / 8; c += blockDim.x) {
        float f[8];
        unpack8<T>(xv[c], f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float v = fminf(fmaxf(f[k], -65504.0f), 65504.0f);
            ss += v * v;
        }
    }
    const float inv = rsqrtf(block_sum(ss, sh) / (float)D + eps);
    const float t = (float)((uint32_t)(row % seq_len) + pos_offset);
    for (uint32_t c = threadIdx.x; c < D / 8; c += blockDim.x) {
        float f[8], g[8];
        unpack8<T>(xv[c], f);
        if (gamma) unpack8<T>(gv[c], g);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float v = fminf(fmaxf(f[k], -65504.0f), 65504.0f) * inv;
            f[k] = gamma ? v * g[k] : v;
        }
        const uint32_t c0 = c * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t p = ((c0 % head_dim) >> 1) + k;
            const float inv_freq = powf(base, -2.0f * (float)p / (float)head_dim);
            float sn, cs;
            sincosf(t * inv_freq, &sn, &cs);
            const float x0 = f[2 * k], x1 = f[2 * k + 1];
            f[2 * k] = x0 * cs - x1 * sn;
            f[2 * k + 1] = x0 * sn + x1 * cs;
        }
        yv[c] = pack8<T>(f);
    }
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_rms_norm(const void* in, void* out, const void* gamma, uint32_t rows, uint32_t D, float eps,
                              int dtype, void* stream) {
    if (rows == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_rms_norm: null pointer");
    EVKCU_CHECK_ARG(D > 0, EVKCU_BAD_SHAPE, "evkcu_rms_norm: D must be > 0");
    bool vec = (D % 8 == 0) && aligned16(in) && aligned16(out) && (!gamma || aligned16(gamma));
    unsigned threads = row_threads(vec ? D / 8 : D);
    const uint32_t per_lane = (D / 8 + 31) / 32;  // 16-byte vectors per lane, one warp per row
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        // Many rows: one warp per row (measured 36.8 -> 28.0 us at 16384 x 2048);
        // a few rows (decode) keep one CTA per row, which spreads them over SMs.
        if (vec && per_lane <= 16 && rows >= 256) {
            const unsigned grid = (rows + 7) / 8;
            auto go = [&](auto kern) {
                return launch_pdl("evkcu_rms_norm", kern, grid, 256, 0, as_stream(stream), (const T*)in, (T*)out,
                                  (const T*)gamma, rows, D, eps);
            };
            if (per_lane <= 1) return go(rms_norm_warp_kernel<T, 1>);
            if (per_lane <= 2) return go(rms_norm_warp_kernel<T, 2>);
            if (per_lane <= 4) return go(rms_norm_warp_kernel<T, 4>);
            if (per_lane <= 8) return go(rms_norm_warp_kernel<T, 8>);
            return go(rms_norm_warp_kernel<T, 16>);
        }
        if (vec)
            return launch_pdl("evkcu_rms_norm", rms_norm_kernel<T, true>, rows, threads, 0, as_stream(stream),
                              (const T*)in, (T*)out, (const T*)gamma, D, eps);
        return launch_pdl("evkcu_rms_norm", rms_norm_kernel<T, false>, rows, threads, 0, as_stream(stream), (const T*)in,
                          (T*)out, (const T*)gamma, D, eps);
    });
}

extern "C" int evkcu_softmax(const void* in, void* out, uint32_t rows, uint32_t L, float scale, int dtype,
                             void* stream) {
    if (rows == 0 || L == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_softmax: null pointer");
    bool vec = (L % 8 == 0) && aligned16(in) && aligned16(out);
    unsigned threads = row_threads(vec ? L / 8 : L);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_softmax", softmax_kernel<T>, rows, threads, 0, as_stream(stream), (const T*)in,
                          (T*)out, L, scale, vec);
    });
}

extern "C" int evkcu_rope(const void* in, void* out, uint32_t batch, uint32_t seq_len, uint32_t dim,
                          uint32_t head_dim, uint32_t pos_offset, float base, int dtype, void* stream) {
    if (batch == 0 || seq_len == 0 || dim == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_rope: null pointer");
    if (head_dim == 0) head_dim = dim;
    EVKCU_CHECK_ARG(dim % 2 == 0 && head_dim % 2 == 0 && dim % head_dim == 0, EVKCU_BAD_SHAPE,
                    "evkcu_rope: dim and head_dim must be even and head_dim must divide dim");
    bool vec = (head_dim % 8 == 0) && aligned16(in) && aligned16(out);
    uint64_t rows = (uint64_t)batch * seq_len;
    uint64_t items = rows * (vec ? dim / 8 : dim / 2);
    DeviceState* s = state();
    uint64_t want = (items + 255) / 256;
    unsigned grid = (unsigned)(want < (uint64_t)s->sm_count * 8 ? want : (uint64_t)s->sm_count * 8);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_rope", rope_kernel<T>, grid, 256, 0, as_stream(stream), (const T*)in, (T*)out, rows,
                          seq_len, dim, head_dim, pos_offset, base, vec);
    });
}

extern "C" int evkcu_rms_norm_rope(const void* in, void* out, const void* gamma, uint32_t rows, uint32_t seq_len,
                                   uint32_t dim, uint32_t head_dim, uint32_t pos_offset, float eps, float base,
                                   int dtype, void* stream) {
    if (rows == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, "evkcu_rms_norm_rope: null pointer");
    if (head_dim == 0) head_dim = dim;
    EVKCU_CHECK_ARG(seq_len > 0 && dim > 0 && dim % 8 == 0 && head_dim % 8 == 0 && dim % head_dim == 0,
                    EVKCU_BAD_SHAPE, "evkcu_rms_norm_rope: dim and head_dim must be multiples of 8, head_dim | dim");
    EVKCU_CHECK_ARG(aligned16(in) && aligned16(out) && (!gamma || aligned16(gamma)), EVKCU_BAD_ALIGN,
                    "evkcu_rms_norm_rope: buffers must be 16-byte aligned");
    const unsigned threads = row_threads(dim / 8);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_rms_norm_rope", rms_norm_rope_kernel<T>, rows, threads, 0, as_stream(stream),
                          (const T*)in, (T*)out, (const T*)gamma, dim, seq_len, head_dim, pos_offset, eps, base);
    });
}
