// decode.cu — single-query (decode) attention over a KV cache.
//
// Reference: shaders/single_query_attention.comp:27-71 (one query, one head,
// max 160 positions, max dim 64; lane 0 does the softmax and the whole PV
// product serially; the shader has no host wrapper in evk_ai.cpp).
// Semantics kept: o = softmax(q . K^T * scale) V over the first cur_len cached
// positions, fp32 arithmetic, scale 1/sqrt(Dh) by default, 0 when the weight
// sum is 0.
//
// Here, split-KV flash-decode: grid (splits, Hkv * head_groups, B).  A CTA
// takes one KV head g, up to 8 of the query heads that read it (GQA/MQA read
// the cache once for all of them) and one contiguous range of positions.
// LPK lanes cooperate on one cached row (16 bytes each, so a row is read as
// whole 32-byte sectors); each lane group keeps its own online-softmax state
// for its rows; groups and warps merge through shuffles and shared memory;
// per-split partials (m, l, o[Dh]) go to scratch and the last CTA of each
// (b, g, head group) merges the splits and writes the output.  The roofline is
// the KV-cache read: B * cur_len * Hkv * Dh * 2 bytes * 2 (K and V).
#include <float.h>

#include <algorithm>

#include "common.cuh"

namespace evkcu {
namespace {

constexpr int kDecThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per CTA

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// partial layout per (b, h, split): m, l, o[Dh]  (fp32)
template <typename T, int LPK, int G>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, T* __restrict__ out, uint32_t H,
    uint32_t Hkv, uint32_t Dh, uint32_t max_len, uint32_t cur_len, const uint32_t* __restrict__ d_cur_len,
    uint32_t chunk, float scale_log2,
    float* __restrict__ partial, unsigned int* __restrict__ tickets) {
    constexpr int KPW = 32 / LPK;  // rows per warp iteration
    constexpr int NW = kDecThreads / 32;
    __shared__ float sm_m[NW][G], sm_l[NW][G];
    __shared__ float sm_o[NW][G][LPK * 8];
    __shared__ bool is_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane % LPK;   // which 8-element slice of the row
    const int grp = lane / LPK;   // which row of the warp iteration
    const uint32_t split = blockIdx.x, nsplit = gridDim.x;
    const uint32_t Gq = H / Hkv;
    const uint32_t hgroups = (Gq + G - 1) / G;
    const uint32_t g = blockIdx.y / hgroups;
    const uint32_t hg = blockIdx.y % hgroups;
    const uint32_t h0 = g * Gq + hg * G;
    const uint32_t nh = min((uint32_t)G, Gq - hg * G);
    const uint32_t b = blockIdx.z;
    const uint32_t d0 = sub * 8;
    const bool dvalid = d0 < Dh;

    float qf[G][8];
#pragma unroll
    for (int i = 0; i < G; ++i) {
        if (i < (int)nh && dvalid) {
            unpack8<T>(*reinterpret_cast<const Vec8*>(q + ((uint64_t)b * H + h0 + i) * Dh + d0), qf[i]);
#pragma unroll
            for (int e = 0; e < 8; ++e) qf[i][e] *= scale_log2;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) qf[i][e] = 0.0f;
        }
    }
    float m[G], l[G], o[G][8];
#pragma unroll
    for (int i = 0; i < G; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[i][e] = 0.0f;
    }
    const uint32_t pbeg = split * chunk;
    // With d_cur_len the length lives in device memory (the grid was sized for
    // max_len), so a captured graph can replay with a growing cache.
    const uint32_t len = d_cur_len ? min(*d_cur_len, max_len) : cur_len;
    const uint32_t pend = min(pbeg + chunk, len);
    const uint64_t row_pitch = (uint64_t)Hkv * Dh;
    const T* kbase = kc + (uint64_t)b * max_len * row_pitch + (uint64_t)g * Dh + d0;
    const T* vbase = vc + (uint64_t)b * max_len * row_pitch + (uint64_t)g * Dh + d0;
    // Each lane group loads U cached rows (K and V, 16 bytes per lane each)
    // before consuming them, so 2*U loads per lane are in flight.
    constexpr int U = 4;
    for (uint32_t p0 = pbeg + warp * KPW * U; p0 < pend; p0 += NW * KPW * U) {
        float kf[U][8], vf[U][8];
        bool valid[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t pos = p0 + u * KPW + grp;
            valid[u] = pos < pend;
            if (valid[u] && dvalid) {
                unpack8<T>(*reinterpret_cast<const Vec8*>(kbase + (uint64_t)pos * row_pitch), kf[u]);
                unpack8<T>(*reinterpret_cast<const Vec8*>(vbase + (uint64_t)pos * row_pitch), vf[u]);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) kf[u][e] = vf[u][e] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int i = 0; i < G; ++i) {
                if (i >= (int)nh) break;
                float sdot = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) sdot = fmaf(qf[i][e], kf[u][e], sdot);
#pragma unroll
                for (int off = LPK / 2; off > 0; off >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, off);
                if (valid[u]) {
                    const float mn = fmaxf(m[i], sdot);
                    const float a = ex2f(m[i] - mn);
                    const float p = ex2f(sdot - mn);
                    l[i] = l[i] * a + p;
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[i][e] = fmaf(o[i][e], a, p * vf[u][e]);
                    m[i] = mn;
                }
            }
        }
    }
    // Merge the KPW row groups of the warp (lanes with equal `sub`).
#pragma unroll
    for (int i = 0; i < G; ++i) {
        if (i >= (int)nh) break;
#pragma unroll
        for (int off = LPK; off < 32; off <<= 1) {
            float m2 = __shfl_xor_sync(0xffffffffu, m[i], off);
            float l2 = __shfl_xor_sync(0xffffffffu, l[i], off);
            float mn = fmaxf(m[i], m2);
            float a = mn == -INFINITY ? 0.0f : ex2f(m[i] - mn);
            float a2 = mn == -INFINITY ? 0.0f : ex2f(m2 - mn);
            l[i] = l[i] * a + l2 * a2;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float o2 = __shfl_xor_sync(0xffffffffu, o[i][e], off);
                o[i][e] = o[i][e] * a + o2 * a2;
            }
            m[i] = mn;
        }
        if (grp == 0) {
            if (sub == 0) {
                sm_m[warp][i] = m[i];
                sm_l[warp][i] = l[i];
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) sm_o[warp][i][d0 + e] = o[i][e];
        }
    }
    __syncthreads();
    // Merge the warps: thread t handles (head i, element d) pairs.
    const uint32_t ncell = nh * Dh;
    float* pbase = partial + (((uint64_t)b * H + h0) * nsplit) * (Dh + 2);
    for (uint32_t c = threadIdx.x; c < ncell + nh; c += blockDim.x) {
        const bool is_ml = c >= ncell;
        const uint32_t i = is_ml ? c - ncell : c / Dh;
        const uint32_t d = is_ml ? 0 : c % Dh;
        float mm = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) mm = fmaxf(mm, sm_m[w][i]);
        float acc = 0.0f, ll = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            float a = mm == -INFINITY ? 0.0f : ex2f(sm_m[w][i] - mm);
            ll += sm_l[w][i] * a;
            if (!is_ml) acc += sm_o[w][i][d] * a;
        }
        float* pr = pbase + ((uint64_t)i * nsplit + split) * (Dh + 2);
        if (is_ml) {
            pr[0] = mm;
            pr[1] = ll;
        } else {
            pr[2 + d] = acc;
        }
    }
    __threadfence();
    __syncthreads();
    const uint32_t tk = (b * gridDim.y + blockIdx.y);
    if (threadIdx.x == 0) is_last = atomicAdd(&tickets[tk], 1u) == nsplit - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Merge the splits and write o / l.
    for (uint32_t c = threadIdx.x; c < ncell; c += blockDim.x) {
        const uint32_t i = c / Dh, d = c % Dh;
        const volatile float* pr = pbase + (uint64_t)i * nsplit * (Dh + 2);
        float mm = -INFINITY;
        for (uint32_t s = 0; s < nsplit; ++s) mm = fmaxf(mm, pr[s * (Dh + 2)]);
        float ll = 0.0f, acc = 0.0f;
        for (uint32_t s = 0; s < nsplit; ++s) {
            float ms = pr[s * (Dh + 2)];
            float a = mm == -INFINITY ? 0.0f : ex2f(ms - mm);
            ll += pr[s * (Dh + 2) + 1] * a;
            acc += pr[s * (Dh + 2) + 2 + d] * a;
        }
        float v = ll > 0.0f ? acc / ll : 0.0f;
        out[((uint64_t)b * H + h0 + i) * Dh + d] = Elem<T>::from_f(v);
    }
    if (threadIdx.x == 0) tickets[tk] = 0u;
}

template <typename T, int LPK>
int launch_decode(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t H, uint32_t Hkv,
                  uint32_t Dh, uint32_t max_len, uint32_t cur_len, const uint32_t* d_cur_len, float scale_log2,
                  cudaStream_t st) {
    DeviceState* ds = state();
    const uint32_t Gq = H / Hkv;
    const uint32_t hgroups = (Gq + kMaxGroup - 1) / kMaxGroup;  // same grouping for G = 1 (Gq = 1)
    const uint64_t ctas_wo_split = (uint64_t)B * Hkv * hgroups;
    // Split positions so that the grid covers ~4 CTAs per SM, at least 64 rows each.
    uint64_t want = std::max<uint64_t>(1, (4ull * ds->sm_count + ctas_wo_split - 1) / ctas_wo_split);
    uint32_t chunk = (uint32_t)std::max<uint64_t>(64, (cur_len + want - 1) / want);
    chunk = (chunk + 31) / 32 * 32;
    const uint32_t nsplit = (cur_len + chunk - 1) / chunk;
    const size_t pbytes = (size_t)B * H * nsplit * (Dh + 2) * sizeof(float);
    if (ctas_wo_split > kMaxTickets) return fail(EVKCU_BAD_SHAPE, "evkcu_single_query_attention: B*Hkv too large");
    const size_t toff = kTicketBytes;
    char* ws = (char*)workspace(WS_DECODE, toff + pbytes);
    if (!ws) return fail(EVKCU_CUDA_ERROR, "evkcu_single_query_attention: scratch allocation failed");
    dim3 grid(nsplit, Hkv * hgroups, B);
    // MHA (one query head per cached head) needs no head group registers.
    if (Gq == 1)
        decode_attn_kernel<T, LPK, 1><<<grid, kDecThreads, 0, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, H,
                                                                   Hkv, Dh, max_len, cur_len, d_cur_len, chunk,
                                                                   scale_log2, (float*)(ws + toff), (unsigned int*)ws);
    else
        decode_attn_kernel<T, LPK, kMaxGroup><<<grid, kDecThreads, 0, st>>>(
            (const T*)q, (const T*)k, (const T*)v, (T*)o, H, Hkv, Dh, max_len, cur_len, d_cur_len, chunk, scale_log2,
            (float*)(ws + toff), (unsigned int*)ws);
    return after_launch("evkcu_single_query_attention");
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_single_query_attention(const void* q, const void* kcache, const void* vcache, void* out,
                                            uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t max_len,
                                            uint32_t cur_len, float scale, int dtype, void* stream) {
    if (B == 0 || H == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(q && kcache && vcache && out, EVKCU_BAD_ARG, "evkcu_single_query_attention: null pointer");
    EVKCU_CHECK_ARG(Hkv >= 1 && H % Hkv == 0, EVKCU_BAD_SHAPE, "evkcu_single_query_attention: H % Hkv != 0");
    EVKCU_CHECK_ARG(Dh % 8 == 0 && Dh >= 8 && Dh <= 256, EVKCU_BAD_SHAPE,
                    "evkcu_single_query_attention: Dh must be a multiple of 8 in [8, 256]");
    EVKCU_CHECK_ARG(cur_len <= max_len, EVKCU_BAD_SHAPE, "evkcu_single_query_attention: cur_len > max_len");
    EVKCU_CHECK_ARG(aligned16(q) && aligned16(kcache) && aligned16(vcache) && aligned16(out), EVKCU_BAD_ALIGN,
                    "evkcu_single_query_attention: pointers must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    if (cur_len == 0) {
        // No cached positions: every weight is zero, the output is zero.
        EVKCU_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)B * H * Dh * 2, st));
        return EVKCU_OK;
    }
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)Dh);
    const float sl2 = scale * 1.4426950408889634f;
    const uint32_t slices = Dh / 8;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (slices <= 2) return launch_decode<T, 2>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, cur_len, nullptr, sl2, st);
        if (slices <= 4) return launch_decode<T, 4>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, cur_len, nullptr, sl2, st);
        if (slices <= 8) return launch_decode<T, 8>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, cur_len, nullptr, sl2, st);
        if (slices <= 16) return launch_decode<T, 16>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, cur_len, nullptr, sl2, st);
        return launch_decode<T, 32>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, cur_len, nullptr, sl2, st);
    });
}

extern "C" int evkcu_single_query_attention_devlen(const void* q, const void* kcache, const void* vcache, void* out,
                                                   uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh,
                                                   uint32_t max_len, const uint32_t* d_cur_len, float scale, int dtype,
                                                   void* stream) {
    if (B == 0 || H == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(q && kcache && vcache && out && d_cur_len, EVKCU_BAD_ARG,
                    "evkcu_single_query_attention_devlen: null pointer");
    EVKCU_CHECK_ARG(Hkv >= 1 && H % Hkv == 0, EVKCU_BAD_SHAPE, "evkcu_single_query_attention_devlen: H % Hkv != 0");
    EVKCU_CHECK_ARG(Dh % 8 == 0 && Dh >= 8 && Dh <= 256 && max_len > 0, EVKCU_BAD_SHAPE,
                    "evkcu_single_query_attention_devlen: Dh must be a multiple of 8 in [8, 256], max_len > 0");
    EVKCU_CHECK_ARG(aligned16(q) && aligned16(kcache) && aligned16(vcache) && aligned16(out), EVKCU_BAD_ALIGN,
                    "evkcu_single_query_attention_devlen: pointers must be 16-byte aligned");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)Dh);
    const float sl2 = scale * 1.4426950408889634f;
    const uint32_t slices = Dh / 8;
    cudaStream_t st = as_stream(stream);
    const uint32_t* dl = d_cur_len;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (slices <= 2) return launch_decode<T, 2>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, max_len, dl, sl2, st);
        if (slices <= 4) return launch_decode<T, 4>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, max_len, dl, sl2, st);
        if (slices <= 8) return launch_decode<T, 8>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, max_len, dl, sl2, st);
        if (slices <= 16) return launch_decode<T, 16>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, max_len, dl, sl2, st);
        return launch_decode<T, 32>(q, kcache, vcache, out, B, H, Hkv, Dh, max_len, max_len, dl, sl2, st);
    });
}
