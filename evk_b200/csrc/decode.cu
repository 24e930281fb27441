// decode.cu — single-query (decode) attention over a KV cache.
//
// Reference: shaders/single_query_attention.comp:27-71 (one query, one head,
// max 160 positions, max dim 64; lane 0 does the softmax and the whole PV
// product serially; the shader has no host wrapper in evk_ai.cpp).
// Semantics kept: o = softmax(q . K^T * scale) V over the first cur_len cached
// positions, fp32 arithmetic, scale 1/sqrt(Dh) by default, 0 when the weight
// sum is 0.
//
// Here, split-KV flash-decode: grid (splits, Hkv * head_groups, B), one
// resident wave.  A CTA takes one KV head g, up to 8 of the query heads that
// read it (GQA/MQA read the cache once for all of them) and one contiguous
// range of positions.  A producer warp streams the range through a
// shared-memory ring as ROWS-position K and V tiles (TMA boxes of Dh x ROWS
// out of the [B * max_len, Hkv * Dh] cache, full/empty mbarriers); eight
// compute warps read them from shared memory.  LPK lanes cooperate on one
// row (16 bytes each); each lane group keeps its own online-softmax state and
// folds in STEPS rows per tile with one rescale; groups and warps merge
// through shuffles and shared memory; per-split partials (m, l, o[Dh]) go to
// scratch and the last CTA of each (b, g, head group) merges the splits in
// split order and writes the output.  The roofline is the KV-cache read:
// B * cur_len * Hkv * Dh * 2 bytes * 2 (K and V).
#include <float.h>

#include <algorithm>

#include "sm100.cuh"

namespace evkcu {
namespace {

using namespace sm100;

constexpr int kDecCompute = 8;                    // compute warps
constexpr int kDecThreads = (kDecCompute + 1) * 32;  // + the producer warp
constexpr int kMaxGroup = 8;                      // query heads per CTA
constexpr int kMaxStages = 8;
constexpr uint32_t kDecSmemTarget = 96 * 1024;    // ring bytes: two CTAs per SM
constexpr uint32_t kTimeoutDecode = 0x401;

// 16-byte shared-memory load (one LDS.128; a warp reading 512 contiguous
// bytes then takes the minimum 4 wavefronts).
__device__ __forceinline__ Vec8 ld_shared_v4(const void* p) {
    Vec8 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
    return v;
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Tile geometry for LPK lanes per cached row.
template <int LPK>
struct DecTile {
    static constexpr int KPW = 32 / LPK;                                   // rows per warp step
    static constexpr int ROWS = KPW * kDecCompute > 64 ? KPW * kDecCompute : 64;  // positions per tile
    static constexpr int STEPS = ROWS / (KPW * kDecCompute);               // steps per warp per tile
};

// partial layout per (b, h, split): m, l, o[Dh]  (fp32)
template <typename T, int LPK, int G>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const T* __restrict__ q,
    T* __restrict__ out, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t max_len, uint32_t cur_len,
    const uint32_t* __restrict__ d_cur_len, uint32_t chunk, float scale_log2, uint32_t stages,
    float* __restrict__ partial, unsigned int* __restrict__ tickets, unsigned int* err) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    constexpr int KPW = DecTile<LPK>::KPW, ROWS = DecTile<LPK>::ROWS, STEPS = DecTile<LPK>::STEPS;
    constexpr int NW = kDecCompute;
    __shared__ float sm_m[NW][G], sm_l[NW][G];
    __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ int s_abort_v;
    __shared__ bool is_last;
    // stages x (K tile, V tile); reused for the warps' o partials at the end.
    extern __shared__ __align__(128) uint8_t ring[];
    float (*sm_o)[G][LPK * 8] = reinterpret_cast<float (*)[G][LPK * 8]>(ring);
    volatile int* s_abort = &s_abort_v;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane % LPK;   // which 8-element slice of the row
    const int grp = lane / LPK;   // which row of the warp step
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
    const uint32_t tile_elems = ROWS * Dh;

    const uint32_t pbeg = split * chunk;
    // With d_cur_len the length lives in device memory (the grid was sized for
    // max_len), so a captured graph can replay with a growing cache.
    const uint32_t len = d_cur_len ? min(*d_cur_len, max_len) : cur_len;
    const uint32_t pend = min(pbeg + chunk, len);
    const uint32_t ntiles = pend > pbeg ? (pend - pbeg + ROWS - 1) / ROWS : 0;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        *s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    float m[G], l[G], o[G][8];
#pragma unroll
    for (int i = 0; i < G; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[i][e] = 0.0f;
    }

    if (warp == NW) {
        // Producer: one lane streams the K/V tiles of [pbeg, pend).
        if (lane == 0 && ntiles > 0) {
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            const uint32_t bytes = tile_elems * 2 * sizeof(T);
            uint32_t issued = 0;
            for (uint32_t t = 0; t < ntiles; ++t) {
                const uint32_t s = t % stages;
                if (!mbar_wait(&empty[s], ((t / stages) & 1) ^ 1, s_abort, err, kTimeoutDecode)) break;
                mbar_arrive_expect_tx(&full[s], bytes);
                T* kt = reinterpret_cast<T*>(ring) + (size_t)s * 2 * tile_elems;
                const int y = (int)((uint64_t)b * max_len + pbeg + t * ROWS);
                tma_load_3d(kt, &tmK, &full[s], (int)(g * Dh), y, 0);
                tma_load_3d(kt + tile_elems, &tmV, &full[s], (int)(g * Dh), y, 0);
                issued = t + 1;
            }
            if (*s_abort) {
                // Let the copies still in flight land before the CTA exits.
                const uint32_t first = issued > stages ? issued - stages : 0;
                for (uint32_t t = first; t < issued; ++t) mbar_drain(&full[t % stages], (t / stages) & 1);
            }
        }
    } else {
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
        for (uint32_t t = 0; t < ntiles; ++t) {
            const uint32_t s = t % stages;
            // Lane 0 waits (one poller per warp keeps the barrier word from
            // serialising 256 pollers); the warp follows its outcome.
            const int ok = __shfl_sync(0xffffffffu,
                                       lane == 0 ? (int)mbar_wait(&full[s], (t / stages) & 1, s_abort, err,
                                                                  kTimeoutDecode)
                                                 : 0,
                                       0);
            if (!ok) break;
            const T* kt = reinterpret_cast<const T*>(ring) + (size_t)s * 2 * tile_elems;
            const T* vt = kt + tile_elems;
            const uint32_t r0 = warp * (KPW * STEPS) + grp;   // this lane group's first row
            const uint32_t pos0 = pbeg + t * ROWS + r0;
            // Rows are folded in blocks of SB steps, one rescale per block
            // (SB < STEPS bounds the registers when many heads share the CTA).
            constexpr int SB = (G >= 4 && STEPS > 2) ? 2 : STEPS;
#pragma unroll
            for (int jb = 0; jb < STEPS; jb += SB) {
                float sd[SB][G];
#pragma unroll
                for (int j = 0; j < SB; ++j) {
                    float kf[8];
                    if (dvalid) {
                        unpack8<T>(ld_shared_v4(kt + (r0 + (jb + j) * KPW) * Dh + d0), kf);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) kf[e] = 0.0f;
                    }
#pragma unroll
                    for (int i = 0; i < G; ++i) {
                        float d = 0.0f;
#pragma unroll
                        for (int e = 0; e < 8; ++e) d = fmaf(qf[i][e], kf[e], d);
                        sd[j][i] = d;
                    }
                }
#pragma unroll
                for (int off = LPK / 2; off > 0; off >>= 1)
#pragma unroll
                    for (int j = 0; j < SB; ++j)
#pragma unroll
                        for (int i = 0; i < G; ++i) sd[j][i] += __shfl_xor_sync(0xffffffffu, sd[j][i], off);
#pragma unroll
                for (int i = 0; i < G; ++i) {
                    float mx = -INFINITY;
#pragma unroll
                    for (int j = 0; j < SB; ++j)
                        if (pos0 + (jb + j) * KPW < pend) mx = fmaxf(mx, sd[j][i]);
                    const float mn = fmaxf(m[i], mx);
                    const float a = mn == -INFINITY ? 1.0f : ex2f(m[i] - mn);
                    float ps = 0.0f;
#pragma unroll
                    for (int j = 0; j < SB; ++j) {
                        sd[j][i] = (pos0 + (jb + j) * KPW < pend) ? ex2f(sd[j][i] - mn) : 0.0f;
                        ps += sd[j][i];
                    }
                    l[i] = l[i] * a + ps;
                    m[i] = mn;
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[i][e] *= a;
                }
#pragma unroll
                for (int j = 0; j < SB; ++j) {
                    float vf[8];
                    // Rows at or past the length hold whatever the cache (or
                    // the next sequence) has there: their weight is 0, and
                    // their values must not enter o (0 * NaN = NaN).
                    if (dvalid && pos0 + (jb + j) * KPW < pend) {
                        unpack8<T>(ld_shared_v4(vt + (r0 + (jb + j) * KPW) * Dh + d0), vf);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) vf[e] = 0.0f;
                    }
#pragma unroll
                    for (int i = 0; i < G; ++i)
#pragma unroll
                        for (int e = 0; e < 8; ++e) o[i][e] = fmaf(sd[j][i], vf[e], o[i][e]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
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
        }
    }
    // All tiles are consumed (or the CTA gave up and the producer drained its
    // copies): the ring now holds the warps' o partials.
    __syncthreads();
    if (warp < NW && grp == 0) {
#pragma unroll
        for (int i = 0; i < G; ++i) {
            if (i >= (int)nh) break;
            if (sub == 0) {
                sm_m[warp][i] = m[i];
                sm_l[warp][i] = l[i];
            }
            if (dvalid) {
#pragma unroll
                for (int e = 0; e < 8; ++e) sm_o[warp][i][d0 + e] = o[i][e];
            }
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
        // Partials come from other CTAs: read them from L2 (.cg), eight
        // splits per batch so the loads overlap; merge in split order.
        const float* pr = pbase + (uint64_t)i * nsplit * (Dh + 2);
        float mm = -INFINITY;
        for (uint32_t s0 = 0; s0 < nsplit; s0 += 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < nsplit) mm = fmaxf(mm, __ldcg(pr + (s0 + j) * (Dh + 2)));
        }
        float ll = 0.0f, acc = 0.0f;
        for (uint32_t s0 = 0; s0 < nsplit; s0 += 8) {
            float ms[8], ls[8], os[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool in = s0 + j < nsplit;
                const float* p = pr + (s0 + j) * (Dh + 2);
                ms[j] = in ? __ldcg(p) : -INFINITY;
                ls[j] = in ? __ldcg(p + 1) : 0.0f;
                os[j] = in ? __ldcg(p + 2 + d) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (s0 + j < nsplit) {
                    const float a = mm == -INFINITY ? 0.0f : ex2f(ms[j] - mm);
                    ll += ls[j] * a;
                    acc += os[j] * a;
                }
            }
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
    constexpr int ROWS = DecTile<LPK>::ROWS;
    DeviceState* ds = state();
    const uint32_t Gq = H / Hkv;
    const uint32_t hgroups = (Gq + kMaxGroup - 1) / kMaxGroup;  // same grouping for G = 1 (Gq = 1)
    const uint64_t ctas_wo_split = (uint64_t)B * Hkv * hgroups;
    if (ctas_wo_split > kMaxTickets) return fail(EVKCU_BAD_SHAPE, "evkcu_single_query_attention: B*Hkv too large");
    auto kern = Gq == 1 ? decode_attn_kernel<T, LPK, 1> : decode_attn_kernel<T, LPK, kMaxGroup>;
    // Ring: as many K/V tile pairs as fit the per-CTA target (at least 2);
    // where registers allow only one CTA per SM, a deeper ring instead.
    const uint32_t stage_bytes = 2u * ROWS * Dh * 2;
    const uint32_t obytes = (uint32_t)(kDecCompute * (Gq == 1 ? 1 : kMaxGroup) * LPK * 8 * sizeof(float));
    auto ring_bytes = [&](uint32_t target, uint32_t* stages) {
        *stages = std::max<uint32_t>(2, std::min<uint32_t>(kMaxStages, target / stage_bytes));
        return std::max(*stages * stage_bytes, obytes);
    };
    uint32_t stages = 0;
    uint32_t smem = ring_bytes(kDecSmemTarget, &stages);
    // Per kernel variant: the attribute once, the occupancy per ring size.
    static bool attr_set[2] = {false, false};
    static uint32_t occ_smem[2] = {0, 0};
    static int occ_blocks[2] = {0, 0};
    const int vi = Gq == 1 ? 0 : 1;
    if (!attr_set[vi]) {
        EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set[vi] = true;
    }
    if (occ_smem[vi] != smem) {
        EVKCU_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_blocks[vi], kern, kDecThreads, smem));
        occ_smem[vi] = smem;
    }
    int per_sm = occ_blocks[vi];
    if (per_sm <= 1) {
        smem = ring_bytes(192 * 1024, &stages);
        per_sm = 1;
    }
    // One resident wave: split positions over the CTA slots left per (b, g, head group).
    const uint64_t slots = (uint64_t)per_sm * ds->sm_count;
    uint64_t want = std::max<uint64_t>(1, slots / ctas_wo_split);
    static const int forced_splits = [] {
        const char* e = getenv("EVKCU_DECODE_SPLITS");
        return e ? atoi(e) : 0;
    }();
    if (forced_splits > 0) want = (uint64_t)forced_splits;
    uint32_t chunk = (uint32_t)std::max<uint64_t>(ROWS, (cur_len + want - 1) / want);
    chunk = (chunk + ROWS - 1) / ROWS * ROWS;
    const uint32_t nsplit = (cur_len + chunk - 1) / chunk;
    const size_t pbytes = (size_t)B * H * nsplit * (Dh + 2) * sizeof(float);
    char* ws = (char*)workspace(WS_DECODE, kTicketBytes + pbytes);
    if (!ws) return fail(EVKCU_CUDA_ERROR, "evkcu_single_query_attention: scratch allocation failed");
    // The caches as [B * max_len rows, Hkv * Dh] matrices; a box is Dh x ROWS.
    CUtensorMap mK, mV;
    const uint64_t pitch = (uint64_t)Hkv * Dh, rows = (uint64_t)B * max_len;
    const int dt = std::is_same<T, __nv_bfloat16>::value ? EVKCU_BF16 : EVKCU_F16;
    int r = make_tmap_3d(&mK, k, pitch, rows, 1, pitch, pitch * rows, Dh, ROWS, dt, false);
    if (r) return r;
    r = make_tmap_3d(&mV, v, pitch, rows, 1, pitch, pitch * rows, Dh, ROWS, dt, false);
    if (r) return r;
    dim3 grid(nsplit, Hkv * hgroups, B);
    return launch_pdl("evkcu_single_query_attention", kern, grid, kDecThreads, smem, st, mK, mV, (const T*)q, (T*)o, H,
                      Hkv, Dh, max_len, cur_len, d_cur_len, chunk, scale_log2, stages, (float*)(ws + kTicketBytes),
                      (unsigned int*)ws, ds->d_error);
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
