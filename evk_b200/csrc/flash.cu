// flash.cu — evk::ai::flash_attention forward on sm_100a.
//
// Reference: evk_ai.cpp:332-369 (host), shaders/flash_attention.comp:53-185.
// The reference runs one 32-lane subgroup per 16 queries with 16x16 fp16
// cooperative-matrix tiles, a serial per-row softmax loop and the online
// rescale done as an extra diagonal-matrix MMA.  Semantics kept here:
// O = softmax(Q K^T * scale) V per head with exp2-form online softmax, rows
// with a zero denominator produce 0, Q/O laid out [B, N, H*Dh] and K/V
// [B, N, Hkv*Dh] (the reference call is Hkv = 1, non-causal).
//
// tcgen05 kernel (Dh = 64 or 128), one CTA per (128-query tile, head, batch):
//   warp 0   TMA producer: Q once, then K_j / V_j 128-key blocks into a
//            STAGES-deep ring (separate K and V barriers).
//   warp 1   TMEM owner + MMA issuer:  S_j = Q K_j^T  (M=128,N=128,K=Dh) into
//            one of two TMEM S buffers, then PV_{j-1} = P_{j-1} V_{j-1}
//            (M=128, N=Dh, K=128) into one of two TMEM PV buffers, so the
//            tensor core computes S_{j+1} while the softmax warps work on S_j.
//   warps 2-5 softmax, one thread per query row (its TMEM lane): row max and
//            exp2 over S_j, P_j -> shared memory (fp16/bf16, 128-byte swizzled
//            K-major, the A operand of the PV MMA), then O = O*alpha + PV in
//            fp32 registers; final 1/l and 16-byte stores.
// Causal tiles stop at the diagonal block; only diagonal / ragged blocks
// evaluate the mask.
//
// Any other Dh (multiple of 16, <= 256) runs a CUDA-core kernel (one warp per
// query row) with the same semantics.
#include <float.h>

#include <algorithm>

#include "sm100.cuh"

namespace evkcu {
namespace {

using namespace sm100;

constexpr int FM = 128;  // queries per CTA
constexpr int FN = 128;  // keys per block
constexpr int kFlashThreads = 192;
constexpr uint32_t kTimeoutFlash = 0x201;

template <int DH>
struct FlashCfg {
    static constexpr int Q_BYTES = FM * DH * 2;
    static constexpr int K_BYTES = FN * DH * 2;
    static constexpr int V_BYTES = FN * DH * 2;
    static constexpr int P_BYTES = FM * FN * 2;  // one P buffer
    static constexpr int STAGES = DH == 64 ? 3 : 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_P = OFF_Q + Q_BYTES;
    static constexpr int OFF_K = OFF_P + 2 * P_BYTES;
    static constexpr int OFF_V = OFF_K + STAGES * K_BYTES;
    static constexpr int OFF_BAR = OFF_V + STAGES * V_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t COL_S = 0;        // two S buffers: 0, 128
    static constexpr uint32_t COL_PV = 2 * FN;  // two PV buffers: 256, 256 + DH
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <typename T, int DH>
__global__ void __launch_bounds__(kFlashThreads, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, T* __restrict__ O, uint32_t N, uint32_t H,
                    uint32_t Hkv, float scale_log2, int causal, uint32_t idesc_s, uint32_t idesc_pv,
                    unsigned int* err) {
    using Cfg = FlashCfg<DH>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Cfg::OFF_Q;
    uint8_t* sP = smem + Cfg::OFF_P;
    uint8_t* sK = smem + Cfg::OFF_K;
    uint8_t* sV = smem + Cfg::OFF_V;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;               // [STAGES]
    uint64_t* v_full = k_full + STAGES;        // [STAGES]
    uint64_t* kv_empty = v_full + STAGES;      // [STAGES]
    uint64_t* s_full = kv_empty + STAGES;      // [2]
    uint64_t* s_free = s_full + 2;             // [2]
    uint64_t* p_full = s_free + 2;             // [2]
    uint64_t* pv_full = p_full + 2;            // [2]
    uint64_t* pv_free = pv_full + 2;           // [2]
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(pv_free + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bh = blockIdx.x;
    const uint32_t b = bh / H, h = bh % H;
    const uint32_t g = h / (H / Hkv);
    const uint32_t num_qt = gridDim.y;
    const uint32_t qt = num_qt - 1 - blockIdx.y;  // heaviest causal tiles first
    const uint32_t q0 = qt * FM;
    const uint32_t kv_blocks_all = (N + FN - 1) / FN;
    const uint32_t nblk = causal ? min(kv_blocks_all, (q0 + FM + FN - 1) / FN) : kv_blocks_all;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_full[i], 1);
            mbar_init(&pv_free[i], 4);
        }
        *s_abort = 0;
        fence_barrier_init();
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(s_tmem, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer ----
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
#pragma unroll
            for (int c = 0; c < DH / 64; ++c)
                tma_load_3d(sQ + c * FM * 128, &tmQ, q_full, (int)(h * DH + c * 64), (int)q0, (int)b);
            for (uint32_t j = 0; j < nblk; ++j) {
                const int st = j % STAGES;
                const uint32_t ph = (j / STAGES) & 1;
                if (!mbar_wait(&kv_empty[st], ph ^ 1, s_abort, err, kTimeoutFlash)) break;
                mbar_arrive_expect_tx(&k_full[st], Cfg::K_BYTES);
#pragma unroll
                for (int c = 0; c < DH / 64; ++c)
                    tma_load_3d(sK + st * Cfg::K_BYTES + c * FN * 128, &tmK, &k_full[st], (int)(g * DH + c * 64),
                                (int)(j * FN), (int)b);
                mbar_arrive_expect_tx(&v_full[st], Cfg::V_BYTES);
#pragma unroll
                for (int c = 0; c < DH / 64; ++c)
                    tma_load_3d(sV + st * Cfg::V_BYTES + c * FN * 128, &tmV, &v_full[st], (int)(g * DH + c * 64),
                                (int)(j * FN), (int)b);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA issuer ----
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0, s_abort, err, kTimeoutFlash);
            tc_fence_after();
            const uint32_t qaddr = smem_u32(sQ);
            auto issue_pv = [&](uint32_t jj) -> bool {
                const int st = jj % STAGES;
                const int pb = jj & 1;
                if (!mbar_wait(&p_full[pb], (jj >> 1) & 1, s_abort, err, kTimeoutFlash)) return false;
                if (!mbar_wait(&pv_free[pb], ((jj >> 1) & 1) ^ 1, s_abort, err, kTimeoutFlash)) return false;
                if (!mbar_wait(&v_full[st], (jj / STAGES) & 1, s_abort, err, kTimeoutFlash)) return false;
                tc_fence_after();
                const uint32_t paddr = smem_u32(sP + pb * Cfg::P_BYTES);
                const uint32_t vaddr = smem_u32(sV + st * Cfg::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < FN / 16; ++kk) {
                    uint64_t ad = make_sw128_desc(paddr + (kk >> 2) * (FM * 128) + (kk & 3) * 32, 16, 1024);
                    uint64_t bd = make_sw128_desc(vaddr + kk * 2048, FN * 128, 1024);
                    mma_f16_ss(tmem + Cfg::COL_PV + pb * DH, ad, bd, idesc_pv, kk != 0);
                }
                mma_commit(&pv_full[pb]);
                mma_commit(&kv_empty[st]);
                return true;
            };
            for (uint32_t j = 0; ok && j < nblk; ++j) {
                const int st = j % STAGES;
                const int sb = j & 1;
                if (!mbar_wait(&k_full[st], (j / STAGES) & 1, s_abort, err, kTimeoutFlash)) break;
                if (!mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, s_abort, err, kTimeoutFlash)) break;
                tc_fence_after();
                const uint32_t kaddr = smem_u32(sK + st * Cfg::K_BYTES);
#pragma unroll
                for (int kk = 0; kk < DH / 16; ++kk) {
                    uint64_t ad = make_sw128_desc(qaddr + (kk >> 2) * (FM * 128) + (kk & 3) * 32, 16, 1024);
                    uint64_t bd = make_sw128_desc(kaddr + (kk >> 2) * (FN * 128) + (kk & 3) * 32, 16, 1024);
                    mma_f16_ss(tmem + Cfg::COL_S + sb * FN, ad, bd, idesc_s, kk != 0);
                }
                mma_commit(&s_full[sb]);
                if (j >= 1 && !issue_pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && nblk > 0) issue_pv(nblk - 1);
        }
    } else {
        // --------------------------------------------- softmax warps ----
        const int quarter = warp & 3;
        const uint32_t row = quarter * 32 + lane;  // TMEM lane == query row in tile
        const uint32_t qidx = q0 + row;
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        float o[DH];
#pragma unroll
        for (int d = 0; d < DH; ++d) o[d] = 0.0f;
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (uint32_t j = 0; j < nblk; ++j) {
            const int sb = j & 1;
            if (!mbar_wait(&s_full[sb], (j >> 1) & 1, s_abort, err, kTimeoutFlash)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t k0 = j * FN;
            const bool need_mask = (k0 + FN > N) || (causal && k0 + FN > q0 + 1);
            // A key is valid when it exists and (non-causal or key <= query).
            const uint32_t kmax = min(N, causal ? qidx + 1 : N);  // keys < kmax are valid
            const uint32_t s_addr = lane_addr + Cfg::COL_S + sb * FN;
            // pass 1: row max of the scaled scores
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < FN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(s_addr + c * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    float v = __uint_as_float(r[e]);
                    if (need_mask && k0 + c * 32 + e >= kmax) v = -INFINITY;
                    mx = fmaxf(mx, v);
                }
            }
            const float m_new = fmaxf(m, mx * scale_log2);
            const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
            const float alpha = ex2(m - m_use);  // m = -inf -> 0
            // pass 2: p = exp2(s*scale_log2 - m), row sum, P -> shared memory
            float rs = 0.0f;
            uint8_t* prow = sP + sb * Cfg::P_BYTES + row * 128;
#pragma unroll
            for (int c = 0; c < FN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(s_addr + c * 32, r);
                tmem_wait_ld();
                float p[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    float v = __uint_as_float(r[e]);
                    float pe = ex2(fmaf(v, scale_log2, -m_use));
                    if (need_mask && k0 + c * 32 + e >= kmax) pe = 0.0f;
                    p[e] = pe;
                    rs += pe;
                }
                // 32 keys = 4 16-byte chunks; key block (c*32)/64, chunk index within the 128-byte row.
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int key = c * 32 + q * 8;
                    const int blk = key >> 6;
                    const int chunk = (key & 63) >> 3;
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = p[q * 8 + e];
                    Vec8 v8 = pack8<T>(f);
                    *reinterpret_cast<Vec8*>(prow + blk * (FM * 128) + ((chunk ^ (row & 7)) << 4)) = v8;
                }
            }
            // S buffer consumed: release it to the MMA warp.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[sb]);
            // P written by generic stores: make it visible to the tensor core.
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);
            l = l * alpha + rs;
            m = m_new;
            // Fold in PV_{j-1} (relative to the previous max), then rescale.
            if (j >= 1) {
                const uint32_t jj = j - 1;
                const int pb = jj & 1;
                if (!mbar_wait(&pv_full[pb], (jj >> 1) & 1, s_abort, err, kTimeoutFlash)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < DH / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(lane_addr + Cfg::COL_PV + pb * DH + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[c * 32 + e] = (o[c * 32 + e] + __uint_as_float(r[e])) * alpha;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&pv_free[pb]);
            } else {
#pragma unroll
                for (int d = 0; d < DH; ++d) o[d] *= alpha;
            }
        }
        if (ok && nblk > 0) {
            const uint32_t jj = nblk - 1;
            const int pb = jj & 1;
            ok = mbar_wait(&pv_full[pb], (jj >> 1) & 1, s_abort, err, kTimeoutFlash);
            tc_fence_after();
            if (ok) {
#pragma unroll
                for (int c = 0; c < DH / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(lane_addr + Cfg::COL_PV + pb * DH + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[c * 32 + e] += __uint_as_float(r[e]);
                }
            }
            tc_fence_before();
        }
        if (ok && qidx < N) {
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            T* orow = O + ((uint64_t)b * N + qidx) * ((uint64_t)H * DH) + (uint64_t)h * DH;
#pragma unroll
            for (int c = 0; c < DH / 8; ++c) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = o[c * 8 + e] * inv;
                reinterpret_cast<Vec8*>(orow)[c] = pack8<T>(f);
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// --------------------------------------------------- CUDA-core fallback ----
// One warp per query row; lanes own Dh/32 (<= 8) of the row's elements.
template <typename T>
__global__ void __launch_bounds__(256) flash_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K,
                                                         const T* __restrict__ V, T* __restrict__ O, uint32_t B,
                                                         uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh,
                                                         float scale_log2, int causal) {
    const int lane = threadIdx.x & 31;
    const uint64_t wid = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t total = (uint64_t)B * H * N;
    if (wid >= total) return;
    const uint32_t qi = (uint32_t)(wid % N);
    const uint32_t h = (uint32_t)((wid / N) % H);
    const uint32_t b = (uint32_t)(wid / ((uint64_t)N * H));
    const uint32_t g = h / (H / Hkv);
    const uint32_t per = Dh / 32 > 0 ? (Dh + 31) / 32 : 1;
    float q[8], o[8];
    const T* qrow = Q + ((uint64_t)b * N + qi) * H * Dh + (uint64_t)h * Dh;
    for (uint32_t i = 0; i < 8; ++i) {
        uint32_t d = lane + 32 * i;
        q[i] = (i < per && d < Dh) ? Elem<T>::to_f(qrow[d]) : 0.0f;
        o[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const uint32_t kend = causal ? min(N, qi + 1) : N;
    for (uint32_t j = 0; j < kend; ++j) {
        const T* krow = K + ((uint64_t)b * N + j) * Hkv * Dh + (uint64_t)g * Dh;
        float s = 0.0f;
        for (uint32_t i = 0; i < per; ++i) {
            uint32_t d = lane + 32 * i;
            if (d < Dh) s += q[i] * Elem<T>::to_f(krow[d]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        s *= scale_log2;
        float mn = fmaxf(m, s);
        float a = ex2(m - mn);
        float p = ex2(s - mn);
        l = l * a + p;
        m = mn;
        const T* vrow = V + ((uint64_t)b * N + j) * Hkv * Dh + (uint64_t)g * Dh;
        for (uint32_t i = 0; i < per; ++i) {
            uint32_t d = lane + 32 * i;
            float vv = d < Dh ? Elem<T>::to_f(vrow[d]) : 0.0f;
            o[i] = o[i] * a + p * vv;
        }
    }
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    T* orow = O + ((uint64_t)b * N + qi) * H * Dh + (uint64_t)h * Dh;
    for (uint32_t i = 0; i < per; ++i) {
        uint32_t d = lane + 32 * i;
        if (d < Dh) orow[d] = Elem<T>::from_f(o[i] * inv);
    }
}

template <typename T, int DH>
int launch_flash_tc(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N, uint32_t H,
                    uint32_t Hkv, float scale_log2, int causal, int dtype, cudaStream_t st) {
    using Cfg = FlashCfg<DH>;
    CUtensorMap mQ, mK, mV;
    int r;
    if ((r = make_tmap_3d(&mQ, q, (uint64_t)H * DH, N, B, (uint64_t)H * DH, (uint64_t)N * H * DH, 64, FM, dtype))) return r;
    if ((r = make_tmap_3d(&mK, k, (uint64_t)Hkv * DH, N, B, (uint64_t)Hkv * DH, (uint64_t)N * Hkv * DH, 64, FN, dtype))) return r;
    if ((r = make_tmap_3d(&mV, v, (uint64_t)Hkv * DH, N, B, (uint64_t)Hkv * DH, (uint64_t)N * Hkv * DH, 64, FN, dtype))) return r;
    auto kern = flash_tc_kernel<T, DH>;
    static bool attr = false;
    if (!attr) {
        EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
        attr = true;
    }
    const int bf = dtype == EVKCU_BF16 ? 1 : 0;
    const uint32_t idesc_s = make_idesc_f16(FM, FN, bf, 0, 0);
    const uint32_t idesc_pv = make_idesc_f16(FM, DH, bf, 0, 1);
    dim3 grid(B * H, (N + FM - 1) / FM);
    kern<<<grid, kFlashThreads, Cfg::SMEM, st>>>(mQ, mK, mV, (T*)o, N, H, Hkv, scale_log2, causal, idesc_s, idesc_pv,
                                                 state()->d_error);
    return after_launch("evkcu_flash_attention(tcgen05)");
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_flash_attention(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N,
                                     uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype,
                                     void* stream) {
    if (B == 0 || N == 0 || H == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(q && k && v && o, EVKCU_BAD_ARG, "evkcu_flash_attention: null pointer");
    EVKCU_CHECK_ARG(dtype == EVKCU_F16 || dtype == EVKCU_BF16, EVKCU_BAD_ARG, "evkcu_flash_attention: unknown dtype");
    EVKCU_CHECK_ARG(Hkv >= 1 && H % Hkv == 0, EVKCU_BAD_SHAPE, "evkcu_flash_attention: H must be a multiple of Hkv");
    EVKCU_CHECK_ARG(Dh % 16 == 0 && Dh >= 16 && Dh <= 256, EVKCU_BAD_SHAPE,
                    "evkcu_flash_attention: Dh must be a multiple of 16 in [16, 256]");
    EVKCU_CHECK_ARG((uint64_t)B * H <= 0x7fffffffu && (N + FM - 1) / FM <= 65535, EVKCU_BAD_SHAPE,
                    "evkcu_flash_attention: grid too large");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)Dh);
    const float scale_log2 = scale * 1.4426950408889634f;
    const int causal = (flags & EVKCU_ATTN_CAUSAL) ? 1 : 0;
    cudaStream_t st = as_stream(stream);
    const bool tma_ok = aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
    if (tma_ok && (Dh == 64 || Dh == 128)) {
        return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
            if (Dh == 64) return launch_flash_tc<T, 64>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype, st);
            return launch_flash_tc<T, 128>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype, st);
        });
    }
    const uint64_t warps = (uint64_t)B * H * N;
    const uint64_t blocks = (warps * 32 + 255) / 256;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        flash_simt_kernel<T><<<(unsigned)blocks, 256, 0, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, B, N, H,
                                                              Hkv, Dh, scale_log2, causal);
        return after_launch("evkcu_flash_attention(simt)");
    });
}
