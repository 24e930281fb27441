// gemm.cu — evk::ai::matmul on sm_100a.
//
// Reference: evk_ai.cpp:254-330 (host), shaders/matmul.comp:44-140 (kernel).
// The reference runs one 32-lane subgroup per output tile with 16x16x16
// cooperative-matrix fragments loaded straight from global memory and an fp16
// accumulator.  Here:
//
//  * tcgen05 path (any M): a warp-specialised CTA per 128 x BN output tile.
//      warp 0 : TMA producer — 128-byte-swizzled A/B k-blocks (64 deep) into
//               a STAGES-deep shared-memory ring (mbarrier full/empty pairs);
//      warp 1 : allocates TMEM, one elected lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into a 128 x BN fp32 TMEM accumulator and
//               releases each ring slot with tcgen05.commit;
//      warps 2-5: epilogue — tcgen05.ld of their 32 TMEM lanes, optional
//               C += (acc_c), one rounding to fp16/bf16, 16-byte stores.
//    transpose_a / transpose_b select MN-major operand descriptors, so no
//    operand is ever transposed in memory.  Batch broadcast (stride 0) maps
//    to a batch extent of 1 in the tensor map.  M/N/K tails are handled by
//    TMA zero fill and epilogue guards.
//
//  * small-M path (decode, M*batch <= 16 with a shared B): a transposed
//    tcgen05 GEMV (see gemv_tc_kernel) that streams B once through TMA — the
//    weight read is the roofline there.
#include <algorithm>
#include <string>
#include <type_traits>

#include "greedy_key.cuh"
#include "sm100.cuh"

namespace evkcu {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 192;
constexpr uint32_t kTimeoutGemm = 0x101;

// ------------------------------------------------- fused QKV epilogue ----
// Inverse frequencies base^(-2p / Dh) for p < Dh / 2, once per CTA.
__device__ __forceinline__ float rope_inv_freq(float base, uint32_t p, uint32_t Dh) {
    return powf(base, -2.0f * (float)p / (float)Dh);
}

__device__ __forceinline__ void qkv_fill_inv_freq(const QkvRope& qr, float* inv_freq) {
    if (!qr.q) return;
    for (uint32_t p = threadIdx.x; p < qr.Dh / 2; p += blockDim.x) inv_freq[p] = rope_inv_freq(qr.base, p, qr.Dh);
}

__global__ void rope_table_kernel(float2* __restrict__ cs, uint32_t len, uint32_t Dh, float base) {
    const uint32_t half = Dh / 2;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)len * half) return;
    const uint32_t pos = (uint32_t)(i / half), p = (uint32_t)(i % half);
    float sn, c;
    sincosf((float)pos * rope_inv_freq(base, p, Dh), &sn, &c);
    cs[i] = make_float2(c, sn);
}

// Destination of output (row, col) of the fused QKV projection (see QkvRope);
// nullptr when the cache row lies beyond max_len.
template <typename T>
__device__ __forceinline__ T* qkv_dst(const QkvRope& qr, uint32_t pos_base, uint32_t row, uint32_t col) {
    const uint32_t qcols = qr.Hq * qr.Dh, kcols = qr.Hk * qr.Dh;
    if (col < qcols) return reinterpret_cast<T*>(qr.q) + (uint64_t)row * qcols + col;
    const uint32_t b = row / qr.S, pos = pos_base + row % qr.S;
    if (pos >= qr.max_len) return nullptr;
    const bool is_k = col < qcols + kcols;
    const uint32_t c = is_k ? col - qcols : col - qcols - kcols;
    return reinterpret_cast<T*>(is_k ? qr.kc : qr.vc) + ((uint64_t)b * qr.max_len + pos) * kcols + c;
}

// Rotates the pair (x0, x1) = columns (2p, 2p + 1) of a q / k head.
__device__ __forceinline__ void qkv_rotate(const QkvRope& qr, const float* inv_freq, uint32_t pos_base, uint32_t row,
                                           uint32_t col, float& x0, float& x1) {
    const uint32_t pos = pos_base + row % qr.S, p = (col % qr.Dh) >> 1;
    float sn, cs;
    if (qr.cs && pos < qr.cs_len) {
        const float2 e = __ldg(qr.cs + (uint64_t)pos * (qr.Dh >> 1) + p);
        cs = e.x;
        sn = e.y;
    } else {
        sincosf((float)pos * inv_freq[p], &sn, &cs);
    }
    const float a = x0 * cs - x1 * sn, b = x0 * sn + x1 * cs;
    x0 = a;
    x1 = b;
}

// CPS = CTAs per SM: 1 (a ~196 KB ring) or 2 (~96 KB each: one CTA's
// epilogue runs while the other's MMAs keep the tensor core busy).
template <int BN, int CPS>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = CPS == 2 ? 96 * 1024 : 196 * 1024;
    static constexpr int STAGES = RING / STAGE_BYTES > 8 ? 8 : (RING / STAGE_BYTES < 2 ? 2 : RING / STAGE_BYTES);
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <typename T, int BN, bool A_MN, bool B_MN, int CPS>
__global__ void __launch_bounds__(kGemmThreads, CPS)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmKc,
                   const __grid_constant__ CUtensorMap tmVc, T* __restrict__ C, uint32_t M, uint32_t N, uint32_t K,
                   uint64_t strideC, int bcastA, int bcastB, int acc_c, uint32_t idesc, unsigned int* err, int gelu,
                   QkvRope qr, int tma_c) {
    using Cfg = GemmCfg<BN, CPS>;
    __shared__ float s_inv_freq[128];
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint64_t* cbar = accum + 1;  // C tile loaded (acc_c with the TMA epilogue)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(cbar + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Raster: groups of kGroupM row tiles, row tile fastest within a group,
    // so the CTAs in flight share a few B column tiles and a group's A rows
    // stay in L2 while B streams past once per group (B is read
    // ceil(row tiles / kGroupM) times instead of once per wave of rows).
    constexpr uint32_t kGroupM = 16;
    uint32_t n0, m0;
    {
        const uint32_t nt = gridDim.x, mt = gridDim.y;
        const uint32_t lin = blockIdx.y * nt + blockIdx.x;
        const uint32_t per_group = kGroupM * nt;
        const uint32_t grp = lin / per_group, first_m = grp * kGroupM;
        const uint32_t gm = min(kGroupM, mt - first_m);  // rows in this (possibly last) group
        const uint32_t in = lin % per_group;
        m0 = (first_m + in % gm) * BM;
        n0 = (in / gm) * BN;
    }
    const uint32_t bz = blockIdx.z;
    const int za = bcastA ? 0 : (int)bz;
    const int zb = bcastB ? 0 : (int)bz;
    const uint32_t num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        mbar_init(cbar, 1);
        *s_abort = 0;
        fence_barrier_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (tma_c) prefetch_tmap(&tmC);
        if (tma_c == 2) {
            prefetch_tmap(&tmKc);
            prefetch_tmap(&tmVc);
        }
    }
    if (warp == 1) {
        tmem_alloc(s_tmem, BN);
        tmem_relinquish();
    }
    qkv_fill_inv_freq(qr, s_inv_freq);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            for (uint32_t kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, s_abort, err, kTimeoutGemm)) break;
                mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                const int k0 = (int)(kb * BK);
                uint8_t* a = sA + s * Cfg::A_BYTES;
                uint8_t* b = sB + s * Cfg::B_BYTES;
                if (!A_MN) {
                    tma_load_3d(a, &tmA, &full[s], k0, (int)m0, za);
                } else {
                    tma_load_3d(a, &tmA, &full[s], (int)m0, k0, za);
                    tma_load_3d(a + 8192, &tmA, &full[s], (int)m0 + 64, k0, za);
                }
                if (!B_MN) {
                    tma_load_3d(b, &tmB, &full[s], k0, (int)n0, zb);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tma_load_3d(b + j * 8192, &tmB, &full[s], (int)n0 + 64 * j, k0, zb);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (uint32_t kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (!mbar_wait(&full[s], ph, s_abort, err, kTimeoutGemm)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(sA + s * Cfg::A_BYTES);
                const uint32_t b = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    uint64_t ad = A_MN ? make_sw128_desc(a + k * 2048, 8192, 1024) : make_sw128_desc(a + k * 32, 16, 1024);
                    uint64_t bd = B_MN ? make_sw128_desc(b + k * 2048, 8192, 1024) : make_sw128_desc(b + k * 32, 16, 1024);
                    mma_f16_ss(tmem, ad, bd, idesc, (kb | k) != 0);
                }
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(accum);
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
        const int q = warp & 3;
        // Lane 0 waits (128 pollers on one barrier word would keep the shared
        // memory banks busy during the whole mainloop); the warp follows.
        const bool ok = __shfl_sync(0xffffffffu,
                                    lane == 0 ? (int)mbar_wait_sleep(accum, 0, s_abort, err, kTimeoutGemm) : 0,
                                    0) != 0;
        tc_fence_after();
        const uint32_t pos_base = qr.q ? (qr.d_pos ? *qr.d_pos : qr.pos0) : 0u;
        if (ok && tma_c) {
            // Staged epilogue: the ring is idle once the accumulator is
            // complete.  The C tile (acc_c) arrives there by TMA, each thread
            // combines its row (TMEM lane) 32 columns at a time in place, and
            // TMA stores write the tile back: coalesced global traffic instead
            // of one 16-byte access per row per instruction.  The staging is
            // BN / 64 boxes of 128 rows x 128 bytes in the 128-byte swizzle
            // (16-byte chunk k of row r at chunk k ^ (r % 8)), so the eight
            // rows of a quarter-warp hit eight different bank groups.
            // tma_c == 2 is the fused QKV epilogue of a prefill whose tiles
            // each lie in one sequence: q and k are rotated in registers and
            // every 64-column box goes to q, the K cache or the V cache.
            uint8_t* stg = smem;
            const bool leader = warp == 2 && lane == 0;
            bool go = true;
            if (acc_c) {
                if (leader) {
                    mbar_arrive_expect_tx(cbar, (uint32_t)BN * BM * 2);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_3d(stg + j * (BM * 128), &tmC, cbar, (int)(n0 + 64 * j), (int)m0, (int)bz);
                }
                const bool got = __shfl_sync(0xffffffffu,
                                             lane == 0 ? (int)mbar_wait(cbar, 0, s_abort, err, kTimeoutGemm) : 0, 0);
                if (!got && leader) mbar_drain(cbar, 0);  // C loads land before the CTA may exit
                go = got;
            }
            const uint32_t rr = q * 32 + lane;  // row within the tile
            // Fused QKV: this row's position and its (cos, sin) table row,
            // once per tile (with Dh % 32 == 0 a 32-column chunk never
            // crosses a head; other head sizes take qkv_rotate per pair).
            const uint32_t qk_cols = (qr.Hq + qr.Hk) * qr.Dh;
            const uint32_t rpos = tma_c == 2 ? pos_base + (m0 + rr) % qr.S : 0u;
            const float2* rtab = (tma_c == 2 && qr.cs && rpos < qr.cs_len && qr.Dh % 32 == 0)
                                     ? qr.cs + (uint64_t)rpos * (qr.Dh >> 1)
                                     : nullptr;
#pragma unroll 1
            for (int c = 0; go && c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, r);
                tmem_wait_ld();
                uint8_t* box = stg + (c >> 1) * (BM * 128) + rr * 128;
                const uint32_t col0 = n0 + c * 32;
                const bool rot = tma_c == 2 && col0 < qk_cols;
                const uint32_t pb = rot ? (col0 % qr.Dh) >> 1 : 0u;  // first rotation pair of the chunk
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const uint32_t kc = (uint32_t)((c & 1) * 4 + g);
                    Vec8* p = reinterpret_cast<Vec8*>(box + ((kc ^ (rr & 7)) << 4));
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[g * 8 + e]);
                    if (rot) {
                        if (rtab) {
                            // pairs pb + 4 g .. pb + 4 g + 3: two 16-byte loads
                            const float4 t0 = __ldg(reinterpret_cast<const float4*>(rtab + pb + 4 * g));
                            const float4 t1 = __ldg(reinterpret_cast<const float4*>(rtab + pb + 4 * g + 2));
                            const float cs4[4] = {t0.x, t0.z, t1.x, t1.z}, sn4[4] = {t0.y, t0.w, t1.y, t1.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a = f[2 * e] * cs4[e] - f[2 * e + 1] * sn4[e];
                                const float b = f[2 * e] * sn4[e] + f[2 * e + 1] * cs4[e];
                                f[2 * e] = a;
                                f[2 * e + 1] = b;
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; e += 2)
                                qkv_rotate(qr, s_inv_freq, pos_base, m0 + rr, col0 + g * 8 + e, f[e], f[e + 1]);
                        }
                    }
                    if (acc_c) {
                        float o[8];
                        unpack8<T>(ld_shared_vec8(p), o);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] += o[e];
                    }
                    if (gelu) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = gelu_f(f[e]);
                    }
                    st_shared_vec8(p, pack8<T>(f));
                }
            }
            fence_proxy_async_smem();
            named_barrier(1, 128);  // the four epilogue warps
            if (leader && go) {
                const uint32_t qcols = qr.Hq * qr.Dh, kcols = qr.Hk * qr.Dh;
#pragma unroll
                for (int j = 0; j < BN / 64; ++j) {
                    const uint32_t col = n0 + 64 * j;
                    if (tma_c != 2) {
                        tma_store_3d(&tmC, stg + j * (BM * 128), (int)col, (int)m0, (int)bz);
                    } else if (col < N) {
                        const int pos = (int)(pos_base + m0 % qr.S), b = (int)(m0 / qr.S);
                        if (col < qcols)
                            tma_store_3d(&tmC, stg + j * (BM * 128), (int)col, (int)m0, 0);
                        else if (col < qcols + kcols)
                            tma_store_3d(&tmKc, stg + j * (BM * 128), (int)(col - qcols), pos, b);
                        else
                            tma_store_3d(&tmVc, stg + j * (BM * 128), (int)(col - qcols - kcols), pos, b);
                    }
                }
                tma_store_commit();
                tma_store_wait_all();
            }
        } else if (ok) {
            const uint32_t row = m0 + q * 32 + lane;
            T* crow = C + (uint64_t)bz * strideC + (uint64_t)row * N;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, r);
                tmem_wait_ld();
                if (row < M) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint32_t col = n0 + c * 32 + g * 8;
                        if (col < N) {
                            float f[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[g * 8 + e]);
                            if (qr.q) {
                                if (col < (qr.Hq + qr.Hk) * qr.Dh) {
#pragma unroll
                                    for (int e = 0; e < 8; e += 2)
                                        qkv_rotate(qr, s_inv_freq, pos_base, row, col + e, f[e], f[e + 1]);
                                }
                                T* qd = qkv_dst<T>(qr, pos_base, row, col);
                                if (qd) *reinterpret_cast<Vec8*>(qd) = pack8<T>(f);
                                continue;
                            }
                            Vec8* dst = reinterpret_cast<Vec8*>(crow + col);
                            if (acc_c) {
                                float o[8];
                                unpack8<T>(*dst, o);
#pragma unroll
                                for (int e = 0; e < 8; ++e) f[e] += o[e];
                            }
                            if (gelu) {
#pragma unroll
                                for (int e = 0; e < 8; ++e) f[e] = gelu_f(f[e]);
                            }
                            *dst = pack8<T>(f);
                        }
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// ------------------------------------------ paired-SM GEMM (M = 256 tiles) ----
// Persistent kernel over 256 x 256 output tiles, one cluster of two CTAs on
// neighbouring SMs per tile at a time.  CTA rank r of the pair loads A rows
// [m0 + 128 r, +128) and B columns [n0 + 128 r, +128) into its own ring; the
// rank-0 CTA issues one tcgen05.mma.cta_group::2 of M = 256, N = 256, K = 16
// that reads both CTAs' operands, and each CTA's TMEM receives its 128 rows.
// Per SM that halves the B operand held in shared memory and streamed from
// L2 for the same tensor work as a 128 x 256 tile, and a 6-deep ring of 32 KB
// stages fits beside the epilogue's staging.
//
// Roles (192 threads per CTA):
//   warp 0 (both CTAs): TMA producer.  Each CTA's loads complete on the
//     rank-0 CTA's full[s] barrier; the MMA's commit (CTA mask 0b11) frees
//     the slot in both CTAs.
//   warp 1 (rank 0): MMA issue into one of two 256-column TMEM accumulators,
//     so the epilogue of tile j overlaps the mainloop of tile j + 1.
//   warps 2-5 (both CTAs): epilogue of the CTA's 128 rows in 64-column boxes
//     through two 16 KB staging buffers and TMA stores; the accumulator is
//     released to the MMA warp (rank 0's tempty, 8 arrivals) as soon as its
//     TMEM columns are in registers.
// No load is multicast: every TMA load writes the issuing CTA's own shared
// memory (only the MMA completion signal goes to both CTAs).  A variant that
// passed the completion on to rank 1 with remote arrives instead measured
// 745 against 1,380 TFLOP/s at 8192^3.  All waits are bounded; a CTA that gives up records a code
// in the device error word and both CTAs meet at the final cluster barrier.
constexpr int PR_ROWS = 128;  // rows (and B columns) per CTA of the pair
constexpr int PR_A_BYTES = PR_ROWS * BK * 2;
constexpr int PR_B_BYTES = PR_ROWS * BK * 2;
constexpr int PR_STAGE_BYTES = PR_A_BYTES + PR_B_BYTES;
constexpr int PR_STAGES = 6;
constexpr int PR_BOX_BYTES = PR_ROWS * 128;  // one 128-row x 64-column box
constexpr int PR_SMEM = PR_STAGES * PR_STAGE_BYTES + 2 * PR_BOX_BYTES + 1024 + 256;
constexpr int kPairThreads = 192;
constexpr uint32_t kTimeoutPair = 0x102;
static_assert(PR_SMEM + 512 <= 232448, "paired GEMM shared memory exceeds the per-CTA limit");

struct PairTile {
    uint32_t m0, n0, z;
};
__device__ __forceinline__ PairTile pair_tile(uint32_t t, uint32_t mt, uint32_t nt) {
    // Groups of 8 row tiles, row tile fastest: the pairs in flight share a
    // few B column tiles and one group's A rows.
    constexpr uint32_t G = 8;
    const uint32_t per_batch = mt * nt;
    PairTile p;
    p.z = t / per_batch;
    const uint32_t lin = t % per_batch, per_group = G * nt, grp = lin / per_group, first_m = grp * G;
    const uint32_t gm = min(G, mt - first_m), in = lin % per_group;
    p.m0 = (first_m + in % gm) * 256;
    p.n0 = (in / gm) * 256;
    return p;
}

template <typename T, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmKc,
                     const __grid_constant__ CUtensorMap tmVc, uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                     int bcastA, int bcastB, int acc_c, uint32_t idesc, unsigned int* err, int gelu, QkvRope qr,
                     int tma_c) {
    __shared__ float s_inv_freq[128];
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + PR_STAGES * PR_A_BYTES;
    uint8_t* stg = smem + PR_STAGES * PR_STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(stg + 2 * PR_BOX_BYTES);
    uint64_t* empty = full + PR_STAGES;
    uint64_t* tfull = empty + PR_STAGES;  // [2] accumulator buffer complete
    uint64_t* tempty = tfull + 2;         // [2] accumulator buffer read (rank 0: 8 arrivals)
    uint64_t* cbar = tempty + 2;          // [2] C box loaded into a staging buffer (acc_c)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(cbar + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const uint32_t rank = cluster_ctarank();
    const uint32_t pair = cluster_id_x(), npairs = cluster_count_x();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t mt = (M + 255) / 256, nt = (N + 255) / 256;
    const uint32_t total = mt * nt * batch;
    const uint32_t num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PR_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);
            mbar_init(&cbar[b], 1);
        }
        *s_abort = 0;
        fence_barrier_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (tma_c) prefetch_tmap(&tmC);
        if (tma_c == 2) {
            prefetch_tmap(&tmKc);
            prefetch_tmap(&tmVc);
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(s_tmem, 512);
        tmem_relinquish_pair();
    }
    qkv_fill_inv_freq(qr, s_inv_freq);
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or load
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < total; t += npairs) {
                const PairTile tl = pair_tile(t, mt, nt);
                const int za = bcastA ? 0 : (int)tl.z, zb = bcastB ? 0 : (int)tl.z;
                const int am = (int)(tl.m0 + PR_ROWS * rank), bn = (int)(tl.n0 + PR_ROWS * rank);
                for (uint32_t kb = 0; kb < num_kb; ++kb, ++it) {
                    const int s = (int)(it % PR_STAGES);
                    const uint32_t ph = (it / PR_STAGES) & 1;
                    if (!mbar_wait_cluster(&empty[s], ph ^ 1, s_abort, err, kTimeoutPair)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * PR_STAGE_BYTES);
                    const uint32_t fb = map_shared_rank(&full[s], 0);
                    const int k0 = (int)(kb * BK);
                    uint8_t* a = sA + s * PR_A_BYTES;
                    uint8_t* b = sB + s * PR_B_BYTES;
                    if (!A_MN) {
                        tma_load_3d_pair(a, &tmA, fb, k0, am, za);
                    } else {
                        tma_load_3d_pair(a, &tmA, fb, am, k0, za);
                        tma_load_3d_pair(a + 8192, &tmA, fb, am + 64, k0, za);
                    }
                    if (!B_MN) {
                        tma_load_3d_pair(b, &tmB, fb, k0, bn, zb);
                    } else {
                        tma_load_3d_pair(b, &tmB, fb, bn, k0, zb);
                        tma_load_3d_pair(b + 8192, &tmB, fb, bn + 64, k0, zb);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (rank == 0 && lane == 0) {
            uint32_t it = 0, j = 0;
            bool ok = true;
            for (uint32_t t = pair; ok && t < total; t += npairs, ++j) {
                const uint32_t buf = j & 1, use = j >> 1;
                if (!mbar_wait_cluster(&tempty[buf], (use & 1) ^ 1, s_abort, err, kTimeoutPair)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * 256;
                for (uint32_t kb = 0; kb < num_kb; ++kb, ++it) {
                    const int s = (int)(it % PR_STAGES);
                    const uint32_t ph = (it / PR_STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, s_abort, err, kTimeoutPair)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(sA + s * PR_A_BYTES);
                    const uint32_t b = smem_u32(sB + s * PR_B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t ad =
                            A_MN ? make_sw128_desc(a + k * 2048, 8192, 1024) : make_sw128_desc(a + k * 32, 16, 1024);
                        const uint64_t bd =
                            B_MN ? make_sw128_desc(b + k * 2048, 8192, 1024) : make_sw128_desc(b + k * 32, 16, 1024);
                        mma_f16_ss_pair(d, ad, bd, idesc, (kb | k) != 0);
                    }
                    mma_commit_pair_mask(&empty[s], 3);  // the slot is free in both CTAs
                }
                if (ok) mma_commit_pair_mask(&tfull[buf], 3);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const uint32_t rr = q * 32 + lane;      // row within the CTA's 128 rows
        const bool leader = warp == 2 && lane == 0;
        const uint32_t pos_base = qr.q ? (qr.d_pos ? *qr.d_pos : qr.pos0) : 0u;
        const uint32_t qk_cols = (qr.Hq + qr.Hk) * qr.Dh;
        uint32_t nbox = 0, j = 0;
        for (uint32_t t = pair; t < total; t += npairs, ++j) {
            const PairTile tl = pair_tile(t, mt, nt);
            const uint32_t buf = j & 1, use = j >> 1;
            int got = 0;
            if (lane == 0) {
                got = (int)mbar_wait_cluster(&tfull[buf], use & 1, s_abort, err, kTimeoutPair);
            }
            if (!__shfl_sync(0xffffffffu, got, 0)) break;
            tc_fence_after();
            const uint32_t mrow0 = tl.m0 + PR_ROWS * rank;  // this CTA's first output row
            const uint32_t rpos = tma_c == 2 ? pos_base + (mrow0 + rr) % qr.S : 0u;
            const float2* rtab =
                (tma_c == 2 && qr.cs && rpos < qr.cs_len) ? qr.cs + (uint64_t)rpos * (qr.Dh >> 1) : nullptr;
            bool go = true;
#pragma unroll 1
            for (int bx = 0; go && bx < 4; ++bx, ++nbox) {
                const uint32_t sb = nbox & 1;
                uint8_t* box = stg + sb * PR_BOX_BYTES;
                const uint32_t col0 = tl.n0 + 64 * bx;
                uint32_t r0[32], r1[32];
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + buf * 256 + bx * 64;
                tmem_ld32(ta, r0);
                tmem_ld32(ta + 32, r1);
                tmem_wait_ld();
                if (bx == 3) {
                    // The accumulator buffer is in registers: hand it back.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0) mbar_arrive(&tempty[buf]);
                        else mbar_arrive_remote(map_shared_rank(&tempty[buf], 0));
                    }
                }
                // The store issued from this buffer two boxes ago has read it.
                if (leader) tma_store_wait_read<1>();
                named_barrier(1, 128);
                if (acc_c) {
                    if (leader) {
                        mbar_arrive_expect_tx(&cbar[sb], (uint32_t)PR_BOX_BYTES);
                        tma_load_3d(box, &tmC, &cbar[sb], (int)col0, (int)mrow0, (int)tl.z);
                    }
                    const int ok =
                        __shfl_sync(0xffffffffu,
                                    lane == 0 ? (int)mbar_wait(&cbar[sb], (nbox >> 1) & 1, s_abort, err, kTimeoutPair)
                                              : 0,
                                    0);
                    if (!ok) {
                        if (leader) mbar_drain(&cbar[sb], (nbox >> 1) & 1);
                        go = false;
                        break;
                    }
                }
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(g < 4 ? r0[g * 8 + e] : r1[(g - 4) * 8 + e]);
                    Vec8* p = reinterpret_cast<Vec8*>(box + rr * 128 + ((g ^ (rr & 7)) << 4));
                    const uint32_t c = col0 + 8 * g;
                    if (tma_c == 2 && c < qk_cols) {
                        if (rtab) {
                            const uint32_t pb = (c % qr.Dh) >> 1;
                            const float4 t0 = __ldg(reinterpret_cast<const float4*>(rtab + pb));
                            const float4 t1 = __ldg(reinterpret_cast<const float4*>(rtab + pb + 2));
                            const float cs4[4] = {t0.x, t0.z, t1.x, t1.z}, sn4[4] = {t0.y, t0.w, t1.y, t1.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a = f[2 * e] * cs4[e] - f[2 * e + 1] * sn4[e];
                                const float b = f[2 * e] * sn4[e] + f[2 * e + 1] * cs4[e];
                                f[2 * e] = a;
                                f[2 * e + 1] = b;
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; e += 2)
                                qkv_rotate(qr, s_inv_freq, pos_base, mrow0 + rr, c + e, f[e], f[e + 1]);
                        }
                    }
                    if (acc_c) {
                        float o[8];
                        unpack8<T>(ld_shared_vec8(p), o);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] += o[e];
                    }
                    if (gelu) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = gelu_f(f[e]);
                    }
                    st_shared_vec8(p, pack8<T>(f));
                }
                fence_proxy_async_smem();
                named_barrier(1, 128);
                if (leader && mrow0 < M && col0 < N) {
                    if (tma_c != 2) {
                        tma_store_3d(&tmC, box, (int)col0, (int)mrow0, (int)tl.z);
                    } else {
                        const uint32_t qcols = qr.Hq * qr.Dh, kcols = qr.Hk * qr.Dh;
                        const int pos = (int)(pos_base + mrow0 % qr.S), b = (int)(mrow0 / qr.S);
                        if (col0 < qcols)
                            tma_store_3d(&tmC, box, (int)col0, (int)mrow0, 0);
                        else if (col0 < qcols + kcols)
                            tma_store_3d(&tmKc, box, (int)(col0 - qcols), pos, b);
                        else
                            tma_store_3d(&tmVc, box, (int)(col0 - qcols - kcols), pos, b);
                    }
                    tma_store_commit();
                }
            }
            if (!go) break;
        }
        if (leader) tma_store_wait_all();
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync_all();  // no CTA leaves while its pair may still touch its memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// --------------------------------------------------------- small-M GEMV ----
// y[m, n] = sum_k x[m, k] * W[k, n]     (W row-major [K, N]; or [N, K] with
// transpose_b, e.g. a tied-embedding LM head), for Mt <= 16 rows of x.
// The weight read is the roofline (2 bytes per weight, each used Mt times),
// and at Mt = 8..16 even the FMAs would outrun the CUDA cores at full HBM
// rate, so the product runs on the tensor cores transposed:
//     y^T[n, m] = sum_k W^T[n, k] * x^T[k, m]
// One CTA owns a 128-column slab of W (the MMA's M = 128) and a range of
// 64-deep k-tiles.  W is the A operand (MN-major for row-major W, K-major for
// transpose_b), x is the B operand (K-major, N = 16 rows, rows >= Mt
// zero-filled by TMA).  Warp 0 streams W/x k-tiles through a GV_STAGES-deep
// ring, warp 1 issues tcgen05.mma into a 128 x 16 fp32 TMEM accumulator,
// warps 2-5 read it back (TMEM lane = output column).  The grid is one
// resident wave (two CTAs per SM); K is split across gridDim.y CTAs whose
// fp32 partials the last CTA of each slab (atomic ticket) adds in split order,
// so results are bit-reproducible.
constexpr int kGemvMaxM = 16;
constexpr int GV_COLS = 128;
constexpr int GV_BK = 64;
constexpr int GV_MMA_N = 16;
constexpr int GV_STAGES = 6;
constexpr int GV_EARLY = 4;  // weight tiles requested before griddepcontrol.wait
constexpr int GV_W_BYTES = GV_COLS * GV_BK * 2;    // 16 KB
constexpr int GV_X_BYTES = GV_MMA_N * GV_BK * 2;   // 2 KB
constexpr int GV_STAGE_BYTES = GV_W_BYTES + GV_X_BYTES;
constexpr int GV_SMEM = GV_STAGES * GV_STAGE_BYTES + 1024 + 256;
constexpr int GV_THREADS = 192;
constexpr uint32_t kTimeoutGemv = 0x301;

template <typename T>
__device__ void gemv_argmax_tail(const float* s_val, uint32_t Mt, uint32_t N, uint32_t n0, const GemvArgmax& am);
template <typename T>
__device__ void gemv_combine_splits(const float* __restrict__ partial, T* __restrict__ Y, uint32_t Mt, uint32_t N,
                                    uint32_t n0, int acc_c, int gelu, int write_y, float* s_val, bool raw,
                                    const QkvRope& qr, const float* inv_freq);
template <typename T>
__device__ void gemv_allreduce_tail(const float* s_val, T* __restrict__ Y, uint32_t Mt, uint32_t N, uint32_t n0,
                                    const GemvAllReduce& ar, unsigned int* err);

template <typename T, bool W_KMAJOR>
__global__ void __launch_bounds__(GV_THREADS, 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   T* __restrict__ Y, uint32_t Mt, uint32_t K, uint32_t N, uint32_t ktiles_per_cta, int acc_c,
                   uint32_t idesc, float* __restrict__ partial, unsigned int* __restrict__ tickets,
                   unsigned int* err, int gelu, GemvArgmax am, GemvAllReduce ar, QkvRope qr) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sX = smem + GV_STAGES * GV_W_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + GV_STAGES * GV_STAGE_BYTES);
    uint64_t* empty = full + GV_STAGES;
    uint64_t* accum = empty + GV_STAGES;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    __shared__ bool is_last;
    __shared__ float s_inv_freq[128];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = blockIdx.x * GV_COLS;
    const uint32_t kt_total = (K + GV_BK - 1) / GV_BK;
    const uint32_t kt0 = blockIdx.y * ktiles_per_cta;
    const uint32_t kt1 = min(kt0 + ktiles_per_cta, kt_total);
    const uint32_t nkt = kt1 > kt0 ? kt1 - kt0 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GV_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *s_abort = 0;
        fence_barrier_init();
        prefetch_tmap(&tmW);
        prefetch_tmap(&tmX);
    }
    if (warp == 1) {
        tmem_alloc(s_tmem, 32);
        tmem_relinquish();
    }
    qkv_fill_inv_freq(qr, s_inv_freq);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    pdl_trigger();
    // Every thread but the producer lane (which waits after requesting the
    // first weight tiles) may read or write data of earlier kernels: x through
    // the MMAs, y and the split scratch in the epilogue and final reduction.
    if (warp != 0 || lane != 0) pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            auto load_w = [&](uint32_t i, int s) {
                const int k0 = (int)((kt0 + i) * GV_BK);
                uint8_t* w = sW + s * GV_W_BYTES;
                if (W_KMAJOR) {
                    tma_load_3d(w, &tmW, &full[s], k0, (int)n0, 0);
                } else {
                    tma_load_3d(w, &tmW, &full[s], (int)n0, k0, 0);
                    tma_load_3d(w + GV_W_BYTES / 2, &tmW, &full[s], (int)n0 + 64, k0, 0);
                }
            };
            // The weights are constant: the first GV_EARLY W tiles are
            // requested before waiting for the kernels that produce x, the
            // rest of the ring after it, each behind its stage's x tile (x
            // queued behind a full ring of weight tiles arrives later:
            // 4 early tiles measured 2-4 % faster than 6 on the C4 GEMVs).
            const uint32_t pre = min(nkt, (uint32_t)GV_STAGES);
            const uint32_t early = min(pre, (uint32_t)GV_EARLY);
            for (uint32_t i = 0; i < early; ++i) {
                mbar_arrive_expect_tx(&full[i], GV_STAGE_BYTES);
                load_w(i, (int)i);
            }
            pdl_wait();
            for (uint32_t i = 0; i < pre; ++i) {
                if (i >= early) {
                    mbar_arrive_expect_tx(&full[i], GV_STAGE_BYTES);
                    load_w(i, (int)i);
                }
                tma_load_3d(sX + i * GV_X_BYTES, &tmX, &full[i], (int)((kt0 + i) * GV_BK), 0, 0);
            }
            for (uint32_t i = pre; i < nkt; ++i) {
                const int s = i % GV_STAGES;
                if (!mbar_wait(&empty[s], ((i / GV_STAGES) & 1) ^ 1, s_abort, err, kTimeoutGemv)) break;
                mbar_arrive_expect_tx(&full[s], GV_STAGE_BYTES);
                load_w(i, s);
                tma_load_3d(sX + s * GV_X_BYTES, &tmX, &full[s], (int)((kt0 + i) * GV_BK), 0, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (uint32_t i = 0; i < nkt; ++i) {
                const int s = i % GV_STAGES;
                if (!mbar_wait(&full[s], (i / GV_STAGES) & 1, s_abort, err, kTimeoutGemv)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(sW + s * GV_W_BYTES);
                const uint32_t b = smem_u32(sX + s * GV_X_BYTES);
#pragma unroll
                for (int k = 0; k < GV_BK / 16; ++k) {
                    const uint64_t ad =
                        W_KMAJOR ? make_sw128_desc(a + k * 32, 16, 1024) : make_sw128_desc(a + k * 2048, 8192, 1024);
                    const uint64_t bd = make_sw128_desc(b + k * 32, 16, 1024);
                    mma_f16_ss(tmem, ad, bd, idesc, (i | k) != 0);
                }
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(accum);
        }
    }
    // Warps 2-5: TMEM lane quarter q = warp % 4 holds output columns
    // n0 + 32q .. +31, one per lane, with the Mt rows of x in columns 0..15.
    float v[GV_MMA_N];
    bool have = false;
    const int q = warp & 3;
    const uint32_t nn = q * 32 + lane;
    if (warp >= 2) {
        have = nkt == 0 || mbar_wait(accum, 0, s_abort, err, kTimeoutGemv);
        tc_fence_after();
        if (nkt == 0) {
#pragma unroll
            for (int m = 0; m < GV_MMA_N; ++m) v[m] = 0.0f;
        } else if (have) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16), r);
            tmem_wait_ld();
#pragma unroll
            for (int m = 0; m < GV_MMA_N; ++m) v[m] = __uint_as_float(r[m]);
        }
        tc_fence_before();
        if (have && gridDim.y == 1 && qr.q) {
            // Fused QKV: rotate with the partner column (adjacent lane),
            // store to q or the caches.
            const uint32_t n = n0 + nn;
            const uint32_t pos_base = qr.d_pos ? *qr.d_pos : qr.pos0;
            const bool rot = n < (qr.Hq + qr.Hk) * qr.Dh;
#pragma unroll
            for (int m = 0; m < GV_MMA_N; ++m) {
                const float partner = __shfl_xor_sync(0xffffffffu, v[m], 1);
                if (m < (int)Mt && n < N) {
                    float x0 = (n & 1) ? partner : v[m], x1 = (n & 1) ? v[m] : partner;
                    if (rot) qkv_rotate(qr, s_inv_freq, pos_base, m, n & ~1u, x0, x1);
                    T* qd = qkv_dst<T>(qr, pos_base, m, n);
                    if (qd) *qd = Elem<T>::from_f((n & 1) ? x1 : x0);
                }
            }
        } else if (have && gridDim.y == 1) {
            const uint32_t n = n0 + nn;
            // With an argmax the TMA ring (idle now) stages the stored values.
            float* s_val = reinterpret_cast<float*>(smem);  // [GV_MMA_N][GV_COLS]
#pragma unroll
            for (int m = 0; m < GV_MMA_N; ++m) {
                if (m < (int)Mt) {
                    float o = v[m];
                    if (n < N) {
                        if (acc_c) o += Elem<T>::to_f(Y[(uint64_t)m * N + n]);
                        if (gelu) o = gelu_f(o);
                        const T st = Elem<T>::from_f(o);
                        if (am.write_y) Y[(uint64_t)m * N + n] = st;
                        o = Elem<T>::to_f(st);
                    }
                    if (am.slab_keys) s_val[m * GV_COLS + nn] = o;
                    if (ar.tp) s_val[m * GV_COLS + nn] = v[m];
                }
            }
        } else if (have) {
            float* my = partial + ((uint64_t)blockIdx.x * gridDim.y + blockIdx.y) * (GV_MMA_N * GV_COLS);
#pragma unroll
            for (int m = 0; m < GV_MMA_N; ++m)
                if (m < (int)Mt) my[m * GV_COLS + nn] = v[m];
            __threadfence();
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
    if (*s_abort) return;
    if (gridDim.y > 1) {
        if (threadIdx.x == 0) is_last = atomicAdd(&tickets[blockIdx.x], 1u) == gridDim.y - 1;
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        gemv_combine_splits<T>(partial, Y, Mt, N, n0, acc_c, gelu, am.write_y,
                               (am.slab_keys || ar.tp) ? reinterpret_cast<float*>(smem) : nullptr, ar.tp != 0, qr,
                               s_inv_freq);
        if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
    }
    if (am.slab_keys) gemv_argmax_tail<T>(reinterpret_cast<const float*>(smem), Mt, N, n0, am);
    if (ar.tp) gemv_allreduce_tail<T>(reinterpret_cast<const float*>(smem), Y, Mt, N, n0, ar, err);
}

// Tensor-parallel all-reduce of one slab's fp32 partial (see GemvAllReduce),
// in the low-latency form of a flag beside every value: each 16-byte store
// carries two (value, flag) pairs, and an aligned 8-byte pair is written and
// read as one unit, so a reader that sees the expected flag also sees the
// value, with no memory fence on either side.  The flag is unique per decode
// step and call site (step * 256 + callsite + 1; never 0, the buffer's
// initial contents).
//   1. push this rank's partial into slot [parity][rank] of every rank's
//      buffer (peer memory over NVLink);
//   2. poll this rank's own buffer (bounded) until every rank's slot shows
//      the flag, summing the values in rank order (the same on every rank,
//      so the replicated residual stays bit-identical);
//   3. add the sum to the residual y.
// A rank cannot get two all-reduces ahead of another (each needs every
// rank's contribution), so a slot is rewritten only after its readers are
// done with it.
__device__ __forceinline__ void st_pair2(uint2* dst, float v0, float v1, uint32_t flag) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(__float_as_uint(v0)), "r"(flag),
                 "r"(__float_as_uint(v1)), "r"(flag)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_pair2(const uint2* src) {
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(src)
                 : "memory");
    return r;
}

template <typename T>
__device__ void gemv_allreduce_tail(const float* s_val, T* __restrict__ Y, uint32_t Mt, uint32_t N, uint32_t n0,
                                    const GemvAllReduce& ar, unsigned int* err) {
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();  // s_val complete
    const uint32_t par = ar.callsite & 1;
    const uint32_t flag = *ar.epoch * 256u + ar.callsite + 1u;
    if (ar.half) {
        // Four columns per 16-byte word: {v0 v1 | flag | v2 v3 | flag}.
        const uint32_t g4 = Mt * GV_COLS / 4, NW = N / 2;  // NW: words of one row
        using T2 = typename Elem<T>::T2;
        for (uint32_t g = threadIdx.x; g < g4; g += blockDim.x) {
            const uint32_t m = (g * 4) / GV_COLS, c = (g * 4) % GV_COLS;
            if (n0 + c >= N) continue;
            const float4 v = *reinterpret_cast<const float4*>(s_val + m * GV_COLS + c);
            const T2 lo = Elem<T>::from_f2(v.x, v.y), hi = Elem<T>::from_f2(v.z, v.w);
            const uint64_t off = ((uint64_t)(par * ar.tp + ar.rank) * GV_MMA_N + m) * NW + (n0 + c) / 2;
            for (uint32_t q = 0; q < ar.tp; ++q)
                st_pair2(ar.buf[q] + off, __uint_as_float(*reinterpret_cast<const uint32_t*>(&lo)),
                         __uint_as_float(*reinterpret_cast<const uint32_t*>(&hi)), flag);
        }
        const uint2* mine = ar.buf[ar.rank];
        const long long t0 = clock64();
        for (uint32_t g = threadIdx.x; g < g4; g += blockDim.x) {
            const uint32_t m = (g * 4) / GV_COLS, c = (g * 4) % GV_COLS, n = n0 + c;
            if (n >= N) continue;
            float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (uint32_t q = 0; q < ar.tp; ++q) {
                const uint2* src = mine + ((uint64_t)(par * ar.tp + q) * GV_MMA_N + m) * NW + n / 2;
                uint4 w = ld_pair2(src);
                for (uint32_t spin = 0; w.y != flag || w.w != flag; ++spin) {
                    if ((spin & 31) == 31) {
                        if (*reinterpret_cast<volatile int*>(&s_fail) || *reinterpret_cast<volatile unsigned int*>(err)) {
                            s_fail = 1;
                            return;
                        }
                        if (clock64() - t0 > kSpinLimitCycles / 2) {
                            atomicCAS(err, 0u, 0x302u);
                            s_fail = 1;
                            return;
                        }
                    }
                    w = ld_pair2(src);
                }
                const float2 p0 = Elem<T>::to_f2(*reinterpret_cast<const T2*>(&w.x));
                const float2 p1 = Elem<T>::to_f2(*reinterpret_cast<const T2*>(&w.z));
                a[0] += p0.x;
                a[1] += p0.y;
                a[2] += p1.x;
                a[3] += p1.y;
            }
            T* y = Y + (uint64_t)m * N + n;
#pragma unroll
            for (int e = 0; e < 4; ++e) y[e] = Elem<T>::from_f(Elem<T>::to_f(y[e]) + a[e]);
        }
        return;
    }
    const uint32_t groups = Mt * GV_COLS / 2;
    for (uint32_t g = threadIdx.x; g < groups; g += blockDim.x) {
        const uint32_t m = (g * 2) / GV_COLS, c = (g * 2) % GV_COLS;
        if (n0 + c >= N) continue;
        const float2 v = *reinterpret_cast<const float2*>(s_val + m * GV_COLS + c);
        const uint64_t off = ((uint64_t)(par * ar.tp + ar.rank) * GV_MMA_N + m) * N + n0 + c;
        for (uint32_t q = 0; q < ar.tp; ++q) st_pair2(ar.buf[q] + off, v.x, v.y, flag);
    }
    const uint2* mine = ar.buf[ar.rank];
    const long long t0 = clock64();
    for (uint32_t g = threadIdx.x; g < groups; g += blockDim.x) {
        const uint32_t m = (g * 2) / GV_COLS, c = (g * 2) % GV_COLS, n = n0 + c;
        if (n >= N) continue;
        float a0 = 0.0f, a1 = 0.0f;
        for (uint32_t q = 0; q < ar.tp; ++q) {
            const uint2* src = mine + ((uint64_t)(par * ar.tp + q) * GV_MMA_N + m) * N + n;
            uint4 w = ld_pair2(src);
            for (uint32_t spin = 0; w.y != flag || w.w != flag; ++spin) {
                if ((spin & 31) == 31) {
                    if (*reinterpret_cast<volatile int*>(&s_fail) || *reinterpret_cast<volatile unsigned int*>(err)) {
                        s_fail = 1;
                        return;
                    }
                    if (clock64() - t0 > kSpinLimitCycles / 2) {
                        atomicCAS(err, 0u, 0x302u);
                        s_fail = 1;
                        return;
                    }
                }
                w = ld_pair2(src);
            }
            a0 += __uint_as_float(w.x);
            a1 += __uint_as_float(w.z);
        }
        T* y = Y + (uint64_t)m * N + n;
        y[0] = Elem<T>::from_f(Elem<T>::to_f(y[0]) + a0);
        y[1] = Elem<T>::from_f(Elem<T>::to_f(y[1]) + a1);
    }
}

// Fused argmax over the GEMV's outputs (greedy sampling of an LM head): each
// slab reduces its staged values (already rounded to the storage type, i.e.
// the logits a separate kernel would read) to one 64-bit selection key per
// row (greedy_key.cuh: the reference's tie rule), and the last slab to finish
// (global ticket) reduces the slab keys to the row's key or token id.
// Maxima of keys are exact, so the result is independent of the order.
template <typename T>
__device__ void gemv_argmax_tail(const float* s_val, uint32_t Mt, uint32_t N, uint32_t n0, const GemvArgmax& am) {
    __shared__ bool last_slab;
    __syncthreads();  // s_val complete
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    for (uint32_t m = warp; m < Mt; m += nwarps) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int e = 0; e < GV_COLS / 32; ++e) {
            const uint32_t c = lane + 32 * e;
            const uint32_t n = n0 + c;
            const unsigned long long k = n < N ? elem_key(s_val[m * GV_COLS + c], am.key_off + n) : 0ull;
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (lane == 0) am.slab_keys[(uint64_t)blockIdx.x * GV_MMA_N + m] = best;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_slab = atomicAdd(am.ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last_slab) return;
    __threadfence();
    for (uint32_t m = warp; m < Mt; m += nwarps) {
        unsigned long long best = 0ull;
        for (uint32_t sl = lane; sl < gridDim.x; sl += 32) {
            const unsigned long long k = __ldcg(am.slab_keys + (uint64_t)sl * GV_MMA_N + m);
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (lane == 0) {
            if (am.keys_out) am.keys_out[m] = best;
            if (am.ids_out) am.ids_out[m] = best ? key_to_offset(best) : 0u;
        }
    }
    if (threadIdx.x == 0) *am.ticket = 0u;
}

// Last CTA of a slab: adds the split partials in split order and applies
// the epilogue; optionally stages the stored values for the argmax.
template <typename T>
__device__ void gemv_combine_splits(const float* __restrict__ partial, T* __restrict__ Y, uint32_t Mt, uint32_t N,
                                    uint32_t n0, int acc_c, int gelu, int write_y, float* s_val, bool raw,
                                    const QkvRope& qr, const float* inv_freq) {
    // Thread g takes 4 consecutive outputs (one float4 of every split's
    // partial) and keeps up to 16 splits' loads in flight before adding them
    // in split order, so the combine costs a few L2 round trips, not one per
    // split.
    const float* base = partial + (uint64_t)blockIdx.x * gridDim.y * (GV_MMA_N * GV_COLS);
    const uint32_t groups = Mt * GV_COLS / 4;
    if (groups < blockDim.x && !qr.q) {
        // Few rows: one output per thread keeps more threads loading.
        for (uint32_t i = threadIdx.x; i < Mt * GV_COLS; i += blockDim.x) {
            const uint32_t m = i / GV_COLS, c = i % GV_COLS, n = n0 + c;
            float sum = 0.0f;
            for (uint32_t y0 = 0; y0 < gridDim.y; y0 += 8) {
                float t[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    t[j] = y0 + j < gridDim.y ? __ldcg(base + (uint64_t)(y0 + j) * (GV_MMA_N * GV_COLS) + i) : 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (y0 + j < gridDim.y) sum += t[j];
            }
            if (raw) {
                s_val[m * GV_COLS + c] = sum;
                continue;
            }
            if (n < N) {
                if (acc_c) sum += Elem<T>::to_f(Y[(uint64_t)m * N + n]);
                if (gelu) sum = gelu_f(sum);
                const T st = Elem<T>::from_f(sum);
                if (write_y) Y[(uint64_t)m * N + n] = st;
                sum = Elem<T>::to_f(st);
            }
            if (s_val) s_val[m * GV_COLS + c] = sum;
        }
        return;
    }
    for (uint32_t g = threadIdx.x; g < groups; g += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (uint32_t y0 = 0; y0 < gridDim.y; y0 += 16) {
            float4 t[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (y0 + j < gridDim.y)
                    t[j] = __ldcg(reinterpret_cast<const float4*>(base + (uint64_t)(y0 + j) * (GV_MMA_N * GV_COLS)) + g);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                if (y0 + j < gridDim.y) {
                    acc.x += t[j].x;
                    acc.y += t[j].y;
                    acc.z += t[j].z;
                    acc.w += t[j].w;
                }
            }
        }
        float sums[4] = {acc.x, acc.y, acc.z, acc.w};
        if (qr.q) {
            // Fused QKV: columns 4g .. 4g + 3 hold two rotation pairs.
            const uint32_t m = (g * 4) / GV_COLS, n = n0 + (g * 4) % GV_COLS;
            if (n >= N) continue;
            const uint32_t pos_base = qr.d_pos ? *qr.d_pos : qr.pos0;
            if (n < (qr.Hq + qr.Hk) * qr.Dh) {
                qkv_rotate(qr, inv_freq, pos_base, m, n, sums[0], sums[1]);
                qkv_rotate(qr, inv_freq, pos_base, m, n + 2, sums[2], sums[3]);
            }
            T* qd = qkv_dst<T>(qr, pos_base, m, n);
            if (qd)
#pragma unroll
                for (int e = 0; e < 4; ++e) qd[e] = Elem<T>::from_f(sums[e]);
            continue;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t i = g * 4 + e;
            const uint32_t m = i / GV_COLS, c = i % GV_COLS, n = n0 + c;
            float sum = sums[e];
            if (raw) {  // the unrounded fp32 sum, for the all-reduce
                s_val[m * GV_COLS + c] = sum;
                continue;
            }
            if (n < N) {
                if (acc_c) sum += Elem<T>::to_f(Y[(uint64_t)m * N + n]);
                if (gelu) sum = gelu_f(sum);
                const T st = Elem<T>::from_f(sum);
                if (write_y) Y[(uint64_t)m * N + n] = st;
                sum = Elem<T>::to_f(st);
            }
            if (s_val) s_val[m * GV_COLS + c] = sum;
        }
    }
}

template <typename T, bool W_KMAJOR>
int launch_gemv_tc(const T* X, const T* W, T* Y, uint32_t Mt, uint32_t K, uint32_t N, GemvEpilogue ep, int dtype,
                   cudaStream_t st, GemvArgmax am = GemvArgmax(), const GemvAllReduce& ar = GemvAllReduce(),
                   const QkvRope& qr = QkvRope()) {
    DeviceState* s = state();
    const uint32_t slabs = (N + GV_COLS - 1) / GV_COLS;
    const uint32_t ktiles = (K + GV_BK - 1) / GV_BK;
    // Weights under 64 MB: one CTA per SM (a 6-deep ring each keeps ~16 MB
    // of loads in flight), leaving the SM's other slot to the next kernel of
    // a decode chain, which (programmatic dependent launch) streams its own
    // weights meanwhile.  Larger weights: two CTAs per SM.  Whole k-tiles per
    // split, at least 4 for weights of 16 MB and more (each split adds a
    // partial to the combine).
    const uint64_t wbytes = (uint64_t)K * N * sizeof(T);
    const uint32_t per_sm = wbytes < (64ull << 20) ? 1u : 2u;
    const uint32_t slots = per_sm * (uint32_t)s->sm_count;
    // Tiny weights (< 16 MB) are pure latency: as many CTAs as there are slots.
    const uint32_t min_tiles = wbytes < (16ull << 20) ? 1u : 4u;
    uint32_t splits =
        std::max<uint32_t>(1, std::min<uint32_t>(std::max<uint32_t>(1, ktiles / min_tiles), slots / slabs));
    const uint32_t per = (ktiles + splits - 1) / splits;
    splits = (ktiles + per - 1) / per;
    CUtensorMap mW, mX;
    int r = W_KMAJOR ? make_tmap_3d(&mW, W, K, N, 1, K, (uint64_t)K * N, GV_BK, GV_COLS, dtype)
                     : make_tmap_3d(&mW, W, N, K, 1, N, (uint64_t)K * N, 64, GV_BK, dtype);
    if (r) return r;
    r = make_tmap_3d(&mX, X, K, Mt, 1, K, (uint64_t)K * Mt, GV_BK, GV_MMA_N, dtype);
    if (r) return r;
    float* partial = nullptr;
    unsigned int* tickets = nullptr;
    const bool argmax = am.keys_out || am.ids_out;
    if (splits > 1 || argmax) {
        // Scratch: slab tickets (the last one is the argmax's global ticket),
        // split partials, then the argmax's per-slab keys.
        if (slabs >= kMaxTickets) return fail(EVKCU_BAD_SHAPE, "evkcu_matmul: N too large for the GEMV path");
        const size_t pbytes = splits > 1 ? (size_t)slabs * splits * GV_MMA_N * GV_COLS * sizeof(float) : 0;
        const size_t kbytes = argmax ? (size_t)slabs * GV_MMA_N * sizeof(unsigned long long) : 0;
        char* ws = (char*)workspace(WS_GEMV, kTicketBytes + pbytes + kbytes);
        if (!ws) return fail(EVKCU_CUDA_ERROR, "evkcu_matmul: workspace allocation failed");
        tickets = (unsigned int*)ws;
        partial = (float*)(ws + kTicketBytes);
        if (argmax) {
            am.ticket = tickets + (kMaxTickets - 1);
            am.slab_keys = (unsigned long long*)(ws + kTicketBytes + pbytes);
        }
    }
    auto kern = gemv_tc_kernel<T, W_KMAJOR>;
    static bool attr_set = false;
    if (!attr_set) {
        EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM));
        attr_set = true;
    }
    const uint32_t idesc = make_idesc_f16(GV_COLS, GV_MMA_N, dtype == EVKCU_BF16 ? 1 : 0, W_KMAJOR ? 0 : 1, 0);
    dim3 grid(slabs, splits);
    return launch_pdl("evkcu_matmul(gemv_tc)", kern, grid, GV_THREADS, GV_SMEM, st, mW, mX, Y, Mt, K, N, per, ep.acc,
                      idesc, partial, tickets, s->d_error, ep.gelu, am, ar, qr);
}

// Tensor maps of the staged (TMA) epilogue, 64-column x 128-row boxes in the
// 128-byte swizzle: the C map for plain C = A B (+ C) (GELU), or the q / K
// cache / V cache maps of a prefill's fused QKV projection.  *tma_c receives
// the epilogue kind: 1 plain, 2 fused QKV, 0 per-row stores (no maps).
int make_c_maps(CUtensorMap& tc, CUtensorMap& tk, CUtensorMap& tv, void* C, uint32_t batch, uint32_t M, uint32_t N,
                uint64_t strideC, const QkvRope& qr, int is_bf16, int* tma_c) {
    memset(&tc, 0, sizeof(tc));
    memset(&tk, 0, sizeof(tk));
    memset(&tv, 0, sizeof(tv));
    const int dt = is_bf16 ? EVKCU_BF16 : EVKCU_F16;
    *tma_c = 0;
    if (!qr.q && !state()->plain_epilogue) {
        const int r = make_tmap_3d(&tc, C, N, M, batch, N, batch > 1 ? strideC : (uint64_t)M * N, 64, BM, dt);
        if (r) return r;
        *tma_c = 1;
    } else if (qr.q && !qr.d_pos && qr.S % BM == 0 && (qr.Hq * qr.Dh) % 64 == 0 && (qr.Hk * qr.Dh) % 64 == 0 &&
               batch == 1 && !state()->plain_epilogue) {
        // Fused QKV of a prefill: q [M, Hq * Dh]; caches [M / S, max_len, Hk * Dh].
        const uint64_t qc = (uint64_t)qr.Hq * qr.Dh, kc = (uint64_t)qr.Hk * qr.Dh, nb = M / qr.S;
        int r = make_tmap_3d(&tc, qr.q, qc, M, 1, qc, qc * M, 64, BM, dt);
        if (!r) r = make_tmap_3d(&tk, qr.kc, kc, qr.max_len, nb, kc, kc * qr.max_len, 64, BM, dt);
        if (!r) r = make_tmap_3d(&tv, qr.vc, kc, qr.max_len, nb, kc, kc * qr.max_len, 64, BM, dt);
        if (r) return r;
        *tma_c = 2;
    }
    return EVKCU_OK;
}

template <typename T, int BN, bool A_MN, bool B_MN, int CPS>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, T* C, uint32_t batch, uint32_t M, uint32_t N, uint32_t K,
              uint64_t strideC, int bcastA, int bcastB, int acc, int is_bf16, int gelu, const QkvRope& qr,
              cudaStream_t st) {
    using Cfg = GemmCfg<BN, CPS>;
    static_assert(Cfg::STAGES * Cfg::STAGE_BYTES >= BN * BM * 2, "C staging must fit in the ring");
    CUtensorMap tc, tk, tv;
    int tma_c = 0;
    if (int r = make_c_maps(tc, tk, tv, C, batch, M, N, strideC, qr, is_bf16, &tma_c)) return r;
    static bool attr_set = false;
    auto kern = gemm_tc_kernel<T, BN, A_MN, B_MN, CPS>;
    if (!attr_set) {
        EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
        attr_set = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, batch);
    uint32_t idesc = make_idesc_f16(BM, BN, is_bf16, A_MN, B_MN);
    kern<<<grid, kGemmThreads, Cfg::SMEM, st>>>(ta, tb, tc, tk, tv, C, M, N, K, strideC, bcastA, bcastB, acc, idesc,
                                                state()->d_error, gelu, qr, tma_c);
    return after_launch("evkcu_matmul(tcgen05)");
}

// Paired-SM GEMM: one persistent cluster of two CTAs per resident SM pair.
// The staged epilogue is required (tma_c != 0).
template <typename T, bool A_MN, bool B_MN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tk,
                const CUtensorMap& tv, int tma_c, uint32_t batch, uint32_t M, uint32_t N, uint32_t K, int bcastA,
                int bcastB, int acc, int is_bf16, int gelu, const QkvRope& qr, uint32_t clusters, cudaStream_t st) {
    auto kern = gemm_pair_kernel<T, A_MN, B_MN>;
    const uint32_t tiles = ((M + 255) / 256) * ((N + 255) / 256) * batch;
    const uint32_t n = std::min(tiles, clusters);
    const uint32_t idesc = make_idesc_f16(256, 256, is_bf16, A_MN, B_MN);
    kern<<<2 * n, kPairThreads, PR_SMEM, st>>>(ta, tb, tc, tk, tv, M, N, K, batch, bcastA, bcastB, acc, idesc,
                                               state()->d_error, gelu, qr, tma_c);
    return after_launch("evkcu_matmul(tcgen05 pair)");
}

// Sets the shared-memory limit of every paired-GEMM instantiation and
// returns how many CTA pairs are resident at once (0 if the device cannot
// run the kernel).  Queried once per device.
uint32_t pair_clusters() {
    DeviceState* ds = state();
    if (ds->pair_clusters) return ds->pair_clusters > 0 ? (uint32_t)ds->pair_clusters : 0u;
    const void* kerns[] = {
        (const void*)gemm_pair_kernel<__half, false, false>,         (const void*)gemm_pair_kernel<__half, false, true>,
        (const void*)gemm_pair_kernel<__half, true, false>,          (const void*)gemm_pair_kernel<__half, true, true>,
        (const void*)gemm_pair_kernel<__nv_bfloat16, false, false>, (const void*)gemm_pair_kernel<__nv_bfloat16, false, true>,
        (const void*)gemm_pair_kernel<__nv_bfloat16, true, false>,  (const void*)gemm_pair_kernel<__nv_bfloat16, true, true>};
    for (const void* k : kerns) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PR_SMEM) != cudaSuccess) {
            cudaGetLastError();
            ds->pair_clusters = -1;
            return 0;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (ds->sm_count / 2), 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = PR_SMEM;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kerns[1], &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        ds->pair_clusters = -1;
        return 0;
    }
    ds->pair_clusters = n;
    return (uint32_t)n;
}

template <typename T, int BN, int CPS>
int dispatch_major_c(bool ta, bool tb, const CUtensorMap& mA, const CUtensorMap& mB, T* C, uint32_t batch, uint32_t M,
                     uint32_t N, uint32_t K, uint64_t sC, int bA, int bB, int acc, int bf, int gelu, const QkvRope& qr,
                     cudaStream_t st) {
    if (!ta && !tb)
        return launch_tc<T, BN, false, true, CPS>(mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
    if (!ta && tb)
        return launch_tc<T, BN, false, false, CPS>(mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
    if (ta && !tb)
        return launch_tc<T, BN, true, true, CPS>(mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
    return launch_tc<T, BN, true, false, CPS>(mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
}

template <typename T, int BN>
int dispatch_major(bool ta, bool tb, const CUtensorMap& mA, const CUtensorMap& mB, T* C, uint32_t batch, uint32_t M,
                   uint32_t N, uint32_t K, uint64_t sC, int bA, int bB, int acc, int bf, int gelu, const QkvRope& qr,
                   cudaStream_t st) {
    // Long K with narrow N (the MLP down-projections): one CTA per SM, whose
    // deeper ring wins (measured 1.42 vs 1.25 PFLOP/s at 16384x8192x2048);
    // otherwise two, overlapping epilogues (1.32 vs 1.29 at 8192^3).
    if (K >= 8192 && N <= 4096)
        return dispatch_major_c<T, BN, 1>(ta, tb, mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
    return dispatch_major_c<T, BN, 2>(ta, tb, mA, mB, C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
}

template <typename T>
int launch_gemv(const T* X, const T* W, T* Y, uint32_t Mt, uint32_t K, uint32_t N, bool tb, int acc, int gelu,
                const QkvRope& qr, cudaStream_t st) {
    const int dtype = std::is_same<T, __nv_bfloat16>::value ? EVKCU_BF16 : EVKCU_F16;
    GemvEpilogue ep;
    ep.acc = acc;
    ep.gelu = gelu;
    if (tb) return launch_gemv_tc<T, true>(X, W, Y, Mt, K, N, ep, dtype, st, GemvArgmax(), GemvAllReduce(), qr);
    return launch_gemv_tc<T, false>(X, W, Y, Mt, K, N, ep, dtype, st, GemvArgmax(), GemvAllReduce(), qr);
}

}  // namespace

}  // namespace evkcu

using namespace evkcu;

namespace evkcu {

int rope_table(float2* cs, uint32_t len, uint32_t Dh, float base, cudaStream_t st) {
    const uint64_t n = (uint64_t)len * (Dh / 2);
    if (n == 0) return EVKCU_OK;
    rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(cs, len, Dh, base);
    return after_launch("rope table");
}

int matmul_ex(const void* A, const void* B, void* C, uint32_t batch, uint32_t M, uint32_t K, uint32_t N,
              uint64_t stride_a, uint64_t stride_b, uint64_t stride_c, uint32_t flags, int dtype, int gelu,
              void* stream, const QkvRope* qkv) {
    const QkvRope qr = qkv ? *qkv : QkvRope();
    if (qkv) {
        EVKCU_CHECK_ARG(qkv->q && qkv->kc && qkv->vc && qkv->Dh % 8 == 0 && qkv->Dh / 2 <= 128 && qkv->S > 0 &&
                            N == (qkv->Hq + 2 * qkv->Hk) * qkv->Dh && batch == 1 && !(flags & EVKCU_MM_ACC_C),
                        EVKCU_BAD_ARG, "matmul_ex: bad fused QKV arguments");
    }
    if (batch == 0 || M == 0 || N == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(A && B && C, EVKCU_BAD_ARG, "evkcu_matmul: null pointer");
    EVKCU_CHECK_ARG(dtype == EVKCU_F16 || dtype == EVKCU_BF16, EVKCU_BAD_ARG, "evkcu_matmul: unknown dtype");
    const bool ta = flags & EVKCU_MM_TRANSPOSE_A, tb = flags & EVKCU_MM_TRANSPOSE_B;
    const int acc = (flags & EVKCU_MM_ACC_C) ? 1 : 0;
    cudaStream_t st = as_stream(stream);
    DeviceState* ds = state();
    EVKCU_CHECK_ARG(ds, EVKCU_CUDA_ERROR, "evkcu_matmul: no device state");
    EVKCU_CHECK_ARG(N % 8 == 0, EVKCU_BAD_SHAPE, "evkcu_matmul: N must be a multiple of 8");
    EVKCU_CHECK_ARG(stride_c % 8 == 0 || batch == 1, EVKCU_BAD_ALIGN, "evkcu_matmul: C batch stride must be a multiple of 8");
    EVKCU_CHECK_ARG(aligned16(A) && aligned16(B) && aligned16(C), EVKCU_BAD_ALIGN,
                    "evkcu_matmul: base pointers must be 16-byte aligned");
    if (K == 0) {
        if (acc) return EVKCU_OK;
        for (uint32_t b = 0; b < batch; ++b)
            EVKCU_CUDA_TRY(cudaMemsetAsync((char*)C + (uint64_t)b * stride_c * 2, 0, (uint64_t)M * N * 2, st));
        return EVKCU_OK;
    }
    EVKCU_CHECK_ARG(K % 8 == 0 && (!ta || M % 8 == 0), EVKCU_BAD_SHAPE,
                    "evkcu_matmul: the contiguous dimension of A and B must be a multiple of 8");
    const int bf = dtype == EVKCU_BF16 ? 1 : 0;

    // Small-M (decode) path: B shared by the whole batch, A rows contiguous.
    const bool a_contig = batch == 1 || stride_a == (uint64_t)M * K;
    const bool c_contig = batch == 1 || stride_c == (uint64_t)M * N;
    const uint64_t Mt = (uint64_t)batch * M;
    if (!ta && Mt <= kGemvMaxM && (batch == 1 || stride_b == 0) && a_contig && c_contig) {
        return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
            return launch_gemv<T>((const T*)A, (const T*)B, (T*)C, (uint32_t)Mt, K, N, tb, acc, gelu, qr, st);
        });
    }

    const int bA = (batch > 1 && stride_a == 0) ? 1 : 0;
    const int bB = (batch > 1 && stride_b == 0) ? 1 : 0;
    EVKCU_CHECK_ARG(bA || batch == 1 || stride_a % 8 == 0, EVKCU_BAD_ALIGN, "evkcu_matmul: A batch stride % 8");
    EVKCU_CHECK_ARG(bB || batch == 1 || stride_b % 8 == 0, EVKCU_BAD_ALIGN, "evkcu_matmul: B batch stride % 8");

    // Tile width: the widest BN that still yields >= one wave of CTAs.
    const uint64_t mt = (M + BM - 1) / BM;
    auto tiles = [&](uint32_t bn) { return mt * ((N + bn - 1) / bn) * batch; };
    int BN = 64;
    if (tiles(256) >= (uint64_t)ds->sm_count) BN = 256;
    else if (tiles(128) >= (uint64_t)ds->sm_count) BN = 128;

    CUtensorMap mA, mB;
    const uint32_t zA = bA ? 1 : batch, zB = bB ? 1 : batch;
    // Paired-SM kernel for large outputs: 256 x 256 tiles, at least one
    // tile per resident pair.
    const uint64_t pair_tiles = (uint64_t)((M + 255) / 256) * ((N + 255) / 256) * batch;
    const bool pair_shape = ds->gemm_pair != 0 && !ds->plain_epilogue && M >= 256 &&
                            (ds->gemm_pair == 1 || pair_tiles >= (uint64_t)(ds->sm_count / 2));
    int r;
    if (!ta)
        r = make_tmap_3d(&mA, A, K, M, zA, K, (zA > 1 ? stride_a : (uint64_t)M * K), BK, BM, dtype);
    else
        r = make_tmap_3d(&mA, A, M, K, zA, M, (zA > 1 ? stride_a : (uint64_t)M * K), 64, BK, dtype);
    if (r) return r;
    if (!tb)
        r = make_tmap_3d(&mB, B, N, K, zB, N, (zB > 1 ? stride_b : (uint64_t)K * N), 64, BK, dtype);
    else
        r = make_tmap_3d(&mB, B, K, N, zB, K, (zB > 1 ? stride_b : (uint64_t)K * N), BK, BN, dtype);
    if (r) return r;
    const uint64_t sC = batch > 1 ? stride_c : 0;
    if (pair_shape) {
        const uint32_t clusters = pair_clusters();
        CUtensorMap tc, tk, tv;
        int tma_c = 0;
        r = make_c_maps(tc, tk, tv, C, batch, M, N, sC, qr, bf, &tma_c);
        if (r) return r;
        if (clusters && tma_c) {
            CUtensorMap mBp = mB;
            if (tb) {  // K-major B: one CTA holds 128 rows of it
                r = make_tmap_3d(&mBp, B, K, N, zB, K, (zB > 1 ? stride_b : (uint64_t)K * N), BK, 128, dtype);
                if (r) return r;
            }
            return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
                if (!ta && !tb)
                    return launch_pair<T, false, true>(mA, mBp, tc, tk, tv, tma_c, batch, M, N, K, bA, bB, acc, bf,
                                                       gelu, qr, clusters, st);
                if (!ta && tb)
                    return launch_pair<T, false, false>(mA, mBp, tc, tk, tv, tma_c, batch, M, N, K, bA, bB, acc, bf,
                                                        gelu, qr, clusters, st);
                if (ta && !tb)
                    return launch_pair<T, true, true>(mA, mBp, tc, tk, tv, tma_c, batch, M, N, K, bA, bB, acc, bf,
                                                      gelu, qr, clusters, st);
                return launch_pair<T, true, false>(mA, mBp, tc, tk, tv, tma_c, batch, M, N, K, bA, bB, acc, bf, gelu,
                                                   qr, clusters, st);
            });
        }
    }
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (BN == 256)
            return dispatch_major<T, 256>(ta, tb, mA, mB, (T*)C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
        if (BN == 128)
            return dispatch_major<T, 128>(ta, tb, mA, mB, (T*)C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
        return dispatch_major<T, 64>(ta, tb, mA, mB, (T*)C, batch, M, N, K, sC, bA, bB, acc, bf, gelu, qr, st);
    });
}

int gemv_allreduce_residual(const void* X, const void* W, void* Y, uint32_t Mt, uint32_t K, uint32_t N,
                            const GemvAllReduce& ar, int dtype, cudaStream_t st) {
    if (Mt == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(X && W && Y && ar.epoch && ar.tp >= 2 && ar.tp <= 8 && ar.rank < ar.tp, EVKCU_BAD_ARG,
                    "gemv_allreduce_residual: bad arguments");
    EVKCU_CHECK_ARG(Mt <= (uint32_t)kGemvMaxM && K > 0 && K % 8 == 0 && N > 0 && N % 8 == 0, EVKCU_BAD_SHAPE,
                    "gemv_allreduce_residual: needs 1..16 rows and K, N multiples of 8");
    GemvArgmax am;
    am.write_y = 0;  // y is written by the all-reduce tail
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        GemvEpilogue ep;
        return launch_gemv_tc<T, false>((const T*)X, (const T*)W, (T*)Y, Mt, K, N, ep, dtype, st, am, ar);
    });
}

int gemv_argmax(const void* X, const void* W, uint32_t Mt, uint32_t K, uint32_t N, bool w_kmajor, uint32_t key_off,
                unsigned long long* keys_out, uint32_t* ids_out, void* y_out, int dtype, cudaStream_t st) {
    if (Mt == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(X && W && (keys_out || ids_out), EVKCU_BAD_ARG, "gemv_argmax: null pointer");
    EVKCU_CHECK_ARG(Mt <= (uint32_t)kGemvMaxM && K > 0 && K % 8 == 0 && N > 0 && N % 8 == 0, EVKCU_BAD_SHAPE,
                    "gemv_argmax: needs 1..16 rows and K, N multiples of 8");
    EVKCU_CHECK_ARG(aligned16(X) && aligned16(W) && (!y_out || aligned16(y_out)), EVKCU_BAD_ALIGN,
                    "gemv_argmax: unaligned pointer");
    GemvArgmax am;
    am.keys_out = keys_out;
    am.ids_out = ids_out;
    am.key_off = key_off;
    am.write_y = y_out ? 1 : 0;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        GemvEpilogue ep;
        if (w_kmajor)
            return launch_gemv_tc<T, true>((const T*)X, (const T*)W, (T*)y_out, Mt, K, N, ep, dtype, st, am);
        return launch_gemv_tc<T, false>((const T*)X, (const T*)W, (T*)y_out, Mt, K, N, ep, dtype, st, am);
    });
}

}  // namespace evkcu

extern "C" int evkcu_matmul(const void* A, const void* B, void* C, uint32_t batch, uint32_t M, uint32_t K, uint32_t N,
                            uint64_t stride_a, uint64_t stride_b, uint64_t stride_c, uint32_t flags, int dtype,
                            void* stream) {
    return matmul_ex(A, B, C, batch, M, K, N, stride_a, stride_b, stride_c, flags, dtype, 0, stream);
}

// Diagnostic export (not in the public header): CTA pairs of the paired-SM
// GEMM resident at once on the current device; 0 if it cannot run there, -1
// if EVKCU_GEMM_PAIR=0 turned it off.
extern "C" int evkcu_debug_gemm_pair_clusters(void) {
    DeviceState* ds = state();
    if (!ds) return 0;
    if (ds->gemm_pair == 0) return -1;
    return (int)pair_clusters();
}
