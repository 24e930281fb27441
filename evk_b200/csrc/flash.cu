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
// tcgen05 kernel (Dh = 64 or 128): one CTA per NT consecutive 128-query
// tiles of one (batch, head); see flash_tc_kernel for the warp roles.  S, O
// and P live in TMEM (P is the TMEM-resident A operand of the PV MMA, so
// shared-memory bandwidth is left to the Q/K/V operands); O is rescaled lazily (FlashAttention-4 style) only when a row's
// running max grows by more than 2^8.  Causal tiles stop at the diagonal
// block; only diagonal / ragged blocks evaluate the mask.
//
// Any other Dh (multiple of 16, <= 256) runs a CUDA-core kernel (one warp per
// query row) with the same semantics.
#include <float.h>

#include <algorithm>

#include "sm100.cuh"

namespace evkcu {
namespace {

using namespace sm100;

constexpr int FM = 128;  // queries per tile (one TMEM lane per query)
constexpr uint32_t kTimeoutFlash = 0x201;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// NT query tiles per CTA, each with its own softmax warpgroup, share every
// K/V block of FN_ keys: while one tile's softmax runs, the tensor core works
// on another's S or PV.  POLY_ of every 8 scores take their exponential from a
// polynomial on the FMA pipe instead of the MUFU unit (ex2_poly2).
//   Dh = 64:  four tiles over 64-key blocks: four softmax warps share each SM
//             sub-partition, so one tile's exponentials overlap the others'
//             row max, P store and barrier waits.
//   Dh = 128: two tiles over 128-key blocks.
template <int DH, int NT, int FN_, int POLY_ = 0, bool QT_ = false, int CH_ = 1>
struct FlashCfg {
    static constexpr int FN = FN_;    // keys per block
    static constexpr int POLY = POLY_;
    // Column halves: with CH = 2 each tile's softmax is two warpgroups, one
    // per half of the S (and O) columns, so four softmax warps share each SM
    // sub-partition; the halves exchange row maxima (and, at the end, row
    // sums) through shared memory under a 64-thread named barrier.
    static constexpr int CH = CH_;
    // Q in TMEM: the softmax warps store their Q rows into TMEM once per
    // item and the S MMA reads its A operand from there (A from shared
    // memory costs a 128 x 16 operand fetch per MMA: 102 vs 73 clocks for
    // M = 128, N = 128, K = 16, measured).
    static constexpr bool QT = QT_;
    static constexpr int Q_BYTES = FM * DH * 2;  // per tile
    static constexpr int KV_BYTES = FN * DH * 2;  // one K or V block
    static constexpr int STAGES =
        NT == 4 ? 8 : NT == 2 ? (DH == 64 ? 5 : (FN == 64 ? 4 : 2)) : (DH == 64 ? 6 : 3);
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int TSTRIDE = TMEM_COLS / NT;  // TMEM columns per tile
    // Per tile t: S (fp32, FN columns), O (fp32, DH columns) and P (FN 16-bit
    // values packed two per column, FN/2 columns).  When the three do not fit
    // the tile's share of TMEM, P is written over the tile's S, and S_t(j + 1)
    // waits until PV_t(j) has read it.
    static constexpr int QCOLS = QT ? DH / 2 : 0;  // Q as packed 16-bit pairs
    static constexpr bool ALIAS_P = FN + DH + FN / 2 + QCOLS > TSTRIDE;
    static_assert(FN + DH + QCOLS <= TSTRIDE, "S, O (and Q) must fit the tile's TMEM share");
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + (QT ? 0 : NT * Q_BYTES);
    static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
    static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
    static constexpr int BAR_BYTES = ((2 + 3 * STAGES + 10 * NT) * 8 + 16 + 127) / 128 * 128;
    static constexpr int OFF_X = OFF_BAR + BAR_BYTES;  // CH = 2: row max / sum exchange
    static constexpr int X_BYTES = CH == 2 ? (2 + 1) * NT * CH * FM * 4 : 0;
    static constexpr int SMEM = OFF_X + X_BYTES + 1024;
    static constexpr int THREADS = 128 + NT * CH * 128;
    static __device__ __forceinline__ uint32_t col_s(int t) { return t * TSTRIDE; }
    static __device__ __forceinline__ uint32_t col_o(int t) { return t * TSTRIDE + FN; }
    static __device__ __forceinline__ uint32_t col_p(int t) { return ALIAS_P ? t * TSTRIDE : t * TSTRIDE + FN + DH; }
    static __device__ __forceinline__ uint32_t col_q(int t) { return t * TSTRIDE + FN + DH; }
};
static_assert(FlashCfg<64, 2, 128>::SMEM <= 227 * 1024 && FlashCfg<128, 2, 128>::SMEM <= 227 * 1024 &&
                  FlashCfg<64, 4, 64>::SMEM <= 227 * 1024 && FlashCfg<64, 2, 128, 0, true>::SMEM <= 227 * 1024 &&
                  FlashCfg<64, 2, 128, 0, false, 2>::SMEM <= 227 * 1024 && FlashCfg<128, 2, 64>::SMEM <= 227 * 1024,
              "flash smem");

// Phase trace (build with -DEVK_FLASH_TRACE only): clock64 stamps of CTA 0's
// first item, read back with evkcu_debug_flash_trace.  Slots 0 / 1: softmax
// tile 0 / 1 (row group 0), 2: S issuer, 3: PV issuer; [block][event].
#ifdef EVK_FLASH_TRACE
__device__ unsigned long long g_ftrace[4][64][8];
#define FTRACE(slot, blk, ev)                                                              \
    do {                                                                                   \
        if (blockIdx.x == 0 && (threadIdx.x & 31) == 0 && (blk) < 64) g_ftrace[slot][blk][ev] = clock64(); \
    } while (0)
#else
#define FTRACE(slot, blk, ev) \
    do {                      \
    } while (0)
#endif

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32x2 arithmetic (sm_100): two lanes of work per issued instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
          "l"(*reinterpret_cast<uint64_t*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

// 2^x for a pair of x <= 0 on the FMA pipe (packed fp32x2), for the scores
// whose exponential is not taken from MUFU.  Standard range reduction: with
// x clamped to >= -126, t = x + 1.5 * 2^23 holds round(x) = j in its low
// mantissa bits, f = x - j lies in [-1/2, 1/2], 2^f comes from a degree-3
// polynomial, and j is added to the result's exponent field as an integer
// (t's bits << 23 keep exactly j * 2^23 modulo 2^32).  The coefficients are a
// minimax fit of 2^f on [-1/2, 1/2] in relative error (Lawson's iteratively
// reweighted least squares, computed for this kernel): maximum relative error
// 7.5e-5, below half a storage ulp of P in fp16 (2.4e-4).  -inf (a masked
// score) gives about 2^-126, which rounds to 0 in P.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    constexpr float kC0 = 0.9999280571937561f, kC1 = 0.6932609677314758f, kC2 = 0.24261116981506348f,
                    kC3 = 0.0551716648042202f;
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 t = fadd2(x, make_float2(kShift, kShift));
    const float2 j = fadd2(t, make_float2(-kShift, -kShift));
    const float2 f = ffma2(j, make_float2(-1.0f, -1.0f), x);
    float2 p = ffma2(f, make_float2(kC3, kC3), make_float2(kC2, kC2));
    p = ffma2(p, f, make_float2(kC1, kC1));
    p = ffma2(p, f, make_float2(kC0, kC0));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// Persistent kernel: one CTA per SM walks work items in zig-zag rounds
// (see item_of); an item is NT consecutive 128-query tiles of
// one (batch, head), heaviest causal items first.  Barriers, TMEM and the
// K/V ring live for the whole kernel, so the next item's Q and K/V loads
// overlap the current item's last blocks and epilogue.
//   warp 0       TMA producer: per item, Q tiles (once the previous item's S
//                MMAs are done: q_empty), then K_j / V_j into a STAGES ring
//                whose index runs across items.
//   warp 1       TMEM owner + S issuer: S_t(j) = Q_t K_j^T once K_j is
//                loaded and softmax t has read S_t(j-1).
//   warp 2       PV issuer: O_t += P_t(j) V_j once P_t(j) is in TMEM (the
//                first PV of an item also waits until the previous item's O_t
//                was read out).  tcgen05.mma issue holds the issuing thread
//                for about the MMAs' execution time, so the two streams get
//                their own warps and neither waits behind the other.
//   warp 3       idle.
//   warpgroup 1+t  softmax of tile t, one thread per query row (= TMEM lane):
//                one TMEM load of the S row, row max, P = exp2 packed to
//                16-bit pairs and stored to TMEM (the A operand of the PV
//                MMA), lazy rescale of the O row in TMEM only when the running
//                max grows by > 2^8, finally O / l from TMEM to global memory.
// Every barrier is waited on (or probed) for exactly one completion at a time,
// and each barrier's next completion depends on the waiter having acted, so
// parity waits are unambiguous across items.
template <typename T, typename Cfg, int DH, int NT>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const T* __restrict__ Qg, T* __restrict__ O, uint32_t N,
                    uint32_t H,
                    uint32_t Hkv, uint32_t BH, float scale_log2, int causal, uint32_t idesc_s, uint32_t idesc_pv,
                    unsigned int* err) {
    constexpr int ST = Cfg::STAGES;
    constexpr int FN = Cfg::FN;
    // Four tiles (P aliased over S): each P chunk goes to TMEM as soon as it
    // is packed.  Two tiles: P is stored after the wait for PV_t(j - 1).
    constexpr bool kEarlyP = Cfg::ALIAS_P && NT == 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Cfg::OFF_Q;
    uint8_t* sK = smem + Cfg::OFF_K;
    uint8_t* sV = smem + Cfg::OFF_V;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* q_empty = q_full + 1;
    uint64_t* k_full = q_empty + 1;     // [ST]
    uint64_t* v_full = k_full + ST;     // [ST]
    uint64_t* kv_empty = v_full + ST;   // [ST]
    uint64_t* s_full = kv_empty + ST;   // [NT]
    uint64_t* s_free = s_full + NT;     // [NT]
    uint64_t* p_full = s_free + NT;     // [NT]
    uint64_t* pv_done = p_full + NT;    // [NT]
    uint64_t* o_free = pv_done + NT;    // [NT]
    uint64_t* q_tm = o_free + NT;       // [NT] Q_t stored in TMEM (Cfg::QT)
    uint64_t* x_bar = q_tm + NT;        // [NT * 4] column-half pairs exchanged a value (Cfg::CH = 2)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(x_bar + 4 * NT);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t kv_all = (N + FN - 1) / FN;
    const uint32_t qtiles = (N + FM - 1) / FM;
    const uint32_t ngroups = (qtiles + NT - 1) / NT;
    const uint32_t items = ngroups * BH;
    // Work item -> (b, h, q0[t], nblk[t]); groups ordered heaviest first.
    auto item_geom = [&](uint32_t w, uint32_t& b, uint32_t& h, uint32_t (&q0)[NT], uint32_t (&nblk)[NT]) {
        const uint32_t grp = ngroups - 1 - w / BH;
        const uint32_t bh = w % BH;
        b = bh / H;
        h = bh % H;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            q0[t] = (grp * NT + t) * FM;
            nblk[t] = q0[t] < N ? (causal ? min(kv_all, (q0[t] + FM + FN - 1) / FN) : kv_all) : 0;
        }
    };

    // Round rd of this CTA takes item rd*G + (c or G-1-c, alternating): a
    // zig-zag over the heaviest-first order keeps the per-CTA sums of causal
    // work within a few percent of each other.
    auto item_of = [&](uint32_t rd) -> uint32_t {
        return rd * gridDim.x + ((rd & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
    };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 2);
        }
        for (int t = 0; t < NT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&s_free[t], 4 * Cfg::CH);
            mbar_init(&p_full[t], 4 * Cfg::CH);
            mbar_init(&pv_done[t], 1);
            mbar_init(&o_free[t], 4 * Cfg::CH);
            mbar_init(&q_tm[t], 4 * Cfg::CH);
            for (int qq = 0; qq < 4; ++qq) mbar_init(&x_bar[4 * t + qq], 2);
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
    // NT = 4: 640 threads leave 96 registers a thread at launch; the control
    // warpgroup (producer, issuers) hands registers to the softmax
    // warpgroups: 128 * 64 + 512 * 104 = 61,440 = 640 * 96.
    if (warp < 4) {
    if constexpr (Cfg::THREADS == 640) asm volatile("setmaxnreg.dec.sync.aligned.u32 64;\n" ::: "memory");
    if (warp == 0) {
        // ------------------------------------------------ TMA producer ----
        if (lane == 0) {
            uint32_t r = 0, it = 0;  // ring index and item count across items
            bool ok = true;
            for (uint32_t rd = 0; ok && rd * gridDim.x < items; ++rd) {
                const uint32_t w = item_of(rd);
                if (w >= items) continue;
                uint32_t b, h, q0[NT], nblk[NT];
                item_geom(w, b, h, q0, nblk);
                uint32_t nmax = 0;
#pragma unroll
                for (int t = 0; t < NT; ++t) nmax = max(nmax, nblk[t]);
                const uint32_t g = h / (H / Hkv);
                if constexpr (!Cfg::QT) {
                    // Q buffer is free once the previous item's S MMAs completed.
                    if (it > 0 && !mbar_wait(q_empty, (it - 1) & 1, s_abort, err, kTimeoutFlash)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(q_full, NT * Cfg::Q_BYTES);
#pragma unroll
                    for (int t = 0; t < NT; ++t)
#pragma unroll
                        for (int c = 0; c < DH / 64; ++c)
                            tma_load_3d(sQ + t * Cfg::Q_BYTES + c * FM * 128, &tmQ, q_full, (int)(h * DH + c * 64),
                                        (int)q0[t], (int)b);
                }
                ++it;
                for (uint32_t j = 0; j < nmax; ++j, ++r) {
                    const int st = r % ST;
                    if (!mbar_wait(&kv_empty[st], ((r / ST) & 1) ^ 1, s_abort, err, kTimeoutFlash)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&k_full[st], Cfg::KV_BYTES);
#pragma unroll
                    for (int c = 0; c < DH / 64; ++c)
                        tma_load_3d(sK + st * Cfg::KV_BYTES + c * FN * 128, &tmK, &k_full[st], (int)(g * DH + c * 64),
                                    (int)(j * FN), (int)b);
                    mbar_arrive_expect_tx(&v_full[st], Cfg::KV_BYTES);
#pragma unroll
                    for (int c = 0; c < DH / 64; ++c)
                        tma_load_3d(sV + st * Cfg::KV_BYTES + c * FN * 128, &tmV, &v_full[st], (int)(g * DH + c * 64),
                                    (int)(j * FN), (int)b);
                }
            }
        }
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------ MMA issuers ----
        // Warp 1 issues every S MMA, warp 2 every PV MMA, each in a static
        // order over the item's blocks.  S_t(j) waits for K_j and for softmax
        // t to have read S_t(j-1); PV_t(j) waits for P_t(j), V_j and (first
        // block of an item) for O_t to have been read out.  The two streams
        // write disjoint TMEM (S vs O) and meet only through the softmax
        // barriers, so neither waits behind the other's events.  Waits block
        // (lane 0 sleeps in try_wait, the other lanes at the broadcast), one
        // elected lane issues.  A ring slot is released by one commit from
        // each issuer (kv_empty counts 2).
        const bool is_s = warp == 1;
        const bool leader = elect_one();
        uint64_t* const s_reuse = Cfg::ALIAS_P ? pv_done : s_free;  // S_t(j) waits on this for j - 1
        const uint32_t qaddr = smem_u32(sQ);
        uint32_t rbase = 0, it = 0;
        uint32_t gs[NT], ep[NT];  // per tile: blocks processed before this item, epilogues finished
#pragma unroll
        for (int t = 0; t < NT; ++t) gs[t] = ep[t] = 0;
        bool ok = true;
        auto probe = [&](bool c) { return __shfl_sync(0xffffffffu, (int)c, 0) != 0; };
        for (uint32_t rd = 0; ok && rd * gridDim.x < items; ++rd) {
            const uint32_t w = item_of(rd);
            if (w >= items) continue;
            uint32_t b, h, q0[NT], nblk[NT];
            item_geom(w, b, h, q0, nblk);
            uint32_t nmax = 0;
#pragma unroll
            for (int t = 0; t < NT; ++t) nmax = max(nmax, nblk[t]);
            if (!Cfg::QT && is_s && !probe(lane == 0 && mbar_wait(q_full, it & 1, s_abort, err, kTimeoutFlash)))
                break;
            tc_fence_after();
            for (uint32_t j = 0; ok && j < nmax; ++j) {
                const uint32_t r = rbase + j;
                if (is_s) {
                    ok = probe(lane == 0 && mbar_wait(&k_full[r % ST], (r / ST) & 1, s_abort, err, kTimeoutFlash));
                    const uint32_t kaddr = smem_u32(sK + (r % ST) * Cfg::KV_BYTES);
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const uint32_t gj = gs[t] + j;  // tile-global block index
                        if (!ok || j >= nblk[t]) continue;
                        // S_t(j) overwrites S_t(j - 1): softmax t must have
                        // read it, and with P aliased into S, PV_t(j - 1)
                        // must have read P (which also implies the former).
                        if (it == 0) FTRACE(2, j, 2 * t);
                        ok = gj == 0 || probe(lane == 0 && mbar_wait(&s_reuse[t], (gj - 1) & 1, s_abort, err,
                                                                     kTimeoutFlash));
                        // Q in TMEM: the first S of an item waits until
                        // softmax t has stored the item's Q rows.
                        if (Cfg::QT && ok && j == 0)
                            ok = probe(lane == 0 && mbar_wait(&q_tm[t], ep[t] & 1, s_abort, err, kTimeoutFlash));
                        if (!ok) break;
                        tc_fence_after();
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < DH / 16; ++kk) {
                                uint64_t bd = make_sw128_desc(kaddr + (kk >> 2) * (FN * 128) + (kk & 3) * 32, 16, 1024);
                                if constexpr (Cfg::QT) {
                                    mma_f16_ts(tmem + Cfg::col_s(t), tmem + Cfg::col_q(t) + kk * 8, bd, idesc_s,
                                               kk != 0);
                                } else {
                                    uint64_t ad = make_sw128_desc(
                                        qaddr + t * Cfg::Q_BYTES + (kk >> 2) * (FM * 128) + (kk & 3) * 32, 16, 1024);
                                    mma_f16_ss(tmem + Cfg::col_s(t), ad, bd, idesc_s, kk != 0);
                                }
                            }
                            mma_commit(&s_full[t]);
                        }
                        __syncwarp();
                        if (it == 0) FTRACE(2, j, 2 * t + 1);
                    }
                    if (!ok) break;
                    // Q is free once every S of this item has completed.
                    if (!Cfg::QT && j + 1 == nmax && leader) mma_commit(q_empty);
                } else {
                    ok = probe(lane == 0 && mbar_wait(&v_full[r % ST], (r / ST) & 1, s_abort, err, kTimeoutFlash));
                    const uint32_t vaddr = smem_u32(sV + (r % ST) * Cfg::KV_BYTES);
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const uint32_t gj = gs[t] + j;
                        if (!ok || j >= nblk[t]) continue;
                        if (it == 0) FTRACE(3, j, 2 * t);
                        ok = probe(lane == 0 && mbar_wait(&p_full[t], gj & 1, s_abort, err, kTimeoutFlash) &&
                                   (j != 0 || ep[t] == 0 ||
                                    mbar_wait(&o_free[t], (ep[t] - 1) & 1, s_abort, err, kTimeoutFlash)));
                        if (!ok) break;
                        tc_fence_after();
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < FN / 16; ++kk) {
                                // A = P_t from TMEM: 16 keys = 8 packed columns per MMA.
                                uint64_t bd = make_sw128_desc(vaddr + kk * 2048, FN * 128, 1024);
                                mma_f16_ts(tmem + Cfg::col_o(t), tmem + Cfg::col_p(t) + kk * 8, bd, idesc_pv,
                                           (j | kk) != 0);
                            }
                            mma_commit(&pv_done[t]);
                        }
                        __syncwarp();
                        if (it == 0) FTRACE(3, j, 2 * t + 1);
                    }
                    if (!ok) break;
                }
                // This issuer is done with ring slot j once its MMAs complete.
                if (leader) mma_commit(&kv_empty[r % ST]);
                __syncwarp();
            }
            ++it;
            rbase += nmax;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                gs[t] += nblk[t];
                if (nblk[t] > 0) ++ep[t];
            }
        }
    }
    } else {
        if constexpr (Cfg::THREADS == 640) asm volatile("setmaxnreg.inc.sync.aligned.u32 104;\n" ::: "memory");
        // --------------------------------------------- softmax warps ----
        constexpr int CH = Cfg::CH;
        constexpr int SC = FN / CH;  // S columns of this warp
        constexpr int OC = DH / CH;  // O columns of this warp
        const int sidx = warp - 4;
        const int t = sidx / (4 * CH);
        const int half = (sidx / 4) % CH;
        const int quarter = warp & 3;
        const uint32_t row = quarter * 32 + lane;  // TMEM lane == query row in the tile
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        const uint32_t s_addr = lane_addr + Cfg::col_s(t) + half * SC;
        const uint32_t o_addr = lane_addr + Cfg::col_o(t) + half * OC;
        const uint32_t p_addr = lane_addr + Cfg::col_p(t) + half * (SC / 2);
        // CH = 2: exchange slots [parity][t][half][row] for maxima, then
        // [t][half][row] for the final row sums; the two warps of a row group
        // meet at mbarrier x_bar[4 t + quarter] (one arrival per warp, bounded
        // wait), xph counting its completed phases.
        float* xch = reinterpret_cast<float*>(smem + Cfg::OFF_X);
        uint64_t* const pair_bar = &x_bar[4 * t + quarter];
        uint32_t xph = 0;
        auto pair_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(pair_bar);
            return mbar_wait(pair_bar, (xph++) & 1, s_abort, err, kTimeoutFlash);
        };
        uint32_t gbase = 0;  // blocks this tile processed in earlier items
        bool ok = true;
        for (uint32_t rd = 0; ok && rd * gridDim.x < items; ++rd) {
            const uint32_t w = item_of(rd);
            if (w >= items) continue;
            uint32_t b, h, q0[NT], nblk[NT];
            item_geom(w, b, h, q0, nblk);
            const uint32_t nb = nblk[t];
            if (nb == 0) continue;
            const uint32_t qidx = q0[t] + row;
            const uint32_t kmax = min(N, causal ? qidx + 1 : N);  // keys < kmax are valid
            if constexpr (Cfg::QT) {
                // This row of Q_t into TMEM (16-bit pairs, the MMA's A
                // layout).  Every S MMA of the previous item has completed:
                // this warp consumed them all.
                uint32_t qw[DH / 2];
                const uint4* src = reinterpret_cast<const uint4*>(
                    Qg + ((uint64_t)b * N + (qidx < N ? qidx : 0)) * ((uint64_t)H * DH) + (uint64_t)h * DH);
#pragma unroll
                for (int c = 0; c < DH / 8; ++c) {
                    const uint4 v = qidx < N ? src[c] : make_uint4(0u, 0u, 0u, 0u);
                    qw[4 * c] = v.x;
                    qw[4 * c + 1] = v.y;
                    qw[4 * c + 2] = v.z;
                    qw[4 * c + 3] = v.w;
                }
#pragma unroll
                for (int c = 0; c < DH / 64; ++c) {
                    uint32_t (&chunk)[32] = *reinterpret_cast<uint32_t (*)[32]>(qw + 32 * c);
                    tmem_st32(lane_addr + Cfg::col_q(t) + 32 * c, chunk);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&q_tm[t]);
            }
            float m_ref = -INFINITY, l = 0.0f;
            for (uint32_t j = 0; j < nb; ++j) {
                const uint32_t gj = gbase + j;
                const bool trace = gbase == 0 && quarter == 0 && half == 0;
                if (trace) FTRACE(t, j, 0);
                if (!mbar_wait(&s_full[t], gj & 1, s_abort, err, kTimeoutFlash)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t sr[SC / 32][32];
                const uint32_t k0 = j * FN + half * SC;  // first key of this warp's columns
                const bool need_mask = (k0 + SC > N) || (causal && k0 + SC > q0[t] + 1);
                // Row max: three-input max, four independent accumulators.
                float mxa[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) mxa[i] = -INFINITY;
                {
#pragma unroll
                    for (int c = 0; c < SC / 32; ++c) tmem_ld32(s_addr + c * 32, sr[c]);
                    tmem_wait_ld();
                    // S is in registers: the tensor core may overwrite it with S_t(j+1).
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_free[t]);
                    if (trace) FTRACE(t, j, 2);
                    if (need_mask) {
#pragma unroll
                        for (int c = 0; c < SC / 32; ++c)
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                if (k0 + c * 32 + e >= kmax) sr[c][e] = __float_as_uint(-INFINITY);
                    }
#pragma unroll
                    for (int c = 0; c < SC / 32; ++c)
#pragma unroll
                        for (int e = 0; e < 32; e += 2)
                            mxa[(e >> 1) & 3] =
                                fmax3(mxa[(e >> 1) & 3], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
                }
                float mx = fmax3(fmaxf(mxa[0], mxa[1]), mxa[2], mxa[3]);
                if (trace) FTRACE(t, j, 3);
                if constexpr (CH == 2) {
                    // The other half's row maximum (same row, other columns).
                    float* slot = xch + (((gj & 1) * NT + t) * CH) * FM;
                    slot[half * FM + row] = mx;
                    if (!pair_sync()) {
                        ok = false;
                        break;
                    }
                    mx = fmaxf(mx, slot[(1 - half) * FM + row]);
                }
                const float m_cand = fmaxf(m_ref, mx * scale_log2);
                // Lazy rescale: keep the reference max unless it grew by > 2^8.
                const bool need = j > 0 && m_cand > m_ref + kRescaleThreshold;
                const float alpha = need ? ex2(m_ref - m_cand) : 1.0f;  // m_ref = -inf -> 0
                if (j == 0 || need) m_ref = m_cand;
                const float m_use = (m_ref == -INFINITY) ? 0.0f : m_ref;
                // p = exp2(s * scale_log2 - m) with packed fp32x2 scale-subtract
                // and sums, packed to 16-bit pairs in place (sr[c][0..15]).
                // This runs before waiting for PV_t(j-1), so the exponentials
                // overlap that MMA.
                const float2 sc2 = make_float2(scale_log2, scale_log2);
                const float2 nm2 = make_float2(-m_use, -m_use);
                float2 rs2[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) rs2[i] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int c = 0; c < SC / 32; ++c) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            // masked entries hold -inf: exp2(-inf) = 0
                            float2 x = ffma2(make_float2(__uint_as_float(sr[c][q * 8 + e]),
                                                         __uint_as_float(sr[c][q * 8 + e + 1])), sc2, nm2);
                            if (e < Cfg::POLY) {
                                const float2 y = ex2_poly2(x);
                                f[e] = y.x;
                                f[e + 1] = y.y;
                            } else {
                                f[e] = ex2(x.x);
                                f[e + 1] = ex2(x.y);
                            }
                            rs2[e >> 1] = fadd2(rs2[e >> 1], make_float2(f[e], f[e + 1]));
                        }
                        const Vec8 pk = pack8<T>(f);
#pragma unroll
                        for (int i = 0; i < 4; ++i) sr[c][q * 4 + i] = pk.w[i];
                    }
                    if constexpr (kEarlyP) {
                        // P over S: S_t(j) was issued only after PV_t(j - 1)
                        // completed, so P_t(j - 1) has been read; storing each
                        // chunk at once keeps fewer registers live.
                        uint32_t pw[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) pw[i] = sr[c][i];
                        tmem_st16(p_addr + c * 16, pw);
                    }
                }
                if (trace) FTRACE(t, j, 4);
                if (!kEarlyP && j > 0) {
                    // PV_t(j-1) must be complete before the P columns are
                    // overwritten and before O is rescaled.
                    if (!mbar_wait(&pv_done[t], (gj - 1) & 1, s_abort, err, kTimeoutFlash)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                if (trace) FTRACE(t, j, 5);
                const float rs = ((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) +
                                 ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y));
                l = l * alpha + rs;
                if (__any_sync(0xffffffffu, need)) {
                    // (PV_t(j - 1) is complete: waited above, or implied by
                    // S_t(j) when P is stored early over S.)
                    constexpr int RC = kEarlyP ? 16 : 32;  // columns per TMEM round trip
#pragma unroll
                    for (int c = 0; c < OC / RC; ++c) {
                        uint32_t rr[RC];
                        if constexpr (RC == 16) tmem_ld16(o_addr + c * RC, rr); else tmem_ld32(o_addr + c * RC, rr);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < RC; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
                        if constexpr (RC == 16) tmem_st16(o_addr + c * RC, rr); else tmem_st32(o_addr + c * RC, rr);
                    }
                }
                if constexpr (!kEarlyP) {
#pragma unroll
                    for (int c = 0; c < SC / 32; ++c) {
                        uint32_t pw[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) pw[i] = sr[c][i];
                        tmem_st16(p_addr + c * 16, pw);
                    }
                }
                // P and any O rescale (TMEM stores) must be complete before
                // the PV MMA is issued.
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[t]);
                if (trace) FTRACE(t, j, 6);
            }
            if (!ok) break;
            // Epilogue: O / l from TMEM to global memory, then O_t is free.
            const uint32_t glast = gbase + nb - 1;
            if (!mbar_wait(&pv_done[t], glast & 1, s_abort, err, kTimeoutFlash)) break;
            tc_fence_after();
            if constexpr (CH == 2) {
                // total row sum = both halves'
                float* slot = xch + (2 * NT * CH + t * CH) * FM;
                slot[half * FM + row] = l;
                if (!pair_sync()) break;
                l += slot[(1 - half) * FM + row];
            }
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            T* orow = O + ((uint64_t)b * N + qidx) * ((uint64_t)H * DH) + (uint64_t)h * DH + half * OC;
#pragma unroll
            for (int c = 0; c < OC / 32; ++c) {
                uint32_t rr[32];
                tmem_ld32(o_addr + c * 32, rr);
                tmem_wait_ld();
                if (qidx < N) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(rr[q * 8 + e]) * inv;
                        reinterpret_cast<Vec8*>(orow + c * 32)[q] = pack8<T>(f);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[t]);
            gbase += nb;
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
                                                         float scale_log2, int causal, uint64_t kv_bstride) {
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
        const T* krow = K + (uint64_t)b * kv_bstride + (uint64_t)j * Hkv * Dh + (uint64_t)g * Dh;
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
        const T* vrow = V + (uint64_t)b * kv_bstride + (uint64_t)j * Hkv * Dh + (uint64_t)g * Dh;
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

template <typename T, int DH, int NT, int FN, int POLY, bool QT = false, int CH = 1>
int launch_flash_tc(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N, uint32_t H,
                    uint32_t Hkv, float scale_log2, int causal, int dtype, uint64_t kv_bstride, cudaStream_t st) {
    using Cfg = FlashCfg<DH, NT, FN, POLY, QT, CH>;
    CUtensorMap mQ, mK, mV;
    int r;
    if ((r = make_tmap_3d(&mQ, q, (uint64_t)H * DH, N, B, (uint64_t)H * DH, (uint64_t)N * H * DH, 64, FM, dtype))) return r;
    // K/V rows beyond N read as zeros even when the batch stride leaves
    // memory there (a KV cache): the map's row extent is N.
    if ((r = make_tmap_3d(&mK, k, (uint64_t)Hkv * DH, N, B, (uint64_t)Hkv * DH, kv_bstride, 64, FN, dtype))) return r;
    if ((r = make_tmap_3d(&mV, v, (uint64_t)Hkv * DH, N, B, (uint64_t)Hkv * DH, kv_bstride, 64, FN, dtype))) return r;
    auto kern = flash_tc_kernel<T, Cfg, DH, NT>;
    static bool attr = false;
    if (!attr) {
        EVKCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
        if (Cfg::THREADS == 640) {
            // The setmaxnreg split (64 registers for the control warpgroup,
            // 104 for the four softmax warpgroups) must fit the registers the
            // block is launched with, or the increase would wait forever.
            cudaFuncAttributes fa{};
            EVKCU_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
            EVKCU_CHECK_ARG(fa.numRegs * Cfg::THREADS >= 128 * 64 + 512 * 104, EVKCU_CUDA_ERROR,
                            "evkcu_flash_attention: kernel built with too few registers for its register split");
        }
        attr = true;
    }
    const int bf = dtype == EVKCU_BF16 ? 1 : 0;
    const uint32_t idesc_s = make_idesc_f16(FM, FN, bf, 0, 0);
    const uint32_t idesc_pv = make_idesc_f16(FM, DH, bf, 0, 1);
    const uint32_t qtiles = (N + FM - 1) / FM;
    const uint64_t items = (uint64_t)B * H * ((qtiles + NT - 1) / NT);
    const unsigned grid = (unsigned)std::min<uint64_t>(items, (uint64_t)state()->sm_count);
    kern<<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(mQ, mK, mV, (const T*)q, (T*)o, N, H, Hkv, B * H, scale_log2, causal,
                                                idesc_s,
                                                idesc_pv, state()->d_error);
    return after_launch("evkcu_flash_attention(tcgen05)");
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

namespace evkcu {

// Dh = 64 kernel variant, read once from EVKCU_FLASH64 (for A/B
// measurement): 0 (default) two tiles over 128-key blocks, all exponentials
// on MUFU; 1 four tiles over 64-key blocks, a quarter of the exponentials on
// the FMA pipe; 2 four tiles, all on MUFU; 3 four tiles, half on the FMA pipe.
// (Four tiles lose at C2: each S MMA reads the whole 128-row Q tile from
// shared memory, which takes longer than its N = 64 columns of math.)
static int flash64_variant() {
    static const int v = [] {
        const char* e = getenv("EVKCU_FLASH64");
        return e ? atoi(e) : 0;
    }();
    return v;
}

// Dh = 128 variant (EVKCU_FLASH128, for A/B measurement): 0 (default) two
// tiles over 64-key blocks, S, O and P each in their own TMEM columns, so the
// next S MMA need not wait for the PV MMA that reads P (C4-shaped causal bf16:
// 174 us against 198 us); 1 two tiles over 128-key blocks with P written over S.
static int flash128_variant() {
    static const int v = [] {
        const char* e = getenv("EVKCU_FLASH128");
        return e ? atoi(e) : 0;
    }();
    return v;
}

int flash_attention_kv_strided(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N,
                               uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype,
                               uint64_t kv_bstride, cudaStream_t st) {
    if (B == 0 || N == 0 || H == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(q && k && v && o, EVKCU_BAD_ARG, "evkcu_flash_attention: null pointer");
    EVKCU_CHECK_ARG(dtype == EVKCU_F16 || dtype == EVKCU_BF16, EVKCU_BAD_ARG, "evkcu_flash_attention: unknown dtype");
    EVKCU_CHECK_ARG(Hkv >= 1 && H % Hkv == 0, EVKCU_BAD_SHAPE, "evkcu_flash_attention: H must be a multiple of Hkv");
    EVKCU_CHECK_ARG(Dh % 16 == 0 && Dh >= 16 && Dh <= 256, EVKCU_BAD_SHAPE,
                    "evkcu_flash_attention: Dh must be a multiple of 16 in [16, 256]");
    EVKCU_CHECK_ARG((uint64_t)B * H <= 0x7fffffffu && (N + FM - 1) / FM <= 65535, EVKCU_BAD_SHAPE,
                    "evkcu_flash_attention: grid too large");
    if (kv_bstride == 0) kv_bstride = (uint64_t)N * Hkv * Dh;
    EVKCU_CHECK_ARG(kv_bstride >= (uint64_t)N * Hkv * Dh, EVKCU_BAD_SHAPE,
                    "evkcu_flash_attention: K/V batch stride smaller than N rows");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)Dh);
    const float scale_log2 = scale * 1.4426950408889634f;
    const int causal = (flags & EVKCU_ATTN_CAUSAL) ? 1 : 0;
    const bool tma_ok = aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) && kv_bstride % 8 == 0;
    if (tma_ok && (Dh == 64 || Dh == 128)) {
        return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
            if (Dh == 64) {
                switch (flash64_variant()) {
                    case 1:
                        return launch_flash_tc<T, 64, 4, 64, 2>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype,
                                                                kv_bstride, st);
                    case 2:
                        return launch_flash_tc<T, 64, 4, 64, 0>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype,
                                                                kv_bstride, st);
                    case 3:
                        return launch_flash_tc<T, 64, 4, 64, 4>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype,
                                                                kv_bstride, st);
                    case 4:
                        return launch_flash_tc<T, 64, 2, 128, 0, true>(q, k, v, o, B, N, H, Hkv, scale_log2, causal,
                                                                       dtype, kv_bstride, st);
                    case 5:
                        return launch_flash_tc<T, 64, 2, 128, 2, true>(q, k, v, o, B, N, H, Hkv, scale_log2, causal,
                                                                       dtype, kv_bstride, st);
                    case 6:
                        return launch_flash_tc<T, 64, 2, 128, 0, false, 2>(q, k, v, o, B, N, H, Hkv, scale_log2,
                                                                           causal, dtype, kv_bstride, st);
                    case 7:
                        return launch_flash_tc<T, 64, 2, 128, 2, false, 2>(q, k, v, o, B, N, H, Hkv, scale_log2,
                                                                           causal, dtype, kv_bstride, st);
                    default:
                        return launch_flash_tc<T, 64, 2, 128, 0>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype,
                                                                 kv_bstride, st);
                }
            }
            if (flash128_variant() == 1)
                return launch_flash_tc<T, 128, 2, 128, 0>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype,
                                                          kv_bstride, st);
            return launch_flash_tc<T, 128, 2, 64, 0>(q, k, v, o, B, N, H, Hkv, scale_log2, causal, dtype, kv_bstride,
                                                     st);
        });
    }
    const uint64_t warps = (uint64_t)B * H * N;
    const uint64_t blocks = (warps * 32 + 255) / 256;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        flash_simt_kernel<T><<<(unsigned)blocks, 256, 0, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, B, N, H,
                                                              Hkv, Dh, scale_log2, causal, kv_bstride);
        return after_launch("evkcu_flash_attention(simt)");
    });
}

}  // namespace evkcu

#ifdef EVK_FLASH_TRACE
extern "C" int evkcu_debug_flash_trace(void* host) {
    return (int)cudaMemcpyFromSymbol(host, evkcu::g_ftrace, sizeof(evkcu::g_ftrace));
}
#endif

extern "C" int evkcu_flash_attention(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N,
                                     uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype,
                                     void* stream) {
    return flash_attention_kv_strided(q, k, v, o, B, N, H, Hkv, Dh, scale, flags, dtype, 0, as_stream(stream));
}
