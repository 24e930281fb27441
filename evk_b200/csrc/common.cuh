// common.cuh — shared host/device helpers of libevkcu (status handling,
// element types, launch accounting, bounded mbarrier waits).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/evkcu.h"

namespace evkcu {

// ---------------------------------------------------------------- status ----
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
void count_launch(uint32_t n = 1);

#define EVKCU_CHECK_ARG(cond, status, msg) \
    do {                                   \
        if (!(cond)) return ::evkcu::fail((status), (msg)); \
    } while (0)

#define EVKCU_CUDA_TRY(expr)                                   \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return ::evkcu::cuda_fail(_e, #expr); \
    } while (0)

// Checks the launch that was just enqueued and counts it.
inline int after_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    count_launch();
    return EVKCU_OK;
}

// ------------------------------------------ programmatic dependent launch ----
// Kernels on the decode path are launched with programmatic stream
// serialization: the next kernel may start while this one drains, runs its
// prologue (barrier setup, TMEM allocation, loads of constant weights) and
// then waits in pdl_wait() until every earlier kernel has completed and its
// writes are visible.  A kernel launched this way must not read data written
// by an earlier kernel, nor write data an earlier kernel reads, before
// pdl_wait().  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------ per-device state ----
// Scratch slots: each op family that needs global scratch owns one, so ops on
// different streams never share scratch.  Scratch is zero-filled when it is
// (re)allocated; kernels that use ticket counters leave them at zero.
enum WorkspaceSlot { WS_GEMV = 0, WS_DECODE = 1, WS_GREEDY = 2, WS_TRAIN = 3, WS_COUNT = 4 };

struct DeviceState {
    int device = -1;
    int sm_count = 0;
    unsigned int* d_error = nullptr;  // device error word for bounded waits
    void* ws[WS_COUNT] = {};
    size_t ws_bytes[WS_COUNT] = {};
    bool pdl = true;  // programmatic dependent launch for the decode-path kernels
    bool plain_epilogue = false;  // GEMM: per-row stores instead of the staged TMA epilogue
    int gemm_pair = -1;           // GEMM: paired-SM kernel (-1 by shape, 0 never, 1 whenever it applies)
    int pair_clusters = 0;        // resident CTA pairs of the paired-SM GEMM (0: not yet queried)
};
// Returns the state of the current device, creating it on first use.
DeviceState* state();
// Returns a zero-initialised scratch buffer of at least `bytes` for `slot` on
// the current device.  Growing it synchronises the device and reallocates, so
// the first call at a new maximum size must not happen during stream capture.
void* workspace(int slot, size_t bytes);

// Every scratch slot starts with a fixed ticket area (split reductions'
// atomic counters, left at zero by the kernels) followed by the partials, so
// calls with different grid shapes never see each other's partials as
// tickets.
constexpr size_t kTicketBytes = 256 * 1024;
constexpr uint32_t kMaxTickets = kTicketBytes / sizeof(unsigned int);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launches a kernel that calls pdl_wait() before its first dependent access,
// with programmatic stream serialization unless disabled for the device.
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    DeviceState* s = state();
    cfg.attrs = attr;
    cfg.numAttrs = (s && s->pdl) ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return after_launch(what);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// --------------------------------------------------------- element types ----
// Storage is 2-byte fp16 (reference) or bf16 (extension); arithmetic is fp32.
template <typename T> struct Elem;
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ float2 to_f2(__half2 x) { return __half22float2(x); }
    static __device__ __forceinline__ __half2 from_f2(float a, float b) { return __floats2half2_rn(a, b); }
    using T2 = __half2;
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float2 to_f2(__nv_bfloat162 x) { return __bfloat1622float2(x); }
    static __device__ __forceinline__ __nv_bfloat162 from_f2(float a, float b) { return __floats2bfloat162_rn(a, b); }
    using T2 = __nv_bfloat162;
};

// Dispatches a templated launcher on the runtime dtype.
#define EVKCU_DISPATCH_DTYPE(dtype, T, ...)                                   \
    [&]() -> int {                                                            \
        if ((dtype) == EVKCU_F16) { using T = __half; return __VA_ARGS__(); } \
        if ((dtype) == EVKCU_BF16) { using T = __nv_bfloat16; return __VA_ARGS__(); } \
        return ::evkcu::fail(EVKCU_BAD_ARG, "unknown dtype");                 \
    }()

// 16-byte vector of 8 two-byte elements.
struct __align__(16) Vec8 {
    uint32_t w[4];
};

// 16-byte shared-memory accesses (one LDS.128 / STS.128 each).
__device__ __forceinline__ Vec8 ld_shared_vec8(const void* p) {
    Vec8 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p)))
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_shared_vec8(void* p, const Vec8& v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))),
                 "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack8(const Vec8& v, float (&f)[8]) {
    using T2 = typename Elem<T>::T2;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        T2 h = *reinterpret_cast<const T2*>(&v.w[i]);
        float2 p = Elem<T>::to_f2(h);
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
    }
}
template <typename T>
__device__ __forceinline__ Vec8 pack8(const float (&f)[8]) {
    using T2 = typename Elem<T>::T2;
    Vec8 v;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        T2 h = Elem<T>::from_f2(f[2 * i], f[2 * i + 1]);
        v.w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return v;
}

// tanh-approximation GELU, shaders/gelu.comp:15-21.  tanh uses the SFU
// approximation (max relative error about 2^-11, below the 2-byte output's
// resolution).
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_f(float x) {
    const float kAlpha = 0.7978845608028654f;
    const float kBeta = 0.044715f;
    float u = kAlpha * (x + kBeta * x * x * x);
    return 0.5f * x * (1.0f + tanh_fast(u));
}

// Epilogue options of the decode GEMV: acc adds the existing y, gelu applies
// GELU to the result (after acc).
struct GemvEpilogue {
    int acc = 0;
    int gelu = 0;
};

// Fused argmax of a decode GEMV (greedy sampling of an LM head without a
// logits round trip).  keys_out[m]: the row's 64-bit greedy key over global
// indices key_off + n (tensor-parallel shards combine keys); ids_out[m]: the
// token id (key_off must be 0).  y_out, when not null, also receives the
// logits.  Scratch pointers are filled in by the launcher.
struct GemvArgmax {
    unsigned long long* slab_keys = nullptr;
    unsigned int* ticket = nullptr;
    unsigned long long* keys_out = nullptr;
    uint32_t* ids_out = nullptr;
    uint32_t key_off = 0;
    int write_y = 1;
};
int gemv_argmax(const void* X, const void* W, uint32_t Mt, uint32_t K, uint32_t N, bool w_kmajor, uint32_t key_off,
                unsigned long long* keys_out, uint32_t* ids_out, void* y_out, int dtype, cudaStream_t st);

// Row-parallel decode GEMV fused with the tensor-parallel all-reduce and the
// residual add: y[m, :] += sum over ranks of (x_r[m, :] . W_r).  Each slab's
// final fp32 partial is pushed into every rank's buf (plain stores over
// NVLink peer mappings) as (value, flag) pairs, the flag being
// *epoch * 256 + callsite + 1; each rank polls its own buf (bounded) until
// every rank's pairs carry the flag, sums them in rank order (identical on
// every rank) and adds the sum to y.  buf[q]: rank q's [2][tp][16][N] pairs
// (double-buffered by call-site parity); callsite < 255.
// With half = 1 the partials travel rounded to the storage type, two values
// per (pair, flag) word (half the bytes; the same numerics as an all-reduce
// of 16-bit partials).
struct GemvAllReduce {
    uint2* buf[8] = {};
    const uint32_t* epoch = nullptr;
    uint32_t tp = 0, rank = 0, callsite = 0, half = 0;
};
int gemv_allreduce_residual(const void* X, const void* W, void* Y, uint32_t Mt, uint32_t K, uint32_t N,
                            const GemvAllReduce& ar, int dtype, cudaStream_t st);

// Epilogue of the fused QKV projection of the LLM driver: the output row r
// (sequence r / S, position pos + r % S with pos = *d_pos when given, else
// pos0) has columns [q heads | k heads | v heads] of Dh each; q and k are
// rotated per head (adjacent pairs (2p, 2p + 1), angle position *
// base^(-2p / Dh), as evk::ai::rope with head_dim = Dh), q goes to
// q[r, Hq * Dh], k and v to row b * max_len + position of the caches
// [B, max_len, Hk * Dh].  The product itself is not stored.  With `cs`, the
// (cos, sin) of each angle come from a table [cs_len][Dh / 2] filled by
// rope_table() (the same fp32 expressions, so the same values) instead of
// a sincosf per pair.
struct QkvRope {
    void* q = nullptr;
    void* kc = nullptr;
    void* vc = nullptr;
    uint32_t Hq = 0, Hk = 0, Dh = 0, S = 1, max_len = 0, pos0 = 0;
    const uint32_t* d_pos = nullptr;
    float base = 10000.0f;
    const float2* cs = nullptr;
    uint32_t cs_len = 0;
};

// Fills cs[pos][p] = (cos, sin)(pos * base^(-2p / Dh)) for pos < len,
// p < Dh / 2, in the fused QKV epilogue's own arithmetic.
int rope_table(float2* cs, uint32_t len, uint32_t Dh, float base, cudaStream_t st);

// evkcu_matmul with an optional GELU applied to each output element (after
// the optional C +=), or the QKV epilogue above, for the library's own
// drivers.
int matmul_ex(const void* A, const void* B, void* C, uint32_t batch, uint32_t M, uint32_t K, uint32_t N,
              uint64_t stride_a, uint64_t stride_b, uint64_t stride_c, uint32_t flags, int dtype, int gelu,
              void* stream, const QkvRope* qkv = nullptr);

// evkcu_flash_attention with K and V read at a batch stride of kv_bstride
// elements (0: N * Hkv * Dh, contiguous), e.g. the first N rows of each
// sequence's KV cache.  For the library's own drivers.
int flash_attention_kv_strided(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N,
                               uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype,
                               uint64_t kv_bstride, cudaStream_t st);

// --------------------------------------------------------- device limits ----
// Upper bound, in clock cycles, of any device-side spin wait (~2 s at 2 GHz).
// A wait that exceeds it records EVKCU_TIMEOUT in the device error word and
// gives up instead of hanging the GPU.
constexpr long long kSpinLimitCycles = 4000000000LL;

}  // namespace evkcu
