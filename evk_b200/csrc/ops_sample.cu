// ops_sample.cu — greedy_sample (argmax over a token window).
//
// Reference: shaders/greedy_sample.comp:24-64.  There, 256 lanes scan
// j = lane, lane+256, ... keeping the first strict maximum (initial value
// -FLT_MAX, initial token = token_base), then a shared-memory tree at strides
// 128..1 where lane l takes lane l+s only if strictly greater.  Unrolling that
// tree: among lanes holding the global maximum, the winner is the lane whose
// index has the smallest bit-reversed value (ties prefer an even lane, then a
// lane = 0 mod 4, ...), and within a lane the smallest j.
//
// This kernel computes the same winner in one pass over the window split
// across CTAs: every element j (window offset) gets the 64-bit key
//     hi32 = order-preserving bits of its value (0 for NaN / -inf, which the
//            reference never selects because `v > -FLT_MAX` is false)
//     lo32 = ~(bitrev8(j & 255) << 24 | (j >> 8))
// and the maximum key over the window identifies the reference's token.
// Partial maxima go to a scratch array; the last CTA of each row (atomic
// ticket) reduces them and writes the id, so one launch does the whole op.
#include <float.h>

#include <mutex>

#include "common.cuh"
#include "greedy_key.cuh"

namespace evkcu {
namespace {

constexpr int kThreads = 256;
constexpr uint32_t kChunk = 4096;  // window elements per CTA

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t t = __shfl_xor_sync(0xffffffffu, k, o);
        k = t > k ? t : k;
    }
    return k;
}

__device__ uint64_t block_max_u64(uint64_t k, uint64_t* sh) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    k = warp_max_u64(k);
    if (lane == 0) sh[wid] = k;
    __syncthreads();
    k = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0ull;
    return warp_max_u64(k);
}

// grid = (chunks, B).  partial: [B][chunks] keys; tickets: [B] counters that
// start at 0 and are reset to 0 by the last CTA of each row.
template <typename T>
__global__ void __launch_bounds__(kThreads) greedy_kernel(const T* __restrict__ logits, void* __restrict__ out,
                                                          uint32_t S, uint32_t V, uint32_t position,
                                                          uint32_t token_base, uint32_t token_count,
                                                          uint32_t out_bytes, uint64_t* __restrict__ partial,
                                                          unsigned int* __restrict__ tickets) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    __shared__ uint64_t sh[32];
    __shared__ bool is_last;
    const uint32_t b = blockIdx.y;
    const uint32_t chunks = gridDim.x;
    const T* row = logits + ((uint64_t)b * S + position) * V + token_base;
    const uint32_t lo = blockIdx.x * kChunk;
    const uint32_t hi = min(lo + kChunk, token_count);
    uint64_t best = 0ull;
    // Vector body over the 16-byte-aligned part of [lo, hi).
    uint32_t mis = (uint32_t)(((uintptr_t)(row + lo) & 15u) / sizeof(T));
    uint32_t vstart = lo + (mis ? (8 - mis) : 0);
    if (vstart > hi) vstart = hi;
    uint32_t nvec = (hi - vstart) / 8;
    for (uint32_t j = lo + threadIdx.x; j < vstart; j += blockDim.x) {
        uint64_t k = elem_key(Elem<T>::to_f(row[j]), j);
        best = k > best ? k : best;
    }
    const Vec8* vrow = reinterpret_cast<const Vec8*>(row + vstart);
    for (uint32_t c = threadIdx.x; c < nvec; c += blockDim.x) {
        float f[8];
        unpack8<T>(vrow[c], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            uint64_t k = elem_key(f[e], vstart + c * 8 + e);
            best = k > best ? k : best;
        }
    }
    for (uint32_t j = vstart + nvec * 8 + threadIdx.x; j < hi; j += blockDim.x) {
        uint64_t k = elem_key(Elem<T>::to_f(row[j]), j);
        best = k > best ? k : best;
    }
    best = block_max_u64(best, sh);

    if (chunks > 1) {
        if (threadIdx.x == 0) {
            partial[(uint64_t)b * chunks + blockIdx.x] = best;
            __threadfence();
            unsigned int t = atomicAdd(&tickets[b], 1u);
            is_last = (t == chunks - 1);
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        uint64_t k = 0ull;
        for (uint32_t c = threadIdx.x; c < chunks; c += blockDim.x) {
            uint64_t p = *((volatile uint64_t*)&partial[(uint64_t)b * chunks + c]);
            k = p > k ? p : k;
        }
        __syncthreads();
        best = block_max_u64(k, sh);
    }
    if (threadIdx.x == 0) {
        uint32_t tok = best ? token_base + key_to_offset(best) : token_base;
        if (out_bytes == 2)
            reinterpret_cast<uint16_t*>(out)[b] = (uint16_t)tok;
        else
            reinterpret_cast<uint32_t*>(out)[b] = tok;
        if (chunks > 1) tickets[b] = 0u;
    }
}

}  // namespace

}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_greedy_sample(const void* logits, void* out, uint32_t B, uint32_t S, uint32_t V,
                                   uint32_t position, uint32_t token_base, uint32_t token_count,
                                   uint32_t out_bytes, int dtype, void* stream) {
    if (B == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(logits && out, EVKCU_BAD_ARG, "evkcu_greedy_sample: null pointer");
    EVKCU_CHECK_ARG(out_bytes == 2 || out_bytes == 4, EVKCU_BAD_ARG, "evkcu_greedy_sample: out_bytes must be 2 or 4");
    EVKCU_CHECK_ARG(position < S, EVKCU_BAD_SHAPE, "evkcu_greedy_sample: position >= seq_len");
    EVKCU_CHECK_ARG((uint64_t)token_base + token_count <= V, EVKCU_BAD_SHAPE,
                    "evkcu_greedy_sample: token window exceeds vocabulary");
    DeviceState* st = state();
    EVKCU_CHECK_ARG(st, EVKCU_CUDA_ERROR, "evkcu_greedy_sample: no device state");
    uint32_t chunks = token_count == 0 ? 1 : (token_count + kChunk - 1) / kChunk;
    // Scratch for the split reduction: [B] tickets (zero) then [B][chunks] keys.
    unsigned int* tickets = nullptr;
    uint64_t* partial = nullptr;
    if (chunks > 1) {
        EVKCU_CHECK_ARG(B <= kMaxTickets, EVKCU_BAD_SHAPE, "evkcu_greedy_sample: batch too large");
        const size_t toff = kTicketBytes;
        char* ws = (char*)workspace(WS_GREEDY, toff + (size_t)B * chunks * 8);
        EVKCU_CHECK_ARG(ws, EVKCU_CUDA_ERROR, "evkcu_greedy_sample: scratch allocation failed");
        tickets = (unsigned int*)ws;
        partial = (uint64_t*)(ws + toff);
    }
    dim3 grid(chunks, B);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_greedy_sample", greedy_kernel<T>, grid, kThreads, 0, as_stream(stream),
                          (const T*)logits, out, S, V, position, token_base, token_count, out_bytes, partial, tickets);
    });
}

// ---------------------------------------------------------------------------
// evkcu_greedy_sample_noalloc — the same kernel with its split-reduction
// scratch in a fixed, file-scope device array instead of library-allocated
// memory, for callers that must not allocate (see evkcu.h).
namespace evkcu {
namespace {

// [kNoAllocTickets] ticket counters, then the per-chunk partial keys.
constexpr size_t kNoAllocScratchBytes = 128 * 1024;
constexpr uint32_t kNoAllocTickets = 1024;
constexpr size_t kNoAllocKeyOffset = kNoAllocTickets * sizeof(unsigned int);
constexpr size_t kNoAllocMaxKeys = (kNoAllocScratchBytes - kNoAllocKeyOffset) / sizeof(uint64_t);

static __device__ __align__(256) unsigned char g_greedy_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array, looked up once per device with that device
// current.  Host code cannot use the symbol itself: on the host it names a
// stand-in object, not the device memory.
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

int noalloc_scratch(void** out) {
    int dev = 0;
    EVKCU_CUDA_TRY(cudaGetDevice(&dev));
    EVKCU_CHECK_ARG(dev >= 0 && dev < 64, EVKCU_UNSUPPORTED, "evkcu_greedy_sample_noalloc: device index >= 64");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        EVKCU_CUDA_TRY(cudaGetSymbolAddress(&p, g_greedy_noalloc_scratch));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return EVKCU_OK;
}

}  // namespace
}  // namespace evkcu

extern "C" int evkcu_greedy_sample_noalloc(const void* logits, void* out, uint32_t B, uint32_t S, uint32_t V,
                                           uint32_t position, uint32_t token_base, uint32_t token_count,
                                           uint32_t out_bytes, int dtype, void* stream) {
    if (B == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(logits && out, EVKCU_BAD_ARG, "evkcu_greedy_sample_noalloc: null pointer");
    EVKCU_CHECK_ARG(out_bytes == 2 || out_bytes == 4, EVKCU_BAD_ARG,
                    "evkcu_greedy_sample_noalloc: out_bytes must be 2 or 4");
    EVKCU_CHECK_ARG(position < S, EVKCU_BAD_SHAPE, "evkcu_greedy_sample_noalloc: position >= seq_len");
    EVKCU_CHECK_ARG((uint64_t)token_base + token_count <= V, EVKCU_BAD_SHAPE,
                    "evkcu_greedy_sample_noalloc: token window exceeds vocabulary");
    const uint32_t chunks = token_count == 0 ? 1 : (token_count + kChunk - 1) / kChunk;
    EVKCU_CHECK_ARG(B <= kNoAllocTickets && (uint64_t)B * chunks <= kNoAllocMaxKeys, EVKCU_BAD_SHAPE,
                    "evkcu_greedy_sample_noalloc: request exceeds the fixed scratch (needs B <= 1024 and "
                    "B * ceil(token_count / 4096) <= 15872); use evkcu_greedy_sample");
    unsigned int* tickets = nullptr;
    uint64_t* partial = nullptr;
    if (chunks > 1) {
        void* base = nullptr;
        const int r = noalloc_scratch(&base);
        if (r != EVKCU_OK) return r;
        tickets = static_cast<unsigned int*>(base);
        partial = reinterpret_cast<uint64_t*>(static_cast<char*>(base) + kNoAllocKeyOffset);
        // The array keeps the previous call's contents: the tickets must start at zero.
        EVKCU_CUDA_TRY(cudaMemsetAsync(tickets, 0, (size_t)B * sizeof(unsigned int), as_stream(stream)));
    }
    dim3 grid(chunks, B);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_greedy_sample_noalloc", greedy_kernel<T>, grid, kThreads, 0, as_stream(stream),
                          (const T*)logits, out, S, V, position, token_base, token_count, out_bytes, partial, tickets);
    });
}
