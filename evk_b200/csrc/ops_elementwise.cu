// ops_elementwise.cu — HBM-bound elementwise ops: add, gelu, scale, zero,
// causal mask, embedding gather.  Each kernel moves 16-byte vectors (8
// elements) per thread where the buffers allow it and falls back to scalar
// loads for the ragged tail.  Grids are grid-stride loops sized to a multiple
// of the SM count.
#include "common.cuh"

namespace evkcu {
namespace {

constexpr int kThreads = 256;

inline unsigned grid_for(uint64_t work_items) {
    DeviceState* s = state();
    int sms = s ? s->sm_count : 148;
    uint64_t want = (work_items + kThreads - 1) / kThreads;
    uint64_t cap = (uint64_t)sms * 8;  // 8 resident 256-thread CTAs per SM
    if (want < 1) want = 1;
    return (unsigned)(want < cap ? want : cap);
}

enum class Unary { Gelu, Scale };

template <typename T, Unary OP>
__global__ void unary_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t n, float s) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    uint64_t nvec = n / 8;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const Vec8* vin = reinterpret_cast<const Vec8*>(in);
    Vec8* vout = reinterpret_cast<Vec8*>(out);
    for (uint64_t v = i; v < nvec; v += stride) {
        float f[8];
        unpack8<T>(vin[v], f);
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = (OP == Unary::Gelu) ? gelu_f(f[k]) : f[k] * s;
        vout[v] = pack8<T>(f);
    }
    for (uint64_t e = nvec * 8 + i; e < n; e += stride) {
        float x = Elem<T>::to_f(in[e]);
        out[e] = Elem<T>::from_f((OP == Unary::Gelu) ? gelu_f(x) : x * s);
    }
}

template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c, uint64_t n) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    uint64_t nvec = n / 8;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const Vec8* va = reinterpret_cast<const Vec8*>(a);
    const Vec8* vb = reinterpret_cast<const Vec8*>(b);
    Vec8* vc = reinterpret_cast<Vec8*>(c);
    for (uint64_t v = i; v < nvec; v += stride) {
        float fa[8], fb[8];
        unpack8<T>(va[v], fa);
        unpack8<T>(vb[v], fb);
#pragma unroll
        for (int k = 0; k < 8; ++k) fa[k] += fb[k];
        vc[v] = pack8<T>(fa);
    }
    for (uint64_t e = nvec * 8 + i; e < n; e += stride)
        c[e] = Elem<T>::from_f(Elem<T>::to_f(a[e]) + Elem<T>::to_f(b[e]));
}

// Scalar fallback for buffers that are not 16-byte aligned.
template <typename T>
__global__ void add_scalar_kernel(const T* a, const T* b, T* c, uint64_t n) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride)
        c[e] = Elem<T>::from_f(Elem<T>::to_f(a[e]) + Elem<T>::to_f(b[e]));
}
template <typename T, Unary OP>
__global__ void unary_scalar_kernel(const T* in, T* out, uint64_t n, float s) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += stride) {
        float x = Elem<T>::to_f(in[e]);
        out[e] = Elem<T>::from_f((OP == Unary::Gelu) ? gelu_f(x) : x * s);
    }
}

// shaders/causal_mask.comp:16-33 — row-per-block so each thread only tests j > i.
template <typename T>
__global__ void causal_mask_kernel(T* __restrict__ scores, uint64_t rows, uint32_t N) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    const T sentinel = Elem<T>::from_f(-65504.0f);
    for (uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        uint32_t i = (uint32_t)(r % N);
        T* row = scores + r * N;
        for (uint32_t j = i + 1 + threadIdx.x; j < N; j += blockDim.x) row[j] = sentinel;
    }
}

// shaders/embed.comp:18-28 — one block row per gathered index, 16-byte vectors.
template <typename T, typename I>
__global__ void embed_kernel(const T* __restrict__ E, const I* __restrict__ idx, T* __restrict__ out,
                             uint32_t vocab, uint32_t dim, uint32_t n_idx, bool vec) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    for (uint32_t r = blockIdx.x; r < n_idx; r += gridDim.x) {
        uint32_t tok = (uint32_t)idx[r];
        if (tok >= vocab) tok = vocab - 1;
        const T* src = E + (uint64_t)tok * dim;
        T* dst = out + (uint64_t)r * dim;
        if (vec) {
            const Vec8* vs = reinterpret_cast<const Vec8*>(src);
            Vec8* vd = reinterpret_cast<Vec8*>(dst);
            for (uint32_t c = threadIdx.x; c < dim / 8; c += blockDim.x) vd[c] = vs[c];
        } else {
            for (uint32_t c = threadIdx.x; c < dim; c += blockDim.x) dst[c] = src[c];
        }
    }
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_add(const void* a, const void* b, void* c, uint64_t n, int dtype, void* stream) {
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(a && b && c, EVKCU_BAD_ARG, "evkcu_add: null pointer");
    bool vec = aligned16(a) && aligned16(b) && aligned16(c);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (vec)
            return launch_pdl("evkcu_add", add_kernel<T>, grid_for(n / 8 + 1), kThreads, 0, as_stream(stream),
                              (const T*)a, (const T*)b, (T*)c, n);
        return launch_pdl("evkcu_add", add_scalar_kernel<T>, grid_for(n), kThreads, 0, as_stream(stream), (const T*)a,
                          (const T*)b, (T*)c, n);
    });
}

template <Unary OP>
static int launch_unary(const void* in, void* out, uint64_t n, float s, int dtype, void* stream, const char* name) {
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(in && out, EVKCU_BAD_ARG, std::string(name) + ": null pointer");
    bool vec = aligned16(in) && aligned16(out);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (vec)
            return launch_pdl(name, unary_kernel<T, OP>, grid_for(n / 8 + 1), kThreads, 0, as_stream(stream),
                              (const T*)in, (T*)out, n, s);
        return launch_pdl(name, unary_scalar_kernel<T, OP>, grid_for(n), kThreads, 0, as_stream(stream), (const T*)in,
                          (T*)out, n, s);
    });
}

extern "C" int evkcu_gelu(const void* in, void* out, uint64_t n, int dtype, void* stream) {
    return launch_unary<Unary::Gelu>(in, out, n, 1.0f, dtype, stream, "evkcu_gelu");
}

extern "C" int evkcu_scale(void* x, uint64_t n, float s, int dtype, void* stream) {
    return launch_unary<Unary::Scale>(x, x, n, s, dtype, stream, "evkcu_scale");
}

extern "C" int evkcu_zero(void* x, uint64_t n, int dtype, void* stream) {
    if (n == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(x, EVKCU_BAD_ARG, "evkcu_zero: null pointer");
    EVKCU_CHECK_ARG(dtype == EVKCU_F16 || dtype == EVKCU_BF16, EVKCU_BAD_ARG, "evkcu_zero: unknown dtype");
    // +0.0 is the all-zero bit pattern in both 2-byte formats.
    EVKCU_CUDA_TRY(cudaMemsetAsync(x, 0, n * 2, as_stream(stream)));
    return EVKCU_OK;
}

extern "C" int evkcu_causal_mask(void* scores, uint32_t batch, uint32_t N, int dtype, void* stream) {
    if (batch == 0 || N == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(scores, EVKCU_BAD_ARG, "evkcu_causal_mask: null pointer");
    uint64_t rows = (uint64_t)batch * N;
    DeviceState* s = state();
    unsigned grid = (unsigned)(rows < (uint64_t)s->sm_count * 16 ? rows : (uint64_t)s->sm_count * 16);
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        return launch_pdl("evkcu_causal_mask", causal_mask_kernel<T>, grid, 256, 0, as_stream(stream), (T*)scores, rows,
                          N);
    });
}

extern "C" int evkcu_embed(const void* E, const void* idx, void* out, uint32_t vocab, uint32_t dim,
                           uint32_t n_idx, uint32_t idx_bytes, int dtype, void* stream) {
    if (n_idx == 0 || dim == 0) return EVKCU_OK;
    EVKCU_CHECK_ARG(E && idx && out, EVKCU_BAD_ARG, "evkcu_embed: null pointer");
    EVKCU_CHECK_ARG(vocab > 0, EVKCU_BAD_SHAPE, "evkcu_embed: empty vocabulary");
    EVKCU_CHECK_ARG(idx_bytes == 2 || idx_bytes == 4, EVKCU_BAD_ARG, "evkcu_embed: idx_bytes must be 2 or 4");
    bool vec = (dim % 8 == 0) && aligned16(E) && aligned16(out);
    DeviceState* s = state();
    unsigned grid = n_idx < (uint32_t)s->sm_count * 16 ? n_idx : (uint32_t)s->sm_count * 16;
    unsigned threads = vec ? (dim / 8 < 128 ? 64 : 128) : 256;
    return EVKCU_DISPATCH_DTYPE(dtype, T, [&] {
        if (idx_bytes == 2)
            return launch_pdl("evkcu_embed", embed_kernel<T, uint16_t>, grid, threads, 0, as_stream(stream), (const T*)E,
                              (const uint16_t*)idx, (T*)out, vocab, dim, n_idx, vec);
        return launch_pdl("evkcu_embed", embed_kernel<T, uint32_t>, grid, threads, 0, as_stream(stream), (const T*)E,
                          (const uint32_t*)idx, (T*)out, vocab, dim, n_idx, vec);
    });
}
