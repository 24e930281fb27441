// evk_core.cpp — CUDA implementation of the evk core subset in evk.h.
//
// Replaces the Vulkan core (evk_vulkan.cpp: buffers via VMA :300-357, command
// buffer ring :1734-1798, submit :2627-2670, fences :1824-1841, timestamps
// :2427-2452) for the evk::ai path:
//   Buffer      cudaMalloc (GPU) or cudaMallocHost (host-visible types)
//   Cmd         one CUDA stream per thread; commands run in stream order,
//               so barrier() has nothing to do
//   submit()    records a CUDA event and returns its index
//   CmdWait()   synchronises that event and publishes timestamps
//   timestamp   cudaEvent pairs, reported in milliseconds
// Errors are fatal (message + abort), as EVK_ASSERT is in the reference
// (evk_vulkan.h:8-15).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <deque>
#include <map>
#include <mutex>
#include <type_traits>

#include "evk.h"
#include "evk_cuda.h"

namespace evk {
namespace {

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        std::fprintf(stderr, "evk(cuda): %s failed: %s\n", what, cudaGetErrorString(e));
        std::abort();
    }
}

struct BufferRes : Resource {
    BufferDesc desc;
    void* ptr = nullptr;
    bool host = false;
    ~BufferRes() override {
        if (!ptr) return;
        if (host)
            cudaFreeHost(ptr);
        else
            cudaFree(ptr);
    }
};

struct PendingStamp {
    cudaEvent_t a, b;
    const char* name;
};

struct CmdState {
    cudaStream_t stream = nullptr;
    Cmd cmd;
    std::vector<PendingStamp> open;  // recorded since the last submit
    uint64_t next_index = 1;
    std::map<uint64_t, cudaEvent_t> submitted;
    std::map<uint64_t, std::vector<PendingStamp>> stamps;
    std::vector<TimestampEntry> done;
    cudaEvent_t epoch = nullptr;
};

thread_local CmdState* g_cmd = nullptr;
Features g_features;
std::mutex g_mu;

CmdState& cmd_state() {
    if (!g_cmd) {
        g_cmd = new CmdState();
        check(cudaStreamCreateWithFlags(&g_cmd->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaEventCreate(&g_cmd->epoch), "cudaEventCreate");
        check(cudaEventRecord(g_cmd->epoch, g_cmd->stream), "cudaEventRecord");
        g_cmd->cmd._internal = g_cmd;
    }
    return *g_cmd;
}

CmdState& state_of(Cmd& c) { return *static_cast<CmdState*>(c._internal ? c._internal : &cmd_state()); }

BufferRes* res_of(const Buffer& b) { return static_cast<BufferRes*>(b.res); }

}  // namespace

void Resource::decRef() {
    if (refCount > 0 && --refCount == 0) delete this;
}

RID ResourceRef::GetRID() const { return res ? res->resourceid : -1; }

Buffer CreateBuffer(const BufferDesc& desc) {
    auto* r = new BufferRes();
    r->desc = desc;
    r->host = desc.memoryType != MemoryType::GPU;
    const size_t sz = desc.size ? desc.size : 16;
    if (r->host)
        check(cudaMallocHost(&r->ptr, sz), "cudaMallocHost");
    else
        check(cudaMalloc(&r->ptr, sz), "cudaMalloc");
    return Buffer(r);
}

void* Buffer::GetPtr() {
    BufferRes* r = res_of(*this);
    return (r && r->host) ? r->ptr : nullptr;
}

uint64_t Buffer::GetReference() {
    BufferRes* r = res_of(*this);
    return r ? reinterpret_cast<uint64_t>(r->ptr) : 0;
}

const BufferDesc& GetDesc(const Buffer& b) { return res_of(b)->desc; }

void WriteBuffer(Buffer& buffer, void* src, uint64_t size, uint64_t offset) {
    check(cudaMemcpy((char*)res_of(buffer)->ptr + offset, src, size, cudaMemcpyDefault), "WriteBuffer");
}

void ReadBuffer(Buffer& buffer, void* dst, uint64_t size, uint64_t offset) {
    check(cudaMemcpy(dst, (char*)res_of(buffer)->ptr + offset, size, cudaMemcpyDefault), "ReadBuffer");
}

bool InitializeEVK(const EvkDesc& info) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return false;
    g_features.coopmat = p.major >= 10;
    g_features.timestamps = true;  // CUDA events are always available
    g_features.raytracing = false;
    (void)info;
    cmd_state();
    return true;
}

void Shutdown() {
    if (g_cmd) {
        cudaStreamSynchronize(g_cmd->stream);
        for (auto& kv : g_cmd->submitted) cudaEventDestroy(kv.second);
        cudaStreamDestroy(g_cmd->stream);
        delete g_cmd;
        g_cmd = nullptr;
    }
}

const Features& GetFeatures() { return g_features; }

const std::vector<TimestampEntry>& CmdTimestamps() { return cmd_state().done; }

void Cmd::barrier() {}

void Cmd::fill(Buffer dst, uint32_t data, uint64_t size, uint64_t offset) {
    CmdState& s = state_of(*this);
    char* p = (char*)res_of(dst)->ptr + offset;
    const uint8_t b0 = data & 0xFF;
    if (data == 0u || data == b0 * 0x01010101u) {
        check(cudaMemsetAsync(p, b0, size, s.stream), "Cmd::fill");
        return;
    }
    std::vector<uint32_t> pattern((size + 3) / 4, data);
    check(cudaMemcpyAsync(p, pattern.data(), size, cudaMemcpyHostToDevice, s.stream), "Cmd::fill");
    check(cudaStreamSynchronize(s.stream), "Cmd::fill");
}

void Cmd::update(Buffer& dst, uint64_t dstOffset, uint64_t size, void* src) { copy(src, dst, size, dstOffset); }

void Cmd::copy(Buffer& src, Buffer& dst, uint64_t size, uint64_t srcOffset, uint64_t dstOffset) {
    CmdState& s = state_of(*this);
    check(cudaMemcpyAsync((char*)res_of(dst)->ptr + dstOffset, (char*)res_of(src)->ptr + srcOffset, size,
                          cudaMemcpyDefault, s.stream),
          "Cmd::copy");
}

void Cmd::copy(void* src, Buffer& dst, uint64_t size, uint64_t dstOffset) {
    // The reference stages `src` at record time (evk_vulkan.cpp:2006-2027);
    // a copy from pageable memory returns once the source has been staged.
    CmdState& s = state_of(*this);
    check(cudaMemcpyAsync((char*)res_of(dst)->ptr + dstOffset, src, size, cudaMemcpyDefault, s.stream), "Cmd::copy");
}

int Cmd::beginTimestamp(const char* name) {
    CmdState& s = state_of(*this);
    PendingStamp p{};
    check(cudaEventCreate(&p.a), "cudaEventCreate");
    check(cudaEventCreate(&p.b), "cudaEventCreate");
    p.name = name;
    check(cudaEventRecord(p.a, s.stream), "cudaEventRecord");
    s.open.push_back(p);
    return (int)s.open.size() - 1;
}

void Cmd::endTimestamp(int id) {
    CmdState& s = state_of(*this);
    check(cudaEventRecord(s.open.at(id).b, s.stream), "cudaEventRecord");
}

uint64_t Cmd::submit() {
    CmdState& s = state_of(*this);
    cudaEvent_t ev;
    check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
    check(cudaEventRecord(ev, s.stream), "cudaEventRecord");
    const uint64_t idx = s.next_index++;
    s.submitted[idx] = ev;
    if (!s.open.empty()) {
        s.stamps[idx] = std::move(s.open);
        s.open.clear();
    }
    return idx;
}

static void retire(CmdState& s, uint64_t idx) {
    // Publish the timestamps of every submission up to idx.
    bool any = false;
    for (auto it = s.stamps.begin(); it != s.stamps.end() && it->first <= idx;) {
        if (!any) {
            s.done.clear();
            any = true;
        }
        for (auto& p : it->second) {
            float a = 0, b = 0;
            cudaEventElapsedTime(&a, s.epoch, p.a);
            cudaEventElapsedTime(&b, s.epoch, p.b);
            s.done.push_back(TimestampEntry{a, b, p.name});
            cudaEventDestroy(p.a);
            cudaEventDestroy(p.b);
        }
        it = s.stamps.erase(it);
    }
    for (auto it = s.submitted.begin(); it != s.submitted.end() && it->first <= idx;) {
        cudaEventDestroy(it->second);
        it = s.submitted.erase(it);
    }
}

Cmd& CmdBegin(Queue) { return cmd_state().cmd; }

bool CmdDone(uint64_t idx) {
    CmdState& s = cmd_state();
    auto it = s.submitted.find(idx);
    if (it == s.submitted.end()) return true;
    if (cudaEventQuery(it->second) != cudaSuccess) return false;
    retire(s, idx);
    return true;
}

void CmdWait(uint64_t idx) {
    CmdState& s = cmd_state();
    auto it = s.submitted.find(idx);
    if (it != s.submitted.end()) check(cudaEventSynchronize(it->second), "CmdWait");
    retire(s, idx);
}

void* cuda_stream(Cmd& cmd) { return state_of(cmd).stream; }

}  // namespace evk
