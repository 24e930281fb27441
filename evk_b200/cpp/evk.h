// evk.h — the subset of evk's core interface (carloshgsilva/evk evk.h) that
// the evk::ai operator path uses, implemented on CUDA by evk_core.cpp.
//
// Declarations keep the reference's names, signatures and ownership model
// (ref-counted resources; Buffer::GetReference returns a 64-bit device
// address, evk.h:243-257, evk_vulkan.cpp:335) so evk::ai callers compile
// unchanged.  Vulkan-only parts (images, pipelines, graphics, ray tracing,
// swapchain) are not part of this backend.  A Cmd is a CUDA stream: commands
// are enqueued immediately in stream order, submit() records an event and
// CmdWait() synchronises on it.
#pragma once

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace evk {

using RID = int;

enum class BufferUsage {
    TransferSrc = 1,
    TransferDst = 2,
    Vertex = 4,
    Index = 8,
    Indirect = 16,
    Storage = 32,
    AccelerationStructure = 64,
    AccelerationStructureInput = 128,
};
inline BufferUsage operator|(BufferUsage a, BufferUsage b) { return (BufferUsage)((uint32_t)a | (uint32_t)b); }

enum class MemoryType {
    CPU,         // pinned host memory (device-addressable)
    GPU,         // device memory
    CPU_TO_GPU,  // pinned host memory
    GPU_TO_CPU,  // pinned host memory
};

struct TimestampEntry {
    double start, end;  // milliseconds
    const char* name;
};

// Intrusively ref-counted resource; the last ResourceRef releases it.
struct Resource {
    RID resourceid = -1;
    uint32_t refCount = 0;
    void incRef() { refCount++; }
    void decRef();
    virtual ~Resource() {}
};

struct ResourceRef {
    Resource* res = nullptr;
    ResourceRef() {}
    ResourceRef(Resource* r) {
        if (r) {
            res = r;
            r->incRef();
        }
    }
    ResourceRef(const ResourceRef& o) { *this = o; }
    ResourceRef(ResourceRef&& o) { *this = std::move(o); }
    ResourceRef& operator=(const ResourceRef& o) {
        if (o.res) o.res->incRef();
        if (res) res->decRef();
        res = o.res;
        return *this;
    }
    ResourceRef& operator=(ResourceRef&& o) {
        if (this != &o) {
            if (res) res->decRef();
            res = o.res;
            o.res = nullptr;
        }
        return *this;
    }
    ~ResourceRef() {
        if (res) res->decRef();
    }
    explicit operator bool() const { return res != nullptr; }
    void release() {
        if (res) {
            res->decRef();
            res = nullptr;
        }
    }
    void swap(ResourceRef& o) {
        Resource* t = o.res;
        o.res = res;
        res = t;
    }
    RID GetRID() const;
};

struct BufferDesc {
    std::string name = "";
    uint64_t size = 0;
    BufferUsage usage = BufferUsage::Storage;
    MemoryType memoryType = MemoryType::GPU;
};

struct Buffer : ResourceRef {
    Buffer(Resource* r = nullptr) : ResourceRef(r) {}
    void* GetPtr();           // host pointer (host-memory buffers), else nullptr
    uint64_t GetReference();  // device address
};
Buffer CreateBuffer(const BufferDesc& desc);
void WriteBuffer(Buffer& buffer, void* src, uint64_t size, uint64_t offset = 0u);
void ReadBuffer(Buffer& buffer, void* dst, uint64_t size, uint64_t offset = 0u);
const BufferDesc& GetDesc(const Buffer& res);

struct EvkDesc {
    std::string applicationName = "";
    std::uint32_t applicationVersion = 0;
    std::string engineName = "";
    std::uint32_t engineVersion = 0;
    std::vector<std::string> instanceLayers = {};
    std::vector<std::string> instanceExtensions = {};
    uint32_t frameBufferingCount = 3;
    bool enableSwapchain = false;
    bool enableValidation = false;
    bool enableTimestamps = false;
};

struct Features {
    bool raytracing = false;
    bool coopmat = false;  // true: the tensor-core ops are available
    bool timestamps = false;
};

bool InitializeEVK(const EvkDesc& info);
void Shutdown();
const Features& GetFeatures();

// Timestamps of the last completed submission (filled by CmdWait/CmdDone).
const std::vector<TimestampEntry>& CmdTimestamps();

enum class Queue { Graphics };

struct Cmd {
    void* _internal = nullptr;

    void barrier();  // stream order already serialises; kept for callers
    void fill(Buffer dst, uint32_t data, uint64_t size, uint64_t offset = 0);
    void update(Buffer& dst, uint64_t dstOffset, uint64_t size, void* src);
    void copy(Buffer& src, Buffer& dst, uint64_t size, uint64_t srcOffset = 0, uint64_t dstOffset = 0);
    void copy(void* src, Buffer& dst, uint64_t size, uint64_t dstOffset = 0);

    int beginTimestamp(const char* name);
    void endTimestamp(int id);

    uint64_t submit();

    template <typename T>
    void timestamp(const char* name, T callback) {
        int id = beginTimestamp(name);
        callback();
        endTimestamp(id);
    }
};

Cmd& CmdBegin(Queue queue = Queue::Graphics);
bool CmdDone(uint64_t submissionIndex);
void CmdWait(uint64_t submissionIndex);

}  // namespace evk
