// context.cu — per-device state, error reporting and launch accounting.
// Replaces evk::ai::initialize/shutdown (evk_ai.cpp:211-252): there are no
// pipelines to create, only a device error word and a reusable workspace.
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace evkcu {

static thread_local std::string g_last_error;
static thread_local uint64_t g_launches = 0;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return EVKCU_CUDA_ERROR;
}

void count_launch(uint32_t n) { g_launches += n; }

static std::mutex g_mu;
static std::vector<DeviceState*> g_states;

DeviceState* state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    if ((int)g_states.size() <= dev) g_states.resize(dev + 1, nullptr);
    if (g_states[dev]) return g_states[dev];
    auto* s = new DeviceState();
    s->device = dev;
    if (cudaDeviceGetAttribute(&s->sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        delete s;
        return nullptr;
    }
    if (cudaMalloc(&s->d_error, sizeof(unsigned int)) != cudaSuccess) {
        delete s;
        return nullptr;
    }
    cudaMemset(s->d_error, 0, sizeof(unsigned int));
    if (const char* v = getenv("EVKCU_DISABLE_PDL")) s->pdl = v[0] == '\0' || v[0] == '0';
    if (const char* v = getenv("EVKCU_GEMM_PLAIN_EPILOGUE")) s->plain_epilogue = v[0] != '\0' && v[0] != '0';
    if (const char* v = getenv("EVKCU_GEMM_PAIR")) s->gemm_pair = atoi(v) ? 1 : 0;
    g_states[dev] = s;
    return s;
}

void* workspace(int slot, size_t bytes) {
    DeviceState* s = state();
    if (!s || slot < 0 || slot >= WS_COUNT) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    if (s->ws_bytes[slot] < bytes) {
        if (s->ws[slot]) {
            cudaDeviceSynchronize();
            cudaFree(s->ws[slot]);
        }
        size_t sz = bytes < (1u << 20) ? (1u << 20) : bytes;
        if (cudaMalloc(&s->ws[slot], sz) != cudaSuccess) {
            s->ws[slot] = nullptr;
            s->ws_bytes[slot] = 0;
            return nullptr;
        }
        cudaMemset(s->ws[slot], 0, sz);
        cudaDeviceSynchronize();
        s->ws_bytes[slot] = sz;
    }
    return s->ws[slot];
}

}  // namespace evkcu

using namespace evkcu;

extern "C" int evkcu_init(int device) {
    if (device >= 0) EVKCU_CUDA_TRY(cudaSetDevice(device));
    if (!state()) return fail(EVKCU_CUDA_ERROR, "evkcu_init: could not create device state");
    return EVKCU_OK;
}

extern "C" int evkcu_shutdown(void) {
    std::lock_guard<std::mutex> lock(g_mu);
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto*& s : g_states) {
        if (!s) continue;
        cudaSetDevice(s->device);
        cudaDeviceSynchronize();
        cudaFree(s->d_error);
        for (int i = 0; i < WS_COUNT; ++i)
            if (s->ws[i]) cudaFree(s->ws[i]);
        delete s;
        s = nullptr;
    }
    cudaSetDevice(cur);
    return EVKCU_OK;
}

extern "C" const char* evkcu_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* evkcu_version(void) { return "evkcu 0.1 sm_100a"; }

extern "C" int evkcu_check_device_error(void) {
    DeviceState* s = state();
    if (!s) return fail(EVKCU_CUDA_ERROR, "no device state");
    EVKCU_CUDA_TRY(cudaDeviceSynchronize());
    unsigned int h = 0;
    EVKCU_CUDA_TRY(cudaMemcpy(&h, s->d_error, sizeof(h), cudaMemcpyDeviceToHost));
    if (h != 0) {
        EVKCU_CUDA_TRY(cudaMemset(s->d_error, 0, sizeof(unsigned int)));
        return fail(EVKCU_TIMEOUT, "a bounded device-side wait gave up (code " + std::to_string(h) + ")");
    }
    return EVKCU_OK;
}

extern "C" uint64_t evkcu_launch_count(void) { return g_launches; }
extern "C" void evkcu_reset_launch_count(void) { g_launches = 0; }
