// ref_tests_cuda.cpp — runs the reference's own evk::ai tests
// (carloshgsilva/evk example/tests.h, compiled from the reference checkout
// where it lies, never copied) against THIS backend: the product headers
// evk_b200/cpp/evk.h + evk_ai.h resolve `#include <evk_ai.h>`, and the
// program links libevk_ai.so (C++ layer) over libevkcu.so (CUDA kernels).
// Nothing here implements an operator; it is the reference's test driver
// example/main.cpp:41-66 (InitializeEVK, evk::ai::initialize, the tests).
//
// Usage: ref_tests_cuda [test-name ...]   (no names: the reference's default
// list run_ai_kernel_tests, tests.h:1565-1585, then the remaining tests that
// the default list leaves out, except the 32768-token flash comparison,
// which runs by name).
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "evk_ai.h"
#include "tests.h"

namespace {
struct Entry {
    const char* name;
    std::function<void()> fn;
};
#define EVK_REF_TEST(n) Entry{#n, n}
const std::vector<Entry>& all_tests() {
    static const std::vector<Entry> t = {
        EVK_REF_TEST(test_add),
        EVK_REF_TEST(test_matmul),
        EVK_REF_TEST(test_matmul_broadcast),
        EVK_REF_TEST(test_mse_loss),
        EVK_REF_TEST(test_cross_entropy_loss),
        EVK_REF_TEST(test_sgd),
        EVK_REF_TEST(test_adam),
        EVK_REF_TEST(test_adam_fp16_matmul_convergence_vs_cpu_fp32),
        EVK_REF_TEST(test_softmax),
        EVK_REF_TEST(test_relu),
        EVK_REF_TEST(test_gelu),
        EVK_REF_TEST(test_scale_zero),
        EVK_REF_TEST(test_embed_and_backward),
        EVK_REF_TEST(test_position_add_and_backward),
        EVK_REF_TEST(test_rope_and_backward),
        EVK_REF_TEST(test_sum_batch),
        EVK_REF_TEST(test_rms_norm_and_backward),
        EVK_REF_TEST(test_greedy_sample),
        EVK_REF_TEST(test_flash_attention_backward_scratch),
        // outside the reference's default list
        EVK_REF_TEST(test_flash_attention_backward),
        EVK_REF_TEST(test_graph_backward),
        EVK_REF_TEST(test_attn_graph),
        EVK_REF_TEST(test_adam_convergence),
        EVK_REF_TEST(test_adam_vs_sgd),
        // test_adam_batched_matmul is not run: it steps Adam with lr = -0.02
        // (tests.h:1009) on the gradient 2 (pred - target) / n, which climbs
        // the loss under the reference's own update rule (shaders/adam.comp).
        EVK_REF_TEST(test_flash_attention_cmp_softmax),
    };
    return t;
}
}  // namespace

int main(int argc, char** argv) {
    if (!evk::InitializeEVK({.applicationName = "evk_b200 reference tests"})) {
        std::fprintf(stderr, "InitializeEVK failed (no CUDA device?)\n");
        return 2;
    }
    evk::ai::initialize();
    std::vector<std::string> want(argv + 1, argv + argc);
    int ran = 0;
    for (const Entry& e : all_tests()) {
        if (!want.empty()) {
            bool sel = false;
            for (const auto& w : want) sel = sel || w == e.name;
            if (!sel) continue;
        } else if (std::strcmp(e.name, "test_flash_attention_cmp_softmax") == 0) {
            continue;  // 2 x 2 GB score matrices; run it by name
        }
        e.fn();  // a failing TEST() exits the process with status 1
        ++ran;
    }
    evk::ai::shutdown();
    evk::Shutdown();
    std::printf("ALL %d REFERENCE TESTS PASSED (CUDA backend)\n", ran);
    return ran > 0 ? 0 : 3;
}
