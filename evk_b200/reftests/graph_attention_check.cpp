// graph_attention_check.cpp — drives the C++ evk::ai layer (libevk_ai.so) the
// way a reference user does: a Graph with q, k, v parameters (B, N, D),
// out = causal_attention(q, k, v), loss = mse_loss(out, target), one
// eval(backward = true) and one SGD step.  Reads the inputs from a file and
// writes out, loss, the q / k / v gradients and the updated q, so
// tests/test_gpu_reference_tests.py can compare them with the CPU oracle.
//
// File format (little endian): uint32 B, N, D, then q, k, v, target as fp16
// (B*N*D each).  Output: out (B*N*D), loss (1), dq, dk, dv (B*N*D each), q
// after Graph::step(lr = 0.5) (B*N*D), all fp16.
#include <cstdio>
#include <vector>

#include "evk_ai.h"

static bool read_all(FILE* f, void* p, size_t n) { return std::fread(p, 1, n, f) == n; }

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s <in> <out>\n", argv[0]);
        return 2;
    }
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    uint32_t dims[3];
    if (!read_all(f, dims, sizeof(dims))) return 2;
    const uint32_t B = dims[0], N = dims[1], D = dims[2];
    const size_t n = (size_t)B * N * D;
    std::vector<float16_t> host(4 * n);
    if (!read_all(f, host.data(), host.size() * sizeof(float16_t))) return 2;
    std::fclose(f);
    if (!evk::InitializeEVK({.applicationName = "graph_attention_check"})) return 2;
    evk::ai::initialize();
    {
        Graph g;
        Tensor& q = g.tensor(Shape({B, N, D}), true);
        Tensor& k = g.tensor(Shape({B, N, D}), true);
        Tensor& v = g.tensor(Shape({B, N, D}), true);
        Tensor& target = g.tensor(Shape({B, N, D}));
        Tensor& out = g.causal_attention(q, k, v);
        Tensor& loss = g.mse_loss(out, target);
        Tensor* in[4] = {&q, &k, &v, &target};
        for (int i = 0; i < 4; ++i) {
            float16_t* d = in[i]->cpu();
            for (size_t j = 0; j < n; ++j) d[j] = host[i * n + j];
            in[i]->cpu_upload();
        }
        g.eval(true);
        g.step(0.5f);
        evk::ai::SubmitCmd(true);
        std::vector<float16_t> res;
        auto take = [&](Tensor& t) {
            t.cpu_download();
            const float16_t* d = t.cpu();
            res.insert(res.end(), d, d + t.shape.count());
        };
        take(out);
        take(loss);
        take(q.grad());
        take(k.grad());
        take(v.grad());
        take(q);
        FILE* o = std::fopen(argv[2], "wb");
        if (!o || std::fwrite(res.data(), sizeof(float16_t), res.size(), o) != res.size()) return 2;
        std::fclose(o);
    }
    evk::ai::shutdown();
    evk::Shutdown();
    std::printf("GRAPH_OK\n");
    return 0;
}
