// ext_check.cpp — drives the evk_ai_ext.h extensions through libevk_ai.so on
// inputs read from a file and writes their outputs, so
// tests/test_gpu_reference_tests.py can compare them with the CPU oracle.
// Cases (fixed shapes, all tensors 2-byte storage unless noted):
//   1 flash_attention_ex   bf16, B 1, N 160, heads 4, Hkv 2, Dh 64, causal
//   2 single_query_attention bf16, B 2, heads 4, Hkv 2, Dh 64, max_len 100, cur_len 77
//   3 rope_ex              bf16, B 2, S 5, D 256, head_dim 64, pos_offset 11
//   4 rms_norm_ex          bf16, 6 rows of 256, eps 1e-5, gamma (256)
//   5 embed_ex             fp16, V 70000, D 16, 10 uint32 ids
//   6 greedy_sample_ex     fp16, logits (2, 1, 70000), uint32 ids
// Input file: the inputs of cases 1..6 in order (q, k, v | q, kc, vc | x | x,
// gamma | E, ids | logits).  Output file: o | out | out | out | out | ids.
#include <cstdio>
#include <vector>

#include "evk_ai_ext.h"

using evk::ai::DType;

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    std::vector<uint16_t> in;
    {
        uint16_t buf[4096];
        size_t got;
        while ((got = std::fread(buf, 2, 4096, f)) > 0) in.insert(in.end(), buf, buf + got);
        std::fclose(f);
    }
    if (!evk::InitializeEVK({.applicationName = "ext_check"})) return 2;
    evk::ai::initialize();
    size_t pos = 0;
    std::vector<uint16_t> res;
    auto load = [&](Tensor& t) {
        uint16_t* d = reinterpret_cast<uint16_t*>(t.cpu());
        for (uint32_t i = 0; i < t.shape.count(); ++i) d[i] = in.at(pos++);
        t.cpu_upload();
    };
    auto take = [&](Tensor& t) {
        t.cpu_download();
        const uint16_t* d = reinterpret_cast<const uint16_t*>(t.cpu());
        res.insert(res.end(), d, d + t.shape.count());
    };
    {
        Tensor q({1, 160, 256}), k({1, 160, 128}), v({1, 160, 128}), o({1, 160, 256});
        load(q), load(k), load(v);
        evk::ai::flash_attention_ex(q, k, v, o, 4, true, 0.0f, DType::BF16);
        take(o);
    }
    {
        Tensor q({2, 256}), kc({2, 100, 128}), vc({2, 100, 128}), o({2, 256});
        load(q), load(kc), load(vc);
        evk::ai::single_query_attention(q, kc, vc, o, 4, 77, 0.0f, DType::BF16);
        take(o);
    }
    {
        Tensor x({2, 5, 256}), o({2, 5, 256});
        load(x);
        evk::ai::rope_ex(x, o, 2, 5, 256, 10000.0f, 64, 11, DType::BF16);
        take(o);
    }
    {
        Tensor x({6, 256}), g({256}), o({6, 256});
        load(x), load(g);
        evk::ai::rms_norm_ex(x, o, 1e-5f, &g, DType::BF16);
        take(o);
    }
    {
        Tensor E({70000, 16}), ids({20}), o({10, 16});  // 10 uint32 ids in 20 two-byte slots
        load(E), load(ids);
        evk::ai::embed_ex(E, ids, o, 4);
        take(o);
    }
    {
        Tensor l({2, 1, 70000}), ids({4});  // 2 uint32 ids
        load(l);
        evk::ai::greedy_sample_ex(l, ids, 0, 0, 70000, 4);
        take(ids);
    }
    evk::ai::SubmitCmd(true);
    FILE* o = std::fopen(argv[2], "wb");
    if (!o || std::fwrite(res.data(), 2, res.size(), o) != res.size()) return 2;
    std::fclose(o);
    evk::ai::shutdown();
    evk::Shutdown();
    std::printf("EXT_OK\n");
    return 0;
}
