// drop_in_check.cpp — runs the reference's own decode loop with the "b200" variants.
//
//   drop_in_check <model.tqwen> <mode> <max_seq> <n_new> <tok0> [tok1 ...]
//   mode: ref            reference CPU path (matvec/ops "ref")
//         ops            QwenModel::forward_token with --matvec-impl b200 --ops-impl b200
//         engine         the GPU decode registry with --engine b200 (gpu_decode_* entries)
//         backend        QwenModel::forward_token on create_b200_backend() (every op of the
//                        IBackend on the GPU), fp32 KV cache
//         backend-f16kv  the same with QwenModel's fp16 KV cache (--kv-f16: attention
//                        through IBackend::attention_decode_f16kv)
// Prints the greedy token after every fed token on one line, as main.cpp's decode
// loop produces them (runtime/main.cpp:1009-1041).
//
//   drop_in_check <data.bin> matmul <M> <K> <N> <G>
//   tinyqwen::matmul_i4 through the reference's dispatcher (the prefill contraction,
//   QwenModel::mm -> CPUBackend::matmul) on data.bin = [W i4 rows][X, N columns of K
//   floats]; writes Y (N columns of M floats) to data.bin.y and prints how many calls
//   reached the b200 variant.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "b200_backend.h"
#include "dispatch.h"
#include "model_loader.h"
#include "profiler.h"
#include "qwen_model.h"

namespace tinyqwen {
extern int g_matmul_calls;  // b200_variants.cpp
}

static int run_matmul(const std::string &path, int M, int K, int N, int G) {
    const size_t wb = (size_t)M * ((K + G - 1) / G) * (4 + G / 2);
    std::vector<uint8_t> w(wb);
    std::vector<float> x((size_t)K * N), y((size_t)M * N);
    FILE *f = std::fopen(path.c_str(), "rb");
    if (!f || std::fread(w.data(), 1, wb, f) != wb ||
        std::fread(x.data(), 4, x.size(), f) != x.size()) {
        std::fprintf(stderr, "matmul: cannot read %s\n", path.c_str());
        if (f) std::fclose(f);
        return 1;
    }
    std::fclose(f);
    tinyqwen::matmul_i4(w.data(), x.data(), y.data(), M, K, N, G);
    f = std::fopen((path + ".y").c_str(), "wb");
    if (!f || std::fwrite(y.data(), 4, y.size(), f) != y.size()) {
        std::fprintf(stderr, "matmul: cannot write %s.y\n", path.c_str());
        if (f) std::fclose(f);
        return 1;
    }
    std::fclose(f);
    std::printf("b200 matmul calls %d\n", tinyqwen::g_matmul_calls);
    return 0;
}

int main(int argc, char **argv) {
    if (argc == 7 && std::strcmp(argv[2], "matmul") == 0)
        return run_matmul(argv[1], std::atoi(argv[3]), std::atoi(argv[4]), std::atoi(argv[5]),
                          std::atoi(argv[6]));
    if (argc < 6) {
        std::fprintf(stderr, "usage: %s model mode max_seq n_new tok...\n", argv[0]);
        return 2;
    }
    const std::string path = argv[1], mode = argv[2];
    const int max_seq = std::atoi(argv[3]), n_new = std::atoi(argv[4]);
    std::vector<int> prompt;
    for (int i = 5; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
    tinyqwen::ModelFile file;
    std::string err;
    if (!file.load(path, &err)) {
        std::fprintf(stderr, "load: %s\n", err.c_str());
        return 1;
    }
    std::vector<int> out;
    if (mode == "engine") {
        if (!tinyqwen::set_gpu_decode_impl_by_name("b200")) {
            std::fprintf(stderr, "no b200 engine registered (have: %s)\n",
                         tinyqwen::available_gpu_decode_impls());
            return 1;
        }
        tinyqwen::GpuDecodeEngine *eng = nullptr;
        if (!tinyqwen::gpu_decode_create(&file, max_seq, &err, &eng)) {
            std::fprintf(stderr, "engine create: %s\n", err.c_str());
            return 1;
        }
        int next = -1;
        for (int t : prompt) out.push_back(next = tinyqwen::gpu_decode_step(eng, t));
        for (int s = 1; s < n_new; ++s) out.push_back(next = tinyqwen::gpu_decode_step(eng, next));
        tinyqwen::gpu_decode_destroy(eng);
    } else if (mode == "backend" || mode == "backend-f16kv") {
        tinyqwen::Profiler profiler(false);
        std::unique_ptr<tinyqwen::QwenModel> model;
        if (!tinyqwen::QwenModel::create(file, max_seq, profiler, &err, &model, create_b200_backend(),
                                         mode == "backend-f16kv")) {
            std::fprintf(stderr, "model create: %s\n", err.c_str());
            return 1;
        }
        int next = -1;
        for (int t : prompt) out.push_back(next = model->forward_token(t));
        for (int s = 1; s < n_new; ++s) out.push_back(next = model->forward_token(next));
    } else {
        const char *impl = mode == "ops" ? "b200" : "ref";
        if (!tinyqwen::set_matvec_i4_impl_by_name(impl) ||
            !tinyqwen::set_matvec_vq2_impl_by_name(impl) || !tinyqwen::set_ops_impl_by_name(impl)) {
            std::fprintf(stderr, "no '%s' matvec/ops variants registered\n", impl);
            return 1;
        }
        tinyqwen::Profiler profiler(false);
        std::unique_ptr<tinyqwen::QwenModel> model;
        if (!tinyqwen::QwenModel::create(file, max_seq, profiler, &err, &model)) {
            std::fprintf(stderr, "model create: %s\n", err.c_str());
            return 1;
        }
        int next = -1;
        for (int t : prompt) out.push_back(next = model->forward_token(t));
        for (int s = 1; s < n_new; ++s) out.push_back(next = model->forward_token(next));
    }
    for (size_t i = 0; i < out.size(); ++i) std::printf(i ? " %d" : "%d", out[i]);
    std::printf("\n");
    return 0;
}
