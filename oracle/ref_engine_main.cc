// Test-only harness around the reference's own C++ FP16 engine.
//
// ORACLE / TEST INFRASTRUCTURE. This program links the reference engine's
// sources (tensor.cu, weight_loader.cc, layers/*.cu, kernels/*.cu,
// models/*.cu of ginzburg-dev/ml-video-denoiser, compiled unchanged by
// oracle/Makefile) in place of its CLI, whose I/O needs stb/tinyexr. It is
// used by the GPU parity tests and by bench.py's reference-engine timing
// only; the product library never links it.
//
// Inputs and outputs are raw little-endian FP16 files (C-contiguous).
//
//   ref_engine nafnet   <manifest> <in> N C H W <out> [reps]
//       NAFNet::forward (src/models/nafnet.cu:341-389)
//   ref_engine temporal <manifest> <in> N T C H W <out> [reps]
//       NAFNetTemporal::forward (src/models/nafnet_temporal.cu:363-503)
//   ref_engine dcn <manifest> <weight> <bias> <in> N C H W <offsets> <masks>
//                  pad stride dilation groups <out> [reps]
//       DeformConv2dLayer::forward (src/layers/deform_conv2d.cu:105-184)
//   ref_engine conv <manifest> <weight> <bias|-> <in> N C H W pad stride
//                   dilation groups <out> [reps]
//       Conv2dLayer::forward (src/layers/conv2d.cu:94-150)
//
// With reps > 0 the forward runs once more untimed, then reps times between
// two CUDA events on one stream (weights prefetched beforehand, as the
// CLI's --prefetch does, cli/main.cc:225-229); the mean milliseconds per
// forward are printed as `{"ms": ...}` on stdout. A C++ exception (for
// example a cuDNN status the library returns) is printed to stderr and the
// program exits 3.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <functional>
#include <iostream>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "denoiser/layers/conv2d.h"
#include "denoiser/layers/deform_conv2d.h"
#include "denoiser/models/nafnet.h"
#include "denoiser/models/nafnet_temporal.h"
#include "denoiser/tensor.h"
#include "denoiser/weight_loader.h"

namespace {

using denoiser::DType;
using denoiser::Tensor;

std::vector<char> read_file(const std::string& path, size_t want) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    const size_t size = static_cast<size_t>(f.tellg());
    if (size != want)
        throw std::runtime_error(path + ": " + std::to_string(size) + " bytes, expected " + std::to_string(want));
    std::vector<char> buf(size);
    f.seekg(0);
    f.read(buf.data(), static_cast<std::streamsize>(size));
    return buf;
}

Tensor load_f16(const std::string& path, std::vector<int64_t> shape) {
    size_t n = 1;
    for (int64_t d : shape) n *= static_cast<size_t>(d);
    const auto buf = read_file(path, n * sizeof(__half));
    return Tensor::from_host(buf.data(), std::move(shape), DType::kFloat16);
}

void save_f16(const Tensor& t, const std::string& path) {
    std::vector<char> buf(t.nbytes());
    t.to_host(buf.data());
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot write " + path);
    f.write(buf.data(), static_cast<std::streamsize>(buf.size()));
}

int to_int(const char* s) { return std::atoi(s); }

// Runs fwd once (its result is the output), then, with reps > 0, once more
// untimed and reps times between CUDA events.
void run(const std::function<Tensor(cudaStream_t)>& fwd, const std::string& out_path, int reps) {
    cudaStream_t s = nullptr;
    CUDA_CHECK(cudaStreamCreate(&s));
    {
        Tensor y = fwd(s);
        CUDA_CHECK(cudaStreamSynchronize(s));
        save_f16(y, out_path);
    }
    if (reps > 0) {
        { Tensor y = fwd(s); }
        CUDA_CHECK(cudaStreamSynchronize(s));
        cudaEvent_t e0, e1;
        CUDA_CHECK(cudaEventCreate(&e0));
        CUDA_CHECK(cudaEventCreate(&e1));
        CUDA_CHECK(cudaEventRecord(e0, s));
        for (int i = 0; i < reps; ++i) {
            Tensor y = fwd(s);
        }
        CUDA_CHECK(cudaEventRecord(e1, s));
        CUDA_CHECK(cudaEventSynchronize(e1));
        float ms = 0.f;
        CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        std::printf("{\"ms\": %.6f, \"reps\": %d}\n", ms / reps, reps);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    CUDA_CHECK(cudaStreamDestroy(s));
}

int usage() {
    std::fprintf(stderr,
                 "usage: ref_engine nafnet <manifest> <in> N C H W <out> [reps]\n"
                 "       ref_engine temporal <manifest> <in> N T C H W <out> [reps]\n"
                 "       ref_engine dcn <manifest> <weight> <bias> <in> N C H W <offsets> <masks> pad stride "
                 "dilation groups <out> [reps]\n"
                 "       ref_engine conv <manifest> <weight> <bias|-> <in> N C H W pad stride dilation groups "
                 "<out> [reps]\n");
    return 2;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return usage();
    const std::string mode = argv[1];
    try {
        if (mode == "nafnet" && (argc == 9 || argc == 10)) {
            denoiser::WeightStore store(argv[2]);
            store.prefetch_all();
            denoiser::NAFNet model(store);
            const Tensor x = load_f16(argv[3], {to_int(argv[4]), to_int(argv[5]), to_int(argv[6]), to_int(argv[7])});
            run([&](cudaStream_t s) { return model.forward(x, s); }, argv[8], argc == 10 ? to_int(argv[9]) : 0);
        } else if (mode == "temporal" && (argc == 10 || argc == 11)) {
            denoiser::WeightStore store(argv[2]);
            store.prefetch_all();
            denoiser::NAFNetTemporal model(store);
            const Tensor x = load_f16(argv[3], {to_int(argv[4]), to_int(argv[5]), to_int(argv[6]), to_int(argv[7]),
                                                to_int(argv[8])});
            run([&](cudaStream_t s) { return model.forward(x, s); }, argv[9], argc == 11 ? to_int(argv[10]) : 0);
        } else if (mode == "dcn" && (argc == 17 || argc == 18)) {
            denoiser::WeightStore store(argv[2]);
            store.prefetch_all();
            const int N = to_int(argv[6]), C = to_int(argv[7]), H = to_int(argv[8]), W = to_int(argv[9]);
            const int pad = to_int(argv[12]), stride = to_int(argv[13]), dil = to_int(argv[14]),
                      dg = to_int(argv[15]);
            denoiser::DeformConv2dLayer layer(store, argv[3], argv[4], pad, stride, dil, dg);
            const int kh = static_cast<int>(store.get(argv[3]).shape()[2]);
            const int kw = static_cast<int>(store.get(argv[3]).shape()[3]);
            const int Ho = (H + 2 * pad - dil * (kh - 1) - 1) / stride + 1;
            const int Wo = (W + 2 * pad - dil * (kw - 1) - 1) / stride + 1;
            const Tensor x = load_f16(argv[5], {N, C, H, W});
            const Tensor off = load_f16(argv[10], {N, 2 * dg * kh * kw, Ho, Wo});
            const Tensor msk = load_f16(argv[11], {N, dg * kh * kw, Ho, Wo});
            run([&](cudaStream_t s) { return layer.forward(x, off, msk, s); }, argv[16],
                argc == 18 ? to_int(argv[17]) : 0);
        } else if (mode == "conv" && (argc == 15 || argc == 16)) {
            denoiser::WeightStore store(argv[2]);
            store.prefetch_all();
            std::optional<std::string> bias;
            if (std::string(argv[4]) != "-") bias = argv[4];
            denoiser::Conv2dLayer layer(store, argv[3], bias, to_int(argv[10]), to_int(argv[11]), to_int(argv[12]),
                                        to_int(argv[13]));
            const Tensor x = load_f16(argv[5], {to_int(argv[6]), to_int(argv[7]), to_int(argv[8]), to_int(argv[9])});
            run([&](cudaStream_t s) { return layer.forward(x, s); }, argv[14], argc == 16 ? to_int(argv[15]) : 0);
        } else {
            return usage();
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_engine: %s\n", e.what());
        return 3;
    }
    return 0;
}
