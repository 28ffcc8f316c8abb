// denoiser::io::load_image / save_image — source-compatible with the
// reference's include/denoiser/io/image_io.h:9-18, over this library's codecs
// (include/denoiser_b200_io.h) instead of stb. PNG, PPM/PGM and PFM; loads
// (1, 3, H, W) FP16 with value / 255 (src/io/image_io.cc:69-84), saves 8-bit
// clamp(v * 255 + 0.5) (image_io.cc:45-61). JPEG throws runtime_error (no
// JPEG codec in this build).
#pragma once

#include <string>
#include <vector>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser_b200_io.h"

namespace denoiser::io {

namespace detail {

inline void io_check(int rc) {
    if (rc == DN_OK) return;
    throw std::runtime_error(dn_last_error());  // the reference throws runtime_error for every I/O failure
}

inline Tensor load_file(const std::string& path, cudaStream_t stream) {
    int c = 0, h = 0, w = 0;
    io_check(dn_image_probe(path.c_str(), &c, &h, &w));
    std::vector<__half> host(static_cast<size_t>(c) * h * w);
    io_check(dn_image_read(path.c_str(), host.data(), c, h, w));
    Tensor t = Tensor::from_host(host.data(), {1, c, h, w}, DType::kFloat16, stream);
    if (stream) CUDA_CHECK(cudaStreamSynchronize(stream));  // `host` dies on return
    return t;
}

inline void save_file(const Tensor& tensor, const std::string& path, cudaStream_t stream, const char* who) {
    if (tensor.dtype() != DType::kFloat16) throw std::runtime_error(std::string(who) + ": expected FP16 input");
    if (tensor.shape().size() != 4 || tensor.batch() != 1)
        throw std::runtime_error(std::string(who) + ": expected (1, C, H, W) tensor");
    const int c = static_cast<int>(tensor.channels()), h = static_cast<int>(tensor.height()),
              w = static_cast<int>(tensor.width());
    std::vector<__half> host(static_cast<size_t>(c) * h * w);
    tensor.to_host(host.data(), stream);
    if (stream)
        CUDA_CHECK(cudaStreamSynchronize(stream));
    else
        CUDA_CHECK(cudaDeviceSynchronize());
    io_check(dn_image_write(path.c_str(), host.data(), c, h, w));
}

}  // namespace detail

inline Tensor load_image(const std::string& path, cudaStream_t stream = nullptr) {
    return detail::load_file(path, stream);
}

inline void save_image(const Tensor& tensor, const std::string& path, cudaStream_t stream = nullptr) {
    detail::save_file(tensor, path, stream, "save_image");
}

}  // namespace denoiser::io
