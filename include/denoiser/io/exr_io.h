// denoiser::io::load_exr / save_exr — source-compatible with the reference's
// include/denoiser/io/exr_io.h:9-18, over this library's OpenEXR codec
// (include/denoiser_b200_io.h) instead of tinyexr: loads R,G,B (else Y, else
// the first channel) as FP16 (src/io/exr_io.cc:76-114); saves 1 (Y) or 3
// (B,G,R) HALF channels (exr_io.cc:122-196).
#pragma once

#include "denoiser/io/image_io.h"

namespace denoiser::io {

inline Tensor load_exr(const std::string& path, cudaStream_t stream = nullptr) {
    return detail::load_file(path, stream);
}

inline void save_exr(const Tensor& tensor, const std::string& path, cudaStream_t stream = nullptr) {
    if (tensor.shape().size() == 4 && tensor.channels() != 1 && tensor.channels() != 3)
        throw std::runtime_error("save_exr: only C=1 or C=3 supported, got C=" + std::to_string(tensor.channels()));
    detail::save_file(tensor, path, stream, "save_exr");
}

}  // namespace denoiser::io
