// denoiser::NAFNetTemporal — source-compatible with the reference's
// include/denoiser/models/nafnet_temporal.h:11-29. Loads both temporal
// export layouts (the C++ engine's temporal_mix.N and the PyTorch model's
// bottleneck_mix / temporal_mix.N.0).
#pragma once

#include <stdexcept>
#include <vector>

#include "denoiser/models/nafnet.h"

namespace denoiser {

class NAFNetTemporal {
public:
    explicit NAFNetTemporal(const WeightStore& store) : e_(store) {
        if (e_.info().kind == 0) throw std::runtime_error("NAFNetTemporal: the manifest holds a spatial model");
    }
    NAFNetTemporal(const NAFNetTemporal&) = delete;
    NAFNetTemporal& operator=(const NAFNetTemporal&) = delete;

    // clip (N, T, C, H, W) FP16 -> denoised centre frame (N, 3, H, W) FP16.
    Tensor forward(const Tensor& clip, cudaStream_t stream = nullptr) const { return e_.run(clip, 5, stream); }

    int num_frames() const noexcept { return e_.info().num_frames; }
    int num_levels() const noexcept { return e_.info().num_levels; }
    const std::vector<int>& enc_channels() const noexcept { return e_.enc(); }
    bool use_warp() const noexcept { return e_.info().use_warp != 0; }

private:
    detail::EngineHandle e_;
};

}  // namespace denoiser
