// The NAFNet inference engine: weights packed once into one device arena in
// the layouts the kernels consume, an activation arena planned per input
// shape, and the launch sequence of the spatial NAFNet
// (src/models/nafnet.cu:341-389) and of the C++ engine's temporal model
// (src/models/nafnet_temporal.cu:363-503).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "kernels.h"
#include "manifest.h"

namespace dnb {

// Packed 1x1 / 2x2 conv for launch_gemm.
struct GemmW {
    size_t bpack = 0;      // arena offset of the packed B tiles
    size_t bias = 0;       // arena offset of the fp32 bias (packed order; LN fold: c2)
    bool has_bias = false;
    size_t c1 = 0;         // LN fold: arena offset of c1 (packed order)
    bool has_c1 = false;
    int NT = 0, KC = 0, n_tiles = 0, k_chunks = 0;
    int a_swz = 0;         // A layout span the kernel uses (KC*2, or 0 = interleaved)
    int K = 0;             // logical K
    int n_out = 0;         // output channels the epilogue writes
};

struct BlockW {
    int C = 0, dw = 0, ffn = 0;
    size_t ln1w = 0, ln1b = 0, ln2w = 0, ln2b = 0, beta = 0, gamma = 0;  // fp32 [C]
    GemmW conv1, conv3, conv4, conv5;
    size_t dw_w = 0, dw_b = 0;     // fp32 [9][2dw], [2dw]
    size_t dw_w16 = 0;             // fp16 [9][2dw]: the same taps, for the mixed-precision depthwise
    size_t sca_w = 0, sca_b = 0;   // fp32 [dw][dw], [dw]
    // Fused two-pass kernels (shallow levels, C <= 64): single-tile B images.
    bool fused = false;
    GemmW f1, f3, f4, f5;          // conv1 (LN folded), conv3, conv4, conv5
    // Tensor-core phase A: Weff B tiles and b1' = b1 + W1 beta1 (fp32 [2dw]).
    bool fa_tc = false;
    size_t fa_w = 0, fa_b1 = 0;
    // Single-kernel second pass (C = D = F = 128 / 256): conv4 with LN2 folded
    // as 128-row tiles [64 a rows | 64 b rows] per 64-channel gate chunk.
    bool deep = false;
    GemmW d4;
};

struct ModelInfo {
    int kind = 0;          // 0 spatial, 1 temporal (C++ engine design), 2 temporal (PyTorch design)
    int in_channels = 3;
    int num_levels = 0;
    int base_channels = 0;
    int num_frames = 1;
    int use_warp = 0;
    std::vector<int> enc_channels;
};

class Engine {
public:
    Engine(const std::string& manifest_path, int device);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    const ModelInfo& info() const { return info_; }
    int device() const { return device_; }

    // Spatial: x (N, C, H, W) fp16 NCHW device -> y (N, 3, H, W).
    // Temporal: x (N, T, C, H, W) clip -> y (N, 3, H, W) (denoised centre frame).
    // Returns DN_OK or a DN_ERR_* code (message via dn_last_error).
    int forward(const __half* x, int N, int T, int C, int H, int W, __half* y, cudaStream_t s);

    // Temporal models, one sequence frame at a time: encode_frame runs the
    // encoder on one (1, C, H, W) frame into cache slot `slot` (0 .. T-1);
    // decode_window denoises the window whose frame t is in slots[t], with
    // `beauty` = the (1, C, H, W) reference frame. A sequence then encodes
    // every frame once instead of T times.
    int encode_frame(const __half* frame, int C, int H, int W, int slot, cudaStream_t s);
    int decode_window(const int* slots, const __half* beauty, int C, int H, int W, __half* y, cudaStream_t s);

    // Waits for `s` and returns DN_ERR_DEVICE if a kernel flagged an error
    // since the last check (the word is cleared).
    int check_device(cudaStream_t s);

    // Per-launch CUDA-event timing of the engine's own kernels (off by
    // default). Each launch is tagged with its kind and its algorithmic bytes
    // (inputs read once + outputs written once) and FLOPs.
    // 0 off, 1 per kernel kind, 2 per kind and shape ("kind@shape")
    void set_profiling(int mode) {
        profiling_ = mode != 0;
        prof_detail_ = mode == 2;
    }
    // 1: fused NAFBlock kernels where they apply (default), with phase A of the
    // 32/64-channel blocks and the ending conv on the tensor cores; 2: the same
    // with those two on the CUDA cores; 0: per-conv kernels everywhere.
    void set_fused(int mode) {
        fused_enabled_ = mode != 0;
        fa_tc_enabled_ = mode != 2;
        fa_split_enabled_ = mode == 3;
        gemm_tma_enabled_ = mode == 1 || mode == 3;
        gemm_pair_enabled_ = mode == 4;
        if (mode == 4) gemm_tma_enabled_ = true;
    }
    // Synchronises, then returns a JSON object: kind -> {launches, ms, bytes, flops}
    // accumulated since the last report (which also resets the counters).
    std::string profile_report();

    size_t weight_bytes() const { return warena_bytes_; }
    size_t activation_bytes() const { return aarena_bytes_; }
    int kernels_per_forward() const { return launches_; }

private:
    struct Level {
        int C = 0;
        std::vector<BlockW> enc, dec;
        GemmW down;  // C -> 2C, 2x2 s2
        GemmW up;    // ups feeding this level: 2C -> 4*C, shuffle to C
    };
    struct Shape {
        int N = 0, T = 0, H = 0, W = 0, Hp = 0, Wp = 0;
        bool operator==(const Shape& o) const {
            return N == o.N && T == o.T && H == o.H && W == o.W;
        }
    };

    void build(const HostWeights& hw);
    void plan(const Shape& s);
    int make_shape(int N, int T, int C, int H, int W, Shape& sh);
    int encode_into(const __half* src, int nimg, int in_stride, int slot0, cudaStream_t s);
    int decode_from(__half* xm, int nimg, const std::vector<__half*>& skips, const __half* beauty, int beauty_stride,
                    __half* out, cudaStream_t s);
    int temporal_tail(const int* slots, const __half* beauty, int beauty_stride, __half* y, cudaStream_t s);
    int run_block(const BlockW& b, __half* x, int nimg, int h, int w, cudaStream_t s);
    int run_stage(const std::vector<BlockW>& blocks, __half* x, int nimg, int h, int w, cudaStream_t s);
    int gemm(const GemmW& g, int pro, int epi, int amode, GemmParams p, cudaStream_t s,
             const uint8_t* bpack_override = nullptr);

    template <class T>
    const T* wptr(size_t off) const {
        return reinterpret_cast<const T*>(warena_ + off);
    }

    int device_ = 0;
    ModelInfo info_;
    int pad_multiple_ = 1;

    // weights
    uint8_t* warena_ = nullptr;
    size_t warena_bytes_ = 0;
    std::vector<Level> levels_;
    std::vector<BlockW> middle_;
    size_t intro_w_ = 0, intro_b_ = 0, ending_w_ = 0, ending_b_ = 0;
    size_t ending_tc_w_ = 0;  // tensor-core ending B tiles (0 = none)
    // temporal (C++ engine design): per level temporal_mix over
    // concat(ref, nbr_1..nbr_{T-1}) with the neighbour mean folded into B,
    // and optional offset heads (1x1, 2C -> 2).
    std::vector<GemmW> tmix_;
    std::vector<GemmW> offset_heads_;
    // temporal (PyTorch design, training/models.py:651-808): bottleneck_mix
    // (T*C -> C 1x1 + NAFBlocks) on the T deep features, per level
    // temporal_mix (T*C -> C 1x1 + NAFBlocks) on the T skips, and optional
    // offset heads (DW 3x3 -> PW 2C->C -> ReLU -> PW C->2) with grid_sample warp.
    GemmW bneck_;
    std::vector<BlockW> bneck_blocks_;
    std::vector<std::vector<BlockW>> tmix_blocks_;
    std::vector<size_t> oh_dw_;               // fp32 [9][2C] per level
    std::vector<GemmW> oh_pw1_, oh_pw2_;

    // activations
    Shape shape_{};
    uint8_t* aarena_ = nullptr;
    size_t aarena_bytes_ = 0;
    std::vector<__half*> enc_x_, dec_x_;  // per level (encoder state/skip, decoder state)
    __half* mid_x_ = nullptr;
    __half *buf_u_ = nullptr, *buf_g_ = nullptr, *buf_y_ = nullptr, *buf_t_ = nullptr;
    std::vector<__half*> fused_skip_;     // temporal: fused skip per level
    __half* warp_buf_ = nullptr;          // temporal: warped neighbours [T-1][...]
    __half* offset_buf_ = nullptr;        // temporal: offsets [HW][8]
    __half* bneck_x_ = nullptr;           // temporal (PyTorch design): fused deep feature
    __half* oh_d_ = nullptr;              // offset head: depthwise output [HW][2C]
    __half* oh_h_ = nullptr;              // offset head: hidden layer [HW][C]
    float* partials_ = nullptr;
    unsigned* counters_ = nullptr;
    float* sca_s_ = nullptr;
    uint8_t* b3s_ = nullptr;              // conv3 B with the SCA scale folded in (single image)
    uint32_t* err_ = nullptr;
    int dw_blocks_max_ = 0;
    int launches_ = 0;

    // profiling
    struct ProfRec {
        std::string kind;
        double bytes, flops;
        cudaEvent_t a, b;
    };
    void prof_begin(const char* kind, double bytes, double flops, cudaStream_t s);
    void prof_end(cudaStream_t s);
    bool profiling_ = false;
    bool prof_detail_ = false;
    std::string prof_tag_;  // shape suffix of the next prof_begin in detail mode
    bool fused_enabled_ = true;
    bool fa_tc_enabled_ = true;
    bool gemm_tma_enabled_ = true;   // stride-2 down by TMA pair loads, staged pixel-shuffle up (modes 1, 3)
    bool gemm_pair_enabled_ = false;  // 1x1 conv GEMMs on CTA pairs, cta_group::2 (mode 4)
    bool fa_split_enabled_ = false;  // phase A of single images: conv1 MMA + CUDA-core depthwise (mode 3)
    std::vector<ProfRec> prof_;
    std::vector<cudaEvent_t> prof_pool_;
    size_t prof_used_ = 0;
};

}  // namespace dnb
