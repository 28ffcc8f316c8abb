// Internal kernel interface of the engine: parameter blocks shared by the
// host planner (engine.cc) and the CUDA kernels, plus their launchers.
// Activations are NHWC fp16 ("rows" = pixels, channels contiguous).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace dnb {

// ---------------------------------------------------------------------------
// tcgen05 row-panel GEMM: out[M, N] = epi( pro(A)[M, K] * B[N, K]^T )
// ---------------------------------------------------------------------------

enum GemmPro : int {
    kProNone = 0,
    kProLayerNorm = 1,  // per-row LayerNorm over K (eps 1e-6), folded into B (gamma) and the epilogue
    kProScale = 2,      // A[m, k] * pro_scale[img(m) * K + k]  (SCA apply)
};

enum GemmEpi : int {
    kEpiStore = 0,       // out = acc + bias
    kEpiGate = 1,        // SimpleGate: out[c] = (acc+b)[c] * (acc+b)[c + half] (in-tile pairs)
    kEpiResidual = 2,    // out = res + res_scale[n] * (acc + bias)
    kEpiShuffleAdd = 3,  // PixelShuffle(2) scatter + skip add
    kEpiShuffleRows = 4, // PixelShuffle(2) + skip add through a staged tile: row-aligned tiles, NT = 4 * out_c,
                         // out_c in {32, 64}; the skip arrives and the two fine rows leave by TMA
};

enum GemmAMode : int {
    kARows = 0,   // row m = pixel m of each segment (1x1 conv; K = nseg * seg_c)
    kAS2x2 = 1,   // 2x2 stride-2 gather: K = 4 * seg_c, tap = k / seg_c
    kARowsPair = 3,  // kARows on CTA pairs (clusters of 2): 256-row tiles, one cta_group::2 MMA per K step,
                     // each CTA loading its 128 A rows and half of the B tile
    kAPairs = 2,  // 2x2 stride-2 by TMA: row-aligned tiles, A chunk = input row 2y+ky viewed as pixel pairs
                  // [Wo][2 seg_c] (k = (2 ky + kx) seg_c + c), needs KC <= 2 seg_c and a swizzled A
};

constexpr int kMaxSeg = 8;

struct GemmParams {
    int M;                     // rows = N_img * Ho * Wo
    int K;                     // logical K
    int hw;                    // pixels per image of the output grid (Ho * Wo)
    int Ho, Wo;                // output grid (S2 gather and pixel shuffle)
    int nseg, seg_c;           // A = concat of nseg segments of seg_c channels
    long long a_img_stride;    // elements between images of every segment source
    const __half* a[kMaxSeg];
    const float* ln_c1;        // LN fold: per packed column sum_k (gamma W)[n,k] (bias holds c2)
    const float* pro_scale;    // [N_img][K]
    const uint8_t* bpack;      // packed B tiles [n_tiles][k_chunks][NT x KC canonical]
    int n_tiles, k_chunks, KC;
    int a_swz;                 // A tile layout: KC*2 (swizzled rows of that span) or 0 (8-column core-matrix columns)
    const float* bias;         // [n_tiles * NT] packed order, may be null
    __half* out;
    int out_c;                 // channels of an output pixel
    int n_out;                 // valid output channels (after gating: half)
    const __half* res;         // residual source (same layout as out)
    const float* res_scale;    // [n_out]
    const __half* skip;        // shuffle-add skip (layout of out)
    uint32_t* err;
    int relu;                  // store epilogue: max(y, 0) (offset-head hidden layer)
};

// NT in {16, 32, 64, 128, 256}
// A GEMM whose per-column parameter vectors do not fit in shared memory beside
// its ring (very wide N) runs as column groups of N tiles, one launch each.
int launch_gemm(const GemmParams& p, int pro, int epi, int amode, int nt, cudaStream_t s);
// Kernels launched by this thread's last launch_gemm call.
int gemm_last_launches();

// Bytes of one packed B tile.
inline size_t gemm_btile_bytes(int nt, int kc) { return static_cast<size_t>(nt) * kc * 2; }

// ---------------------------------------------------------------------------
// Depthwise 3x3 (zero pad) + bias + SimpleGate + global average pool + SCA
// ---------------------------------------------------------------------------

struct DwParams {
    const __half* u;       // [N, H, W, 2D]
    __half* g;             // [N, H, W, D]
    const float* w;        // [9][2D] taps (ky*3+kx) x channel
    const __half* w16;     // [9][2D] the same taps in fp16 (the weights' own precision)
    const float* b;        // [2D]
    int N, H, W, D;
    float* partials;       // [N][blocks][D]
    unsigned* counter;     // [N], zero on entry, reset by the last block
    const float* sca_w;    // [D][D] (out, in)
    const float* sca_b;    // [D]
    float* s_out;          // [N][D] channel attention scale
    uint32_t* err;         // device error word (bounded-wait timeouts)
    // Optional (single image): write bdst = bsrc with column k scaled by
    // s[k], i.e. the packed conv3 B operand with the SCA scale folded in
    // (layout of launch_gemm: tiles [n_tile][k_chunk] of NT x KC, no-swizzle
    // K-major core matrices); b_rows = conv3 output channels.
    const uint8_t* bsrc;
    uint8_t* bdst;
    int b_rows, b_nt, b_kc, b_kchunks;
};

int launch_dw_gate_sca(const DwParams& p, int blocks_per_img, cudaStream_t s);
// SCA alone from existing partials [N][nb][D] (used after the fused phase A).
int launch_sca(const DwParams& p, int nb, cudaStream_t s);
int dw_blocks_per_img(int H, int W, int D);
// TMA-tiled variant (8x32 output tiles x 32-channel slices), then SCA.
bool dw_tile_supported(int D);
int dw_tile_blocks_per_img(int H, int W);
int launch_dw_tile(const DwParams& p, cudaStream_t s);

// ---------------------------------------------------------------------------
// Dense 3x3 convs at the network boundary (CUDA cores)
// ---------------------------------------------------------------------------

// intro: NCHW fp16 input (N, Cin, H, W) -> nan_to_num -> reflect pad to
// (Hp, Wp) -> 3x3 conv (zero pad 1) + bias -> NHWC fp16 (N, Hp, Wp, C0).
struct IntroParams {
    const __half* x;
    int N, Cin, H, W, Hp, Wp, C0;
    int in_batch_stride;   // elements between images of x (Cin*H*W, or T*Cin*H*W for clips)
    const float* w;        // [C0][Cin][3][3]
    const float* b;        // [C0]
    __half* y;
    uint32_t* err;         // error word of the tensor-core form
};
int launch_intro(const IntroParams& p, cudaStream_t s);
// The same conv on the tensor cores (intro_tc.cu): an im2col MMA per strip row.
bool intro_tc_supported(int Cin, int C0);
int launch_intro_tc(const IntroParams& p, cudaStream_t s);

// ending: NHWC (N, Hp, Wp, C0) -> 3x3 conv C0 -> 3 + bias, crop to (H, W),
// + beauty (nan_to_num of the first 3 channels of the NCHW input) -> NCHW fp16.
struct EndingParams {
    const __half* x;       // NHWC
    int N, Hp, Wp, C0, H, W;
    const float* w;        // [3][3][3][C0] (out, ky, kx, c)
    const float* b;        // [3]
    const __half* beauty;  // NCHW input
    int beauty_batch_stride;
    __half* y;             // NCHW (N, 3, H, W)
    // Tensor-core form (fused_a_tc.cu): B tiles [3 kx][C0/16 K steps][ky = 2, 1, 0]
    // of 16 output rows (3 used) x 16 channels; nullptr = the CUDA-core kernel.
    const uint8_t* weff;
    uint32_t* err;
};
int launch_ending(const EndingParams& p, cudaStream_t s);
bool ending_tc_supported(int C0);
int launch_ending_tc(const EndingParams& p, cudaStream_t s);

}  // namespace dnb
