// Depthwise 3x3 + bias + SimpleGate + pool partials for the deep levels.
// A persistent CTA owns one 32-channel slice of one image and walks that
// image's TH x TW output tiles; two halo buffers let the TMA load of the
// tile after next overlap the current tile's math, and the slice's taps stay
// in registers for the whole walk. Per tile:
//   * two TMA loads bring the (TH+2) x (TW+2) halo of both gate halves of the
//     slice (u channels [c, c+32) and [D+c, D+c+32)) into shared memory,
//     zero-filled outside the image (the conv's zero padding);
//   * a thread owns one gate half x 8 channels (fp16 taps in registers) at
//     one column and produces four vertically adjacent outputs from a 6-row
//     window, multiplying fp16 inputs by fp16 taps into fp32 sums with
//     mixed-precision FMAs (the fp32 result of the widened operands, without
//     converting them); the halves of a gate pair are lanes l and l^8;
//   * the gated tile leaves by one TMA store; each thread adds the stored
//     fp16 values of its column to running sums, in the CTA's fixed tile
//     order; after the walk they reduce over columns and warps in a fixed
//     order into partials[img][blockIdx.x][channel] (one pool row per CTA
//     keeps the SCA kernel's re-reduction short).
// Each input element crosses the memory system once (plus the 1-pixel halo),
// instead of once per tap.
//
// Replaces the reference's grouped cudnnConvolutionForward (conv2) +
// simple_gate_kernel + global_avg_pool_kernel passes (src/models/nafnet.cu
// :162-172, src/kernels/nafnet_kernels.cu:94-126) at the deep levels.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <string>

#include "kernels.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "status.h"

namespace dnb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace {

constexpr int kCS = 32;            // gated channels per CTA
constexpr int kTH = 8, kTW = 32;   // output tile
constexpr int kR = 4;              // output rows per thread per window
constexpr int kHH = kTH + 2, kWW = kTW + 2;
constexpr int kP = kHH * kWW;      // halo pixels
constexpr int kRowB = kCS * 2;     // 64 bytes per halo pixel and half
constexpr int kBufB = ((kP * kRowB + 127) / 128) * 128;
constexpr int kOutB = kTH * kTW * kCS * 2;
constexpr int kThreads = 256;
constexpr int kSmem = 128 + 4 * kBufB + kOutB + (kThreads / 32) * kCS * 4;  // 2 halo buffers x 2 gate halves

// Lane layout inside a warp (32 lanes = 4 columns): bits 0-1 channel group,
// bit 2 column low bit, bit 3 gate half, bit 4 column high bit. Eight
// consecutive lanes then read 128 contiguous bytes of one half (no bank
// conflicts) and the two halves of a gate pair are lanes l and l^8.
__global__ void __launch_bounds__(kThreads, 2)
    dw_tile_kernel(const __grid_constant__ DwParams p, const __grid_constant__ CUtensorMap mu,
                   const __grid_constant__ CUtensorMap mg) {
    if (threadIdx.x == 0) {
        prefetch_tmap(&mu);
        prefetch_tmap(&mg);
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
    uint8_t* sOut = smem + 4 * kBufB;                              // [TH*TW][CS] fp16
    float* sRed = reinterpret_cast<float*>(sOut + kOutB);          // [warps][CS]
    __shared__ uint64_t bar[2];

    const int tid = threadIdx.x;
    const int tiles_x = (p.W + kTW - 1) / kTW;
    const int ntiles = tiles_x * ((p.H + kTH - 1) / kTH);
    const int img = blockIdx.z;
    const int D = p.D;
    const int cs0 = blockIdx.y * kCS;

    pdl_trigger();
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    const int lane = tid & 31;
    const int cg = lane & 3;
    const int half = (lane >> 3) & 1;
    const int px = (tid >> 5) * 4 + ((lane >> 4) << 1) + ((lane >> 2) & 1);  // 0..31
    const int cin = half * D + cs0 + cg * 8;
    uint32_t w[9][4];  // taps of channels (cin + 2i, cin + 2i + 1) as fp16 pairs
    float bias[8];
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        const uint4 v = *reinterpret_cast<const uint4*>(p.w16 + t * 2 * D + cin);
        w[t][0] = v.x;
        w[t][1] = v.y;
        w[t][2] = v.z;
        w[t][3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) bias[i] = p.b[cin + i];
    __syncthreads();  // barriers initialised before anyone waits on them
    pdl_wait();
    // Halo of tile t (both gate halves) into buffer b.
    auto load = [&](int t, int b) {
        const int ty0 = (t / tiles_x) * kTH, tx0 = (t % tiles_x) * kTW;
        uint8_t* dst = smem + b * 2 * kBufB;
        mbar_arrive_expect_tx(&bar[b], 2 * kP * kRowB);
        tma_load_4d(dst, &mu, cs0, tx0 - 1, ty0 - 1, img, &bar[b]);
        tma_load_4d(dst + kBufB, &mu, D + cs0, tx0 - 1, ty0 - 1, img, &bar[b]);
    };
    if (tid == 0) {
        if (static_cast<int>(blockIdx.x) < ntiles) load(blockIdx.x, 0);
        if (static_cast<int>(blockIdx.x + gridDim.x) < ntiles) load(blockIdx.x + gridDim.x, 1);
    }

    // Running pool sums over the CTA's tiles (in its fixed tile order) of
    // channels cs0 + cg * 8 + half * 4 + i at this thread's column.
    float ps[4] = {0, 0, 0, 0};
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int b = it & 1;
        const int ty0 = (t / tiles_x) * kTH, tx0 = (t % tiles_x) * kTW;
        if (tid == 0) bulk_wait_read0();  // the previous tile's store has read sOut
        const bool ok = mbar_wait(&bar[b], (it >> 1) & 1);
        if (!__syncthreads_and(ok)) {
            if (tid == 0) report_error(p.err, 0x50, kErrMbarTimeout);
            break;
        }
        const uint8_t* src = smem + b * 2 * kBufB + half * kBufB + cg * 16;
        const bool col_in = tx0 + px < p.W;
#pragma unroll 1
        for (int py = 0; py < kTH; py += kR) {
            // kR output rows from a window of kR + 2 input rows: each loaded
            // pixel feeds every output row whose 3x3 window holds it, with
            // fp16 x fp16 products accumulated in fp32 (no unpacking).
            float acc[kR][8];
#pragma unroll
            for (int r = 0; r < kR; ++r)
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[r][i] = bias[i];
#pragma unroll
            for (int rr = 0; rr < kR + 2; ++rr) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const uint4 v = *reinterpret_cast<const uint4*>(src + ((py + rr) * kWW + px + kx) * kRowB);
                    const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int r = 0; r < kR; ++r) {
                        const int ky = rr - r;
                        if (ky < 0 || ky > 2) continue;
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            fma_mix2(acc[r][2 * i], acc[r][2 * i + 1], q[i], w[ky * 3 + kx][i]);
                    }
                }
            }
#pragma unroll
            for (int r2 = 0; r2 < kR; ++r2) {
                // this lane keeps channels [4*half, 4*half+4) of its group
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float lo = acc[r2][j], hi = acc[r2][4 + j];
                    const float mine = half ? hi : lo;
                    const float give = half ? lo : hi;
                    o[j] = mine * __shfl_xor_sync(0xffffffffu, give, 8);
                }
                const int oy = py + r2;
                const uint32_t h01 = pack_half2(o[0], o[1]), h23 = pack_half2(o[2], o[3]);
                *reinterpret_cast<uint2*>(sOut + ((oy * kTW + px) * kCS + cg * 8 + half * 4) * 2) = make_uint2(h01, h23);
                if (col_in && ty0 + oy < p.H) {
                    const float2 f01 = unpack_half2(h01), f23 = unpack_half2(h23);
                    ps[0] += f01.x;
                    ps[1] += f01.y;
                    ps[2] += f23.x;
                    ps[3] += f23.y;
                }
            }
        }
        fence_async_smem();
        __syncthreads();  // every thread is done with halo buffer b and sOut is complete
        if (tid == 0) {
            tma_store_4d(&mg, cs0, tx0, ty0, img, sOut);
            bulk_commit();
            if (t + 2 * static_cast<int>(gridDim.x) < ntiles) load(t + 2 * gridDim.x, b);
        }
    }
    // Pool partials of the walk: the 4 columns of a warp (lane bits 2 and 4),
    // then the 8 warps in order.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        ps[i] += __shfl_xor_sync(0xffffffffu, ps[i], 4);
        ps[i] += __shfl_xor_sync(0xffffffffu, ps[i], 16);
    }
    if ((lane & 0x14) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sRed[(tid >> 5) * kCS + cg * 8 + half * 4 + i] = ps[i];
    }
    __syncthreads();
    if (tid < kCS) {
        float sum = 0.f;
#pragma unroll
        for (int w8 = 0; w8 < kThreads / 32; ++w8) sum += sRed[w8 * kCS + tid];
        p.partials[(static_cast<size_t>(img) * gridDim.x + blockIdx.x) * D + cs0 + tid] = sum;
    }
    if (tid == 0) bulk_wait0();
}

int encode4(CUtensorMap* m, const void* base, int C, int W, int H, int N, int box_c, int box_w, int box_h) {
    auto fn = tensor_map_encoder();
    if (!fn) return dn_fail(DN_ERR_CUDA, "dw_tile: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                                static_cast<cuuint64_t>(N)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(W) * C * 2,
                                   static_cast<cuuint64_t>(H) * W * C * 2};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(box_c), static_cast<cuuint32_t>(box_w),
                               static_cast<cuuint32_t>(box_h), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return dn_fail_str(DN_ERR_CUDA, "dw_tile: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return DN_OK;
}

}  // namespace

bool dw_tile_supported(int D) { return D % kCS == 0; }

int dw_tile_blocks_per_img(int H, int W) { return ((H + kTH - 1) / kTH) * ((W + kTW - 1) / kTW); }

int launch_dw_tile(const DwParams& p, cudaStream_t s) {
    if (!dw_tile_supported(p.D)) return dn_fail(DN_ERR_UNSUPPORTED, "dw_tile: channels must be a multiple of 32");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(dw_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dw_tile: smem attribute");
        configured = true;
    }
    CUtensorMap mu, mg;
    int rc = encode4(&mu, p.u, 2 * p.D, p.W, p.H, p.N, kCS, kWW, kHH);
    if (rc == DN_OK) rc = encode4(&mg, p.g, p.D, p.W, p.H, p.N, kCS, kTW, kTH);
    if (rc != DN_OK) return rc;
    const int tiles = dw_tile_blocks_per_img(p.H, p.W);
    // At most two CTAs per SM in total (one wave: a CTA over the limit would
    // start only when another has walked all of its tiles); the tiles are
    // then spread evenly, so every CTA walks the same ceil(tiles / grid_x).
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int per = (p.D / kCS) * p.N;
    const int gmax = std::max(1, std::min(tiles, 2 * sms / per));
    const int walk = (tiles + gmax - 1) / gmax;
    const int gx = (tiles + walk - 1) / walk;
    cudaError_t e = launch_pdl(dw_tile_kernel, dim3(gx, p.D / kCS, p.N), dim3(kThreads), kSmem, s, p, mu, mg);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dw_tile: launch");
    return launch_sca(p, gx, s);
}

}  // namespace dnb
