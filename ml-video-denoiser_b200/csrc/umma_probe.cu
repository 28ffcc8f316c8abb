// Single-tile tcgen05 GEMM used to validate the UMMA descriptor conventions
// of this engine (no-swizzle K-major operands, fp32 TMEM accumulators, the
// 32x32b TMEM read-back) against a host reference:
//     D[128 x N] = A[128 x K] * B[N x K]^T      (fp16 in, fp32 out)
// It is exposed through the C-ABI as dn_umma_probe and exercised by the GPU
// tests; the production kernels use exactly the same helpers.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sm100.cuh"
#include "status.h"

namespace dnb {
namespace {

constexpr int kM = 128;

__global__ void __launch_bounds__(128) umma_probe_kernel(const __half* __restrict__ A,
                                                          const __half* __restrict__ B,
                                                          float* __restrict__ D, int N, int K,
                                                          uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_base_slot;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const uint32_t sbo = static_cast<uint32_t>(K / 8) * 128u;  // 8-row group stride
    uint8_t* sA = smem;
    uint8_t* sB = smem + kM * K * 2;

    // Stage A (row = thread) and B (rows strided by 128) into the K-major
    // no-swizzle layout: core matrix = 8 rows x 16 B.
    for (int j = 0; j < K / 8; ++j) {
        const uint4 v = *reinterpret_cast<const uint4*>(A + static_cast<size_t>(tid) * K + j * 8);
        *reinterpret_cast<uint4*>(sA + kmajor_offset(tid, j, sbo)) = v;
    }
    for (int n = tid; n < N; n += kM) {
        for (int j = 0; j < K / 8; ++j) {
            const uint4 v = *reinterpret_cast<const uint4*>(B + static_cast<size_t>(n) * K + j * 8);
            *reinterpret_cast<uint4*>(sB + kmajor_offset(n, j, sbo)) = v;
        }
    }
    fence_async_smem();

    uint32_t ncols = 32;
    while (ncols < static_cast<uint32_t>(N)) ncols <<= 1;
    if (warp == 0) {
        tmem_alloc(&tmem_base_slot, ncols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base_slot;

    if (tid == 0) {
        const uint32_t idesc = idesc_f16_f32(kM, N);
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        for (int k = 0; k < K / 16; ++k) {
            // One K=16 step spans two K-adjacent core matrices (lbo = 128 B).
            const uint64_t ad = sdesc_kmajor(a0 + k * 256, 128, sbo);
            const uint64_t bd = sdesc_kmajor(b0 + k * 256, 128, sbo);
            mma_f16(tbase, ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        mma_commit(&bar);
    }
    __syncwarp();
    const bool ok = mbar_wait(&bar, 0);
    if (!ok && (tid & 31) == 0) report_error(err, 1, kErrMbarTimeout);
    tc_fence_after();

    if (ok) {
        const int row = warp * 32 + (tid & 31);
        for (int c = 0; c < N; c += 16) {
            float v[16];
            tmem_ld16(tmem_addr(tbase, warp * 32, c), v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) D[static_cast<size_t>(row) * N + c + i] = v[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tbase, ncols);
}

}  // namespace
}  // namespace dnb

extern "C" int dn_umma_probe(const void* A, const void* B, float* D, int N, int K,
                             uint32_t* err_dev, void* stream) {
    using namespace dnb;
    if (!A || !B || !D) return dn_fail(DN_ERR_INVALID_ARG, "dn_umma_probe: null pointer");
    if (N < 16 || N > 256 || N % 16 != 0 || K < 16 || K > 256 || K % 16 != 0)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_umma_probe: need 16<=N<=256, 16<=K<=256, both %16");
    const size_t smem = static_cast<size_t>(128 + N) * K * 2;
    cudaError_t e = cudaFuncSetAttribute(umma_probe_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_umma_probe: set smem");
    umma_probe_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(A), static_cast<const __half*>(B), D, N, K, err_dev);
    e = cudaGetLastError();
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_umma_probe: launch");
    return DN_OK;
}
