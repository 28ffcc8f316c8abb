// Temporal NAFNet with deformable alignment (FP16, batch 1, 3-channel
// frames), as an engine component with a per-frame cache:
//
//   f_t   = feat(frame_t)                            3x3 conv, 3 -> F (NHWC)
//   om_ct = offset(concat(f_c, f_t))                 3x3 conv, 2F -> 3*dg*9
//         = Q_c + P_t,  Q_c = W_ctr * f_c + b,  P_t = W_nbr * f_t
//   a_t   = dcn(f_t, om_ct[:2*dg*9], om_ct[2*dg*9:]) DCNv2 3x3, F -> F (sigmoid masks)
//   a_c   = f_c
//   fused = b_f + sum_t W_f,t a_t + frame_c          1x1 fusion, T*F -> 3
//   out   = NAFNet(fused)                            the spatial engine
//
// The reference has DeformConv2dLayer (src/layers/deform_conv2d.cu:105-184)
// but wires it into no model; this is the wiring of the temporal model with
// deformable alignment, split so that each frame's share is computed once:
//   * encode_frame(t) stores the frame, its features f_t (NHWC, read by the
//     later convs without a transpose) and P_t, the neighbour half of the
//     offset conv (216 channels, no bias), in cache slot t;
//   * decode_window computes the centre half Q_c (with the bias) once per
//     window; the deformable conv of each neighbour reads its offsets and
//     masks as Q_c + P_t (two FP16 terms summed in FP32), and its epilogue
//     applies that neighbour's share of the 1x1 fusion conv to the 64
//     aligned channels in registers, adding it to an FP32 three-plane
//     accumulator that the centre term initialised; the last neighbour
//     writes the FP16 trunk input. Neither the 2F-channel pairs, nor the
//     T*F-channel concatenation, nor the aligned features are materialised,
//     so no layer input exceeds 2^31 elements at 2160x3840.
// The window's centre is slot T/2 of the window; edge replication = a
// repeated slot, like dn_model_decode_window.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "conv_internal.h"
#include "denoiser_b200.h"
#include "denoiser_b200_aligned.h"
#include "launch.cuh"
#include "manifest.h"
#include "status.h"

namespace dnb {
namespace {

// acc[j][pix] = b[j] + sum_f wc[j][f] * feat[pix][f] + centre[j][pix]
// (or, with out16, the FP16 value of that sum).
template <int F>
__global__ void __launch_bounds__(256) fuse_init_kernel(const __half* __restrict__ feat, const float* __restrict__ wc,
                                                        const float* __restrict__ b, const __half* __restrict__ centre,
                                                        float* __restrict__ acc, __half* __restrict__ out16,
                                                        int64_t HW, int wstride) {
    __shared__ float sw[3][F];
    for (int i = threadIdx.x; i < 3 * F; i += blockDim.x) sw[i / F][i % F] = wc[(i / F) * wstride + i % F];
    __syncthreads();
    const int64_t pix = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (pix >= HW) return;
    float s[3] = {b[0], b[1], b[2]};
    const uint4* src = reinterpret_cast<const uint4*>(feat + pix * F);
#pragma unroll
    for (int q = 0; q < F / 8; ++q) {
        const uint4 v = src[q];
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
#pragma unroll
            for (int j = 0; j < 3; ++j) s[j] = fmaf(sw[j][q * 8 + 2 * i + 1], x.y, fmaf(sw[j][q * 8 + 2 * i], x.x, s[j]));
        }
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const float v = s[j] + __half2float(centre[j * HW + pix]);
        if (out16)
            out16[j * HW + pix] = __float2half(v);
        else
            acc[j * HW + pix] = v;
    }
}

template <typename T>
void free_dev(T*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

}  // namespace
}  // namespace dnb

using namespace dnb;

struct dn_aligned {
    int device = 0;
    int T = 0, F = 0, dg = 0, cin = 3, n_om = 0, nt_dcn = 0;
    dn_conv2d* feat = nullptr;     // 3 -> F, NHWC out
    dn_conv2d* off_ctr = nullptr;  // F -> n_om, centre half + bias
    dn_conv2d* off_nbr = nullptr;  // F -> n_om, neighbour half
    dn_dcn* dcn = nullptr;         // F -> F
    dn_model* trunk = nullptr;
    float* fw = nullptr;  // device [T][3][nt_dcn]: fusion weights of frame t
    float* fb = nullptr;  // device [3]
    // Per-size buffers.
    int H = 0, W = 0;
    std::vector<__half*> frames, feats, P;  // slot buffers
    __half* xt = nullptr;                   // NHWC copy of a frame
    __half* Q = nullptr;
    float* acc = nullptr;
    __half* fused = nullptr;

    void free_buffers() {
        for (auto* v : {&frames, &feats, &P})
            for (auto*& p : *v) free_dev(p);
        free_dev(xt);
        free_dev(Q);
        free_dev(acc);
        free_dev(fused);
        H = W = 0;
    }
};

namespace {

struct DevGuardA {
    int prev = -1;
    explicit DevGuardA(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DevGuardA() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

void destroy_parts(dn_aligned* A) {
    if (A->feat) dn_conv2d_destroy(A->feat);
    if (A->off_ctr) dn_conv2d_destroy(A->off_ctr);
    if (A->off_nbr) dn_conv2d_destroy(A->off_nbr);
    if (A->dcn) dn_dcn_destroy(A->dcn);
    if (A->trunk) dn_model_destroy(A->trunk);
    free_dev(A->fw);
    free_dev(A->fb);
    A->free_buffers();
}

// Buffers for frames of H x W (reallocated, after a synchronisation, when
// the size changes; the cached slots are lost then).
int plan(dn_aligned* A, int H, int W, cudaStream_t s) {
    if (A->H == H && A->W == W) return DN_OK;
    if (H <= 0 || W <= 0) return dn_fail(DN_ERR_INVALID_ARG, "aligned temporal: empty frame");
    const int64_t HW = static_cast<int64_t>(H) * W;
    if (HW * A->n_om >= (1LL << 31) || HW * 2 * A->F >= (1LL << 31))
        return dn_fail(DN_ERR_UNSUPPORTED, "aligned temporal: frame too large (a layer output exceeds 2^31 elements)");
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return dn_cuda_fail(e, "aligned temporal: synchronise before re-plan");
    A->free_buffers();
    A->frames.assign(A->T, nullptr);
    A->feats.assign(A->T, nullptr);
    A->P.assign(A->T, nullptr);
    for (int t = 0; t < A->T && e == cudaSuccess; ++t) {
        e = cudaMalloc(&A->frames[t], HW * A->cin * 2);
        if (e == cudaSuccess) e = cudaMalloc(&A->feats[t], HW * A->F * 2);
        if (e == cudaSuccess) e = cudaMalloc(&A->P[t], HW * A->n_om * 2);
    }
    if (e == cudaSuccess) e = cudaMalloc(&A->xt, HW * A->cin * 2);
    if (e == cudaSuccess) e = cudaMalloc(&A->Q, HW * A->n_om * 2);
    if (e == cudaSuccess) e = cudaMalloc(&A->acc, HW * 3 * 4);
    if (e == cudaSuccess) e = cudaMalloc(&A->fused, HW * 3 * 2);
    if (e != cudaSuccess) {
        A->free_buffers();
        return dn_cuda_fail(e, "aligned temporal: buffers");
    }
    A->H = H;
    A->W = W;
    return DN_OK;
}

int launch_fuse_init(dn_aligned* A, int slot, const float* wc, __half* out16, cudaStream_t s) {
    const int64_t HW = static_cast<int64_t>(A->H) * A->W;
    const dim3 grid(static_cast<unsigned>((HW + 255) / 256));
    if (A->F == 64)
        fuse_init_kernel<64><<<grid, 256, 0, s>>>(A->feats[slot], wc, A->fb, A->frames[slot], A->acc, out16, HW,
                                                  A->nt_dcn);
    else if (A->F == 32)
        fuse_init_kernel<32><<<grid, 256, 0, s>>>(A->feats[slot], wc, A->fb, A->frames[slot], A->acc, out16, HW,
                                                  A->nt_dcn);
    else if (A->F == 128)
        fuse_init_kernel<128><<<grid, 256, 0, s>>>(A->feats[slot], wc, A->fb, A->frames[slot], A->acc, out16, HW,
                                                   A->nt_dcn);
    else
        return dn_fail(DN_ERR_UNSUPPORTED, "aligned temporal: feature channels must be 32, 64 or 128");
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "aligned temporal: fusion init launch");
}

}  // namespace

extern "C" {

int dn_aligned_create(const char* align_manifest, const char* trunk_manifest, int device, dn_aligned** out) {
    if (!align_manifest || !trunk_manifest || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_create: null argument");
    *out = nullptr;
    auto A = std::make_unique<dn_aligned>();
    A->device = device;
    try {
        HostWeights hw(align_manifest);
        const char* keys[] = {"align.feat.weight",   "align.feat.bias", "align.offset.weight", "align.offset.bias",
                              "align.dcn.weight",    "align.dcn.bias",  "align.fuse.weight",   "align.fuse.bias"};
        for (const char* k : keys)
            if (!hw.contains(k)) return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + k);
        const auto& sf = hw.entry("align.feat.weight").shape;
        const auto& so = hw.entry("align.offset.weight").shape;
        const auto& sd = hw.entry("align.dcn.weight").shape;
        const auto& su = hw.entry("align.fuse.weight").shape;
        if (sf.size() != 4 || so.size() != 4 || sd.size() != 4 || su.size() != 4)
            return dn_fail(DN_ERR_FORMAT, "dn_aligned_create: conv weights must be 4-D");
        A->cin = static_cast<int>(sf[1]);
        A->F = static_cast<int>(sf[0]);
        A->n_om = static_cast<int>(so[0]);
        A->T = hw.arch().num_frames;
        if (A->cin != 3) return dn_fail(DN_ERR_UNSUPPORTED, "dn_aligned_create: 3-channel frames only");
        if (A->F != 32 && A->F != 64 && A->F != 128)
            return dn_fail(DN_ERR_UNSUPPORTED, "dn_aligned_create: feature channels must be 32, 64 or 128");
        if (A->n_om % 27 != 0 || so[1] != 2 * A->F || sf[2] != 3 || sf[3] != 3 || so[2] != 3 || so[3] != 3 ||
            sd[0] != A->F || sd[1] != A->F || su[0] != 3 || su[1] != static_cast<int64_t>(A->T) * A->F || su[2] != 1 ||
            su[3] != 1 || A->T < 1)
            return dn_fail(DN_ERR_FORMAT, "dn_aligned_create: inconsistent alignment weight shapes");
        A->dg = A->n_om / 27;
        const auto wf = hw.to_f32("align.feat.weight"), bf = hw.to_f32("align.feat.bias");
        const auto wo = hw.to_f32("align.offset.weight"), bo = hw.to_f32("align.offset.bias");
        const auto wd = hw.to_f32("align.dcn.weight"), bd = hw.to_f32("align.dcn.bias");
        const auto wu = hw.to_f32("align.fuse.weight"), bu = hw.to_f32("align.fuse.bias");
        // The offset conv's input channels split into the centre half and the neighbour half.
        const int F = A->F, KK = 9;
        std::vector<float> wctr(static_cast<size_t>(A->n_om) * F * KK), wnbr(wctr.size());
        for (int o = 0; o < A->n_om; ++o)
            for (int c = 0; c < F; ++c)
                for (int k = 0; k < KK; ++k) {
                    wctr[(static_cast<size_t>(o) * F + c) * KK + k] = wo[(static_cast<size_t>(o) * 2 * F + c) * KK + k];
                    wnbr[(static_cast<size_t>(o) * F + c) * KK + k] =
                        wo[(static_cast<size_t>(o) * 2 * F + F + c) * KK + k];
                }
        DN_TRY(conv2d_build(wf.data(), bf.data(), F, 3, 3, 3, 1, 1, 1, 1, device, &A->feat));
        int rc = conv2d_build(wctr.data(), bo.data(), A->n_om, F, 3, 3, 1, 1, 1, 1, device, &A->off_ctr);
        if (rc == DN_OK) rc = conv2d_build(wnbr.data(), nullptr, A->n_om, F, 3, 3, 1, 1, 1, 1, device, &A->off_nbr);
        if (rc == DN_OK) rc = dcn_build(wd.data(), bd.data(), F, F, 3, 3, 1, 1, 1, A->dg, device, &A->dcn);
        if (rc != DN_OK) {
            destroy_parts(A.get());
            return rc;
        }
        A->nt_dcn = dcn_nt(A->dcn);
        // Fusion weights per frame, rounded to FP16 like every exported weight.
        std::vector<float> fw(static_cast<size_t>(A->T) * 3 * A->nt_dcn, 0.f), fb(3);
        for (int t = 0; t < A->T; ++t)
            for (int j = 0; j < 3; ++j)
                for (int c = 0; c < F; ++c)
                    fw[(static_cast<size_t>(t) * 3 + j) * A->nt_dcn + c] =
                        __half2float(__float2half(wu[static_cast<size_t>(j) * A->T * F + t * F + c]));
        for (int j = 0; j < 3; ++j) fb[j] = __half2float(__float2half(bu[j]));
        DevGuardA g(device);
        cudaError_t e = cudaMalloc(&A->fw, fw.size() * 4);
        if (e == cudaSuccess) e = cudaMalloc(&A->fb, 3 * 4);
        if (e == cudaSuccess) e = cudaMemcpy(A->fw, fw.data(), fw.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(A->fb, fb.data(), 3 * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            destroy_parts(A.get());
            return dn_cuda_fail(e, "dn_aligned_create: upload");
        }
    } catch (const IoError& ex) {
        destroy_parts(A.get());
        return dn_fail_str(DN_ERR_IO, ex.what());
    } catch (const NotFoundError& ex) {
        destroy_parts(A.get());
        return dn_fail_str(DN_ERR_NOT_FOUND, ex.what());
    } catch (const std::exception& ex) {
        destroy_parts(A.get());
        return dn_fail_str(DN_ERR_FORMAT, ex.what());
    }
    int rc = dn_model_create(trunk_manifest, device, &A->trunk);
    if (rc == DN_OK) {
        dn_model_info info{};
        rc = dn_model_get_info(A->trunk, &info);
        if (rc == DN_OK && (info.kind != 0 || info.in_channels != 3))
            rc = dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_create: the trunk must be a 3-channel spatial NAFNet");
    }
    if (rc != DN_OK) {
        destroy_parts(A.get());
        return rc;
    }
    *out = A.release();
    return DN_OK;
}

int dn_aligned_destroy(dn_aligned* A) {
    if (!A) return DN_OK;
    DevGuardA g(A->device);
    destroy_parts(A);
    delete A;
    return DN_OK;
}

int dn_aligned_info(const dn_aligned* A, int* num_frames, int* in_channels, int* feat_channels, int* deform_groups) {
    if (!A) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_info: null model");
    if (num_frames) *num_frames = A->T;
    if (in_channels) *in_channels = A->cin;
    if (feat_channels) *feat_channels = A->F;
    if (deform_groups) *deform_groups = A->dg;
    return DN_OK;
}

int dn_aligned_encode_frame(dn_aligned* A, const void* frame, int H, int W, int slot, void* stream) {
    if (!A || !frame) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_encode_frame: null argument");
    if (slot < 0 || slot >= A->T) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_encode_frame: slot outside [0, T)");
    DevGuardA g(A->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DN_TRY(plan(A, H, W, s));
    const int64_t HW = static_cast<int64_t>(H) * W;
    cudaError_t e = cudaMemcpyAsync(A->frames[slot], frame, HW * A->cin * 2, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return dn_cuda_fail(e, "dn_aligned_encode_frame: frame copy");
    DN_TRY(conv2d_to_nhwc(static_cast<const __half*>(frame), A->xt, 1, A->cin, static_cast<int>(HW), s));
    DN_TRY(conv2d_run_nhwc(A->feat, A->xt, 1, H, W, A->feats[slot], true, s));
    return conv2d_run_nhwc(A->off_nbr, A->feats[slot], 1, H, W, A->P[slot], false, s);
}

int dn_aligned_align_window(dn_aligned* A, const int* slots, int T, void* fused, void* stream) {
    if (!A || !slots || !fused) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_align_window: null argument");
    if (T != A->T) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_align_window: window length != num_frames");
    for (int t = 0; t < T; ++t)
        if (slots[t] < 0 || slots[t] >= A->T)
            return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_align_window: slot outside [0, T)");
    if (A->H == 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_align_window: no frame encoded");
    DevGuardA g(A->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int c = T / 2, sc = slots[c];
    const int64_t HW = static_cast<int64_t>(A->H) * A->W;
    auto* out16 = static_cast<__half*>(fused);
    const size_t wstride = static_cast<size_t>(3) * A->nt_dcn;
    DN_TRY(launch_fuse_init(A, sc, A->fw + c * wstride, T == 1 ? out16 : nullptr, s));
    if (T == 1) return DN_OK;
    DN_TRY(conv2d_run_nhwc(A->off_ctr, A->feats[sc], 1, A->H, A->W, A->Q, false, s));
    const int64_t moff = static_cast<int64_t>(2) * A->dg * 9 * HW;  // first mask plane
    const int last = (c == T - 1) ? T - 2 : T - 1;
    for (int t = 0; t < T; ++t) {
        if (t == c) continue;
        const int st = slots[t];
        DcnFuse fz{A->fw + t * wstride, A->acc, t == last ? out16 : nullptr};
        DN_TRY(dcn_run_nhwc(A->dcn, A->feats[st], A->Q, A->Q + moff, A->P[st], A->P[st] + moff, 1, A->H, A->W, nullptr,
                            &fz, s));
    }
    return DN_OK;
}

int dn_aligned_decode_window(dn_aligned* A, const int* slots, int T, void* y, void* stream) {
    if (!A || !y) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_decode_window: null argument");
    DN_TRY(dn_aligned_align_window(A, slots, T, A->fused, stream));
    const int64_t shape[4] = {1, 3, A->H, A->W};
    return dn_model_forward(A->trunk, A->fused, shape, 4, y, stream);
}

int dn_aligned_forward(dn_aligned* A, const void* clip, int H, int W, void* y, void* stream) {
    if (!A || !clip || !y) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_forward: null argument");
    const int64_t frame = static_cast<int64_t>(A->cin) * H * W;
    std::vector<int> slots(A->T);
    for (int t = 0; t < A->T; ++t) {
        DN_TRY(dn_aligned_encode_frame(A, static_cast<const __half*>(clip) + t * frame, H, W, t, stream));
        slots[t] = t;
    }
    return dn_aligned_decode_window(A, slots.data(), A->T, y, stream);
}

int dn_aligned_sync(dn_aligned* A, void* stream) {
    if (!A) return dn_fail(DN_ERR_INVALID_ARG, "dn_aligned_sync: null model");
    DevGuardA g(A->device);
    DN_TRY(dn_model_sync(A->trunk, stream));
    DN_TRY(conv2d_check(A->feat));
    DN_TRY(conv2d_check(A->off_ctr));
    DN_TRY(conv2d_check(A->off_nbr));
    return dcn_check(A->dcn);
}

}  // extern "C"
