// C-ABI of the model engine: the drop-in boundary behind NAFNet::forward /
// NAFNetTemporal::forward (include/denoiser/models/nafnet.h:11-28,
// nafnet_temporal.h:11-29 of the reference) and the CLI's per-frame loop.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <new>
#include <string>

#include "engine.h"
#include "status.h"

using namespace dnb;

struct dn_model {
    std::unique_ptr<Engine> eng;
    // Device staging for the host-buffer entry point.
    void* dx = nullptr;
    void* dy = nullptr;
    size_t dx_bytes = 0, dy_bytes = 0;
    // Pipelined host-buffer calls: two staging pairs, one stream per copy
    // direction, and the events that order copies and forwards.
    struct Pipe {
        void* dx[2] = {nullptr, nullptr};
        void* dy[2] = {nullptr, nullptr};
        size_t dx_bytes = 0, dy_bytes = 0;
        cudaStream_t h2d = nullptr, d2h = nullptr;
        cudaEvent_t in_ready[2] = {}, in_free[2] = {}, out_ready[2] = {}, out_free[2] = {};
        unsigned count = 0;  // calls issued
        bool init = false;
    } pipe;
};

namespace {

template <class F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const NotFoundError& e) {
        return dn_fail(DN_ERR_NOT_FOUND, e.what());
    } catch (const IoError& e) {
        return dn_fail(DN_ERR_IO, e.what());
    } catch (const FormatError& e) {
        return dn_fail(DN_ERR_FORMAT, e.what());
    } catch (const std::bad_alloc&) {
        return dn_fail(DN_ERR_CUDA, "host out of memory");
    } catch (const std::exception& e) {
        return dn_fail(DN_ERR_CUDA, e.what());
    } catch (...) {
        return dn_fail(DN_ERR_CUDA, "unknown error");
    }
}

// Parses (N,C,H,W) or (N,T,C,H,W) for the model kind.
int parse_shape(const Engine& e, const int64_t* shape, int ndim, int& N, int& T, int& C, int& H, int& W) {
    if (!shape) return dn_fail(DN_ERR_INVALID_ARG, "forward: null shape");
    const bool temporal = e.info().kind != 0;
    if (temporal && ndim != 5) return dn_fail(DN_ERR_INVALID_ARG, "NAFNetTemporal::forward: expected 5-D (N,T,C,H,W) clip");
    if (!temporal && ndim != 4) return dn_fail(DN_ERR_INVALID_ARG, "NAFNet::forward: expected 4-D NCHW input");
    for (int i = 0; i < ndim; ++i)
        if (shape[i] <= 0 || shape[i] > (1 << 20)) return dn_fail(DN_ERR_INVALID_ARG, "forward: bad dimension");
    N = static_cast<int>(shape[0]);
    T = temporal ? static_cast<int>(shape[1]) : 1;
    C = static_cast<int>(shape[temporal ? 2 : 1]);
    H = static_cast<int>(shape[temporal ? 3 : 2]);
    W = static_cast<int>(shape[temporal ? 4 : 3]);
    return DN_OK;
}

}  // namespace

extern "C" {

int dn_model_create(const char* manifest_path, int device, dn_model** out) {
    if (!manifest_path || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_create: null argument");
    *out = nullptr;
    return guarded([&] {
        int count = 0;
        cudaError_t e = cudaGetDeviceCount(&count);
        if (e != cudaSuccess) return dn_cuda_fail(e, "cudaGetDeviceCount");
        if (device < 0 || device >= count)
            return dn_fail_str(DN_ERR_INVALID_ARG, "CUDA device " + std::to_string(device) + " not available (" +
                                                       std::to_string(count) + " devices found)");
        auto m = std::make_unique<dn_model>();
        m->eng = std::make_unique<Engine>(manifest_path, device);
        *out = m.release();
        return DN_OK;
    });
}

int dn_model_destroy(dn_model* m) {
    if (!m) return DN_OK;
    return guarded([&] {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(m->eng->device());
        if (m->dx) cudaFree(m->dx);
        if (m->dy) cudaFree(m->dy);
        auto& q = m->pipe;
        if (q.init) {
            cudaStreamSynchronize(q.h2d);
            cudaStreamSynchronize(q.d2h);
            for (int k = 0; k < 2; ++k) {
                if (q.dx[k]) cudaFree(q.dx[k]);
                if (q.dy[k]) cudaFree(q.dy[k]);
                for (cudaEvent_t ev : {q.in_ready[k], q.in_free[k], q.out_ready[k], q.out_free[k]})
                    cudaEventDestroy(ev);
            }
            cudaStreamDestroy(q.h2d);
            cudaStreamDestroy(q.d2h);
        }
        cudaSetDevice(prev);
        delete m;
        return DN_OK;
    });
}

int dn_model_get_info(const dn_model* m, dn_model_info* info) {
    if (!m || !info) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_get_info: null argument");
    const ModelInfo& i = m->eng->info();
    info->kind = i.kind;
    info->in_channels = i.in_channels;
    info->num_levels = i.num_levels;
    info->base_channels = i.base_channels;
    info->num_frames = i.num_frames;
    info->use_warp = i.use_warp;
    for (int l = 0; l < 8; ++l)
        info->enc_channels[l] = l < static_cast<int>(i.enc_channels.size()) ? i.enc_channels[l] : 0;
    return DN_OK;
}

int dn_model_forward(dn_model* m, const void* x, const int64_t* shape, int ndim, void* y, void* stream) {
    if (!m || !x || !y) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_forward: null argument");
    return guarded([&] {
        int N, T, C, H, W;
        const int rc = parse_shape(*m->eng, shape, ndim, N, T, C, H, W);
        if (rc != DN_OK) return rc;
        return m->eng->forward(static_cast<const __half*>(x), N, T, C, H, W, static_cast<__half*>(y),
                               static_cast<cudaStream_t>(stream));
    });
}

int dn_model_encode_frame(dn_model* m, const void* frame, int C, int H, int W, int slot, void* stream) {
    if (!m || !frame) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_encode_frame: null argument");
    return guarded([&] {
        return m->eng->encode_frame(static_cast<const __half*>(frame), C, H, W, slot, static_cast<cudaStream_t>(stream));
    });
}

int dn_model_decode_window(dn_model* m, const int* slots, int T, const void* beauty, int C, int H, int W, void* y,
                           void* stream) {
    if (!m || !slots || !beauty || !y) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_decode_window: null argument");
    if (T != m->eng->info().num_frames)
        return dn_fail(DN_ERR_INVALID_ARG, "dn_model_decode_window: T differs from the model's num_frames");
    return guarded([&] {
        return m->eng->decode_window(slots, static_cast<const __half*>(beauty), C, H, W, static_cast<__half*>(y),
                                     static_cast<cudaStream_t>(stream));
    });
}

int dn_model_forward_host(dn_model* m, const void* x_host, const int64_t* shape, int ndim, void* y_host,
                          void* stream) {
    if (!m || !x_host || !y_host) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_forward_host: null argument");
    return guarded([&] {
        int N, T, C, H, W;
        int rc = parse_shape(*m->eng, shape, ndim, N, T, C, H, W);
        if (rc != DN_OK) return rc;
        const size_t xb = static_cast<size_t>(N) * T * C * H * W * 2;
        const size_t yb = static_cast<size_t>(N) * 3 * H * W * 2;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(m->eng->device());
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaError_t e = cudaSuccess;
        if (m->dx_bytes < xb) {
            if (m->dx) cudaFree(m->dx);
            m->dx = nullptr;
            e = cudaMalloc(&m->dx, xb);
            m->dx_bytes = e == cudaSuccess ? xb : 0;
        }
        if (e == cudaSuccess && m->dy_bytes < yb) {
            if (m->dy) cudaFree(m->dy);
            m->dy = nullptr;
            e = cudaMalloc(&m->dy, yb);
            m->dy_bytes = e == cudaSuccess ? yb : 0;
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(m->dx, x_host, xb, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) {
            cudaSetDevice(prev);
            return dn_cuda_fail(e, "dn_model_forward_host: staging");
        }
        rc = m->eng->forward(static_cast<const __half*>(m->dx), N, T, C, H, W, static_cast<__half*>(m->dy), s);
        if (rc == DN_OK) {
            e = cudaMemcpyAsync(y_host, m->dy, yb, cudaMemcpyDeviceToHost, s);
            if (e != cudaSuccess) rc = dn_cuda_fail(e, "dn_model_forward_host: copy back");
        }
        if (rc == DN_OK) rc = m->eng->check_device(s);
        cudaSetDevice(prev);
        return rc;
    });
}

int dn_model_forward_host_async(dn_model* m, const void* x_host, const int64_t* shape, int ndim, void* y_host,
                                void* stream) {
    if (!m || !x_host || !y_host) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_forward_host_async: null argument");
    return guarded([&] {
        int N, T, C, H, W;
        int rc = parse_shape(*m->eng, shape, ndim, N, T, C, H, W);
        if (rc != DN_OK) return rc;
        const size_t xb = static_cast<size_t>(N) * T * C * H * W * 2;
        const size_t yb = static_cast<size_t>(N) * 3 * H * W * 2;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(m->eng->device());
        struct Restore {
            int d;
            ~Restore() { cudaSetDevice(d); }
        } restore{prev};
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        auto& q = m->pipe;
        cudaError_t e = cudaSuccess;
        if (!q.init) {
            e = cudaStreamCreateWithFlags(&q.h2d, cudaStreamNonBlocking);
            if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&q.d2h, cudaStreamNonBlocking);
            for (int k = 0; k < 2 && e == cudaSuccess; ++k)
                for (cudaEvent_t* ev : {&q.in_ready[k], &q.in_free[k], &q.out_ready[k], &q.out_free[k]})
                    if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
            if (e != cudaSuccess) return dn_cuda_fail(e, "dn_model_forward_host_async: set-up");
            q.init = true;
        }
        if (q.dx_bytes < xb || q.dy_bytes < yb) {
            // Larger frames: let every queued call finish before the staging grows.
            cudaStreamSynchronize(q.h2d);
            cudaStreamSynchronize(q.d2h);
            cudaStreamSynchronize(s);
            for (int k = 0; k < 2 && e == cudaSuccess; ++k) {
                if (q.dx_bytes < xb) {
                    if (q.dx[k]) cudaFree(q.dx[k]);
                    q.dx[k] = nullptr;
                    e = cudaMalloc(&q.dx[k], xb);
                }
                if (e == cudaSuccess && q.dy_bytes < yb) {
                    if (q.dy[k]) cudaFree(q.dy[k]);
                    q.dy[k] = nullptr;
                    e = cudaMalloc(&q.dy[k], yb);
                }
            }
            if (e != cudaSuccess) {
                q.dx_bytes = q.dy_bytes = 0;
                return dn_cuda_fail(e, "dn_model_forward_host_async: staging");
            }
            q.dx_bytes = std::max(q.dx_bytes, xb);
            q.dy_bytes = std::max(q.dy_bytes, yb);
        }
        const int k = static_cast<int>(q.count & 1u);
        const bool reuse = q.count >= 2;  // staging pair k was used two calls ago
        // Input copy: once the forward two calls back has read this staging
        // buffer. It does not wait for the work already queued on the
        // caller's stream (the previous call's forward): that is what lets
        // it overlap that forward. The host data is ready at the call.
        if (reuse) e = cudaStreamWaitEvent(q.h2d, q.in_free[k], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(q.dx[k], x_host, xb, cudaMemcpyHostToDevice, q.h2d);
        if (e == cudaSuccess) e = cudaEventRecord(q.in_ready[k], q.h2d);
        // Forward on the caller's stream, once the input has landed and the
        // output copy two calls back has read this output buffer.
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, q.in_ready[k], 0);
        if (e == cudaSuccess && reuse) e = cudaStreamWaitEvent(s, q.out_free[k], 0);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dn_model_forward_host_async: input copy");
        rc = m->eng->forward(static_cast<const __half*>(q.dx[k]), N, T, C, H, W, static_cast<__half*>(q.dy[k]), s);
        if (rc != DN_OK) return rc;
        e = cudaEventRecord(q.in_free[k], s);
        if (e == cudaSuccess) e = cudaEventRecord(q.out_ready[k], s);
        // Output copy on its own stream: it overlaps the next call's forward.
        if (e == cudaSuccess) e = cudaStreamWaitEvent(q.d2h, q.out_ready[k], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(y_host, q.dy[k], yb, cudaMemcpyDeviceToHost, q.d2h);
        if (e == cudaSuccess) e = cudaEventRecord(q.out_free[k], q.d2h);
        if (e != cudaSuccess) return dn_cuda_fail(e, "dn_model_forward_host_async: output copy");
        ++q.count;
        return DN_OK;
    });
}

int dn_model_host_join(dn_model* m, void* stream) {
    if (!m) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_host_join: null model");
    return guarded([&] {
        auto& q = m->pipe;
        if (!q.init || q.count == 0) return DN_OK;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(m->eng->device());
        // Output copies run in call order on one stream: the last one's event
        // covers every queued call.
        cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), q.out_free[(q.count - 1) & 1u], 0);
        cudaSetDevice(prev);
        return e == cudaSuccess ? DN_OK : dn_cuda_fail(e, "dn_model_host_join");
    });
}

int dn_model_sync(dn_model* m, void* stream) {
    if (!m) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_sync: null model");
    return guarded([&] { return m->eng->check_device(static_cast<cudaStream_t>(stream)); });
}

int dn_model_stats(const dn_model* m, size_t* weight_bytes, size_t* activation_bytes, int* kernels_per_forward) {
    if (!m) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_stats: null model");
    if (weight_bytes) *weight_bytes = m->eng->weight_bytes();
    if (activation_bytes) *activation_bytes = m->eng->activation_bytes();
    if (kernels_per_forward) *kernels_per_forward = m->eng->kernels_per_forward();
    return DN_OK;
}

int dn_model_set_fused(dn_model* m, int enable) {
    if (!m) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_set_fused: null model");
    if (enable < 0 || enable > 4) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_set_fused: mode must be 0 to 4");
    m->eng->set_fused(enable);
    return DN_OK;
}

int dn_model_profile(dn_model* m, int enable) {
    if (!m) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_profile: null model");
    if (enable < 0 || enable > 2) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_profile: enable must be 0, 1 or 2");
    m->eng->set_profiling(enable);
    return DN_OK;
}

int dn_model_profile_report(dn_model* m, char* buf, size_t len) {
    if (!m || !buf || len == 0) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_profile_report: bad argument");
    return guarded([&] {
        const std::string r = m->eng->profile_report();
        if (r.size() + 1 > len) return dn_fail(DN_ERR_INVALID_ARG, "dn_model_profile_report: buffer too small");
        std::memcpy(buf, r.c_str(), r.size() + 1);
        return DN_OK;
    });
}

}  // extern "C"
