// denoiser::Tensor — device-resident NCHW tensor, source-compatible with the
// reference's include/denoiser/tensor.h:43-138 (same names, ownership and
// exceptions). Header-only; needs the CUDA runtime. The cuDNN helpers
// (to_cudnn_dtype, make_cudnn_descriptor, CUDNN_CHECK) exist only when
// DENOISER_WITH_CUDNN is defined: this library itself uses no cuDNN.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#ifdef DENOISER_WITH_CUDNN
#include <cudnn.h>
#endif

namespace denoiser {

enum class DType : uint8_t { kFloat32, kFloat16 };

constexpr size_t dtype_size(DType dtype) noexcept { return dtype == DType::kFloat16 ? sizeof(__half) : sizeof(float); }

[[nodiscard]] inline std::string cuda_error_string(cudaError_t err) {
    return std::string("CUDA error: ") + cudaGetErrorString(err);
}

inline void check_cuda(cudaError_t err, const char* file, int line) {
    if (err != cudaSuccess) throw std::runtime_error(std::string(file) + ":" + std::to_string(line) + " " + cuda_error_string(err));
}

#define CUDA_CHECK(expr) denoiser::check_cuda((expr), __FILE__, __LINE__)

#ifdef DENOISER_WITH_CUDNN
constexpr cudnnDataType_t to_cudnn_dtype(DType dtype) noexcept {
    return dtype == DType::kFloat16 ? CUDNN_DATA_HALF : CUDNN_DATA_FLOAT;
}
inline void check_cudnn(cudnnStatus_t status, const char* file, int line) {
    if (status != CUDNN_STATUS_SUCCESS)
        throw std::runtime_error(std::string(file) + ":" + std::to_string(line) + " cuDNN error: " +
                                 cudnnGetErrorString(status));
}
#define CUDNN_CHECK(expr) denoiser::check_cudnn((expr), __FILE__, __LINE__)
#endif

class Tensor {
public:
    Tensor() = default;

    // Uninitialised device tensor; every dimension must be > 0.
    //
    // Unlike the reference (cudaMalloc per tensor, cudaFree in the destructor,
    // src/tensor.cu:13-23, 66-71, which blocks the host and synchronises the
    // whole device on every free), memory comes from the device's
    // stream-ordered pool: cudaMallocAsync on `stream`, and the destructor
    // returns it with cudaFreeAsync on the legacy default stream. That free
    // is ordered after the work already queued on every blocking stream
    // (streams from cudaStreamCreate, the reference CLI's kind) and needs no
    // stream to outlive the tensor, so the reference's lifetime rules hold;
    // work on a stream created with cudaStreamNonBlocking that still reads a
    // tensor must be synchronised before the tensor is destroyed.
    static Tensor empty(std::vector<int64_t> shape, DType dtype, cudaStream_t stream = nullptr) {
        int64_t n = 1;
        for (int64_t d : shape) {
            if (d <= 0) throw std::invalid_argument("Tensor::empty: all dimensions must be > 0");
            n *= d;
        }
        void* p = nullptr;
        CUDA_CHECK(cudaMallocAsync(&p, static_cast<size_t>(n) * dtype_size(dtype), stream));
        return Tensor(p, std::move(shape), dtype, true);
    }

    // Device copy of host data; synchronous when stream == nullptr.
    static Tensor from_host(const void* data, std::vector<int64_t> shape, DType dtype, cudaStream_t stream = nullptr) {
        if (!data) throw std::invalid_argument("Tensor::from_host: data must not be null");
        Tensor t = empty(std::move(shape), dtype, stream);
        t.copy(t.d_ptr_, data, cudaMemcpyHostToDevice, stream);
        return t;
    }

    Tensor(Tensor&& o) noexcept
        : d_ptr_(o.d_ptr_), shape_(std::move(o.shape_)), dtype_(o.dtype_), owns_memory_(o.owns_memory_) {
        o.d_ptr_ = nullptr;
        o.owns_memory_ = false;
    }
    Tensor& operator=(Tensor&& o) noexcept {
        if (this != &o) {
            release();
            d_ptr_ = o.d_ptr_;
            shape_ = std::move(o.shape_);
            dtype_ = o.dtype_;
            owns_memory_ = o.owns_memory_;
            o.d_ptr_ = nullptr;
            o.owns_memory_ = false;
        }
        return *this;
    }
    Tensor(const Tensor&) = delete;
    Tensor& operator=(const Tensor&) = delete;
    ~Tensor() { release(); }

    Tensor clone(cudaStream_t stream = nullptr) const {
        if (!is_valid()) return Tensor{};
        Tensor t = empty(shape_, dtype_, stream);
        copy(t.d_ptr_, d_ptr_, cudaMemcpyDeviceToDevice, stream);
        return t;
    }

    void to_host(void* out, cudaStream_t stream = nullptr) const {
        if (!is_valid()) throw std::runtime_error("Tensor::to_host: tensor is empty");
        if (!out) throw std::invalid_argument("Tensor::to_host: output pointer must not be null");
        copy(out, d_ptr_, cudaMemcpyDeviceToHost, stream);
    }

    const std::vector<int64_t>& shape() const noexcept { return shape_; }
    DType dtype() const noexcept { return dtype_; }
    void* data() noexcept { return d_ptr_; }
    const void* data() const noexcept { return d_ptr_; }
    float* data_f32() noexcept { return static_cast<float*>(d_ptr_); }
    const float* data_f32() const noexcept { return static_cast<const float*>(d_ptr_); }
    __half* data_f16() noexcept { return static_cast<__half*>(d_ptr_); }
    const __half* data_f16() const noexcept { return static_cast<const __half*>(d_ptr_); }
    bool is_valid() const noexcept { return d_ptr_ != nullptr; }
    int64_t numel() const noexcept {
        if (shape_.empty()) return 0;
        int64_t n = 1;
        for (int64_t d : shape_) n *= d;
        return n;
    }
    size_t nbytes() const noexcept { return static_cast<size_t>(numel()) * dtype_size(dtype_); }
    int64_t batch() const { return dim(0); }
    int64_t channels() const { return dim(1); }
    int64_t height() const { return dim(2); }
    int64_t width() const { return dim(3); }

    // Non-owning view of channels [start, end) (the reference's rule: the
    // view starts start*H*W elements in, so it addresses image 0's channels).
    Tensor slice_channels(int64_t start, int64_t end) const {
        if (shape_.size() != 4) throw std::runtime_error("slice_channels requires a 4-D (NCHW) tensor");
        const int64_t C = shape_[1];
        if (start < 0 || end > C || start >= end)
            throw std::out_of_range("slice_channels: invalid range [" + std::to_string(start) + ", " +
                                    std::to_string(end) + ") for C=" + std::to_string(C));
        auto* p = static_cast<uint8_t*>(d_ptr_) + static_cast<size_t>(start * shape_[2] * shape_[3]) * dtype_size(dtype_);
        return Tensor(p, {shape_[0], end - start, shape_[2], shape_[3]}, dtype_, false);
    }

#ifdef DENOISER_WITH_CUDNN
    cudnnTensorDescriptor_t make_cudnn_descriptor() const {
        if (shape_.size() != 4) throw std::runtime_error("make_cudnn_descriptor requires a 4-D (NCHW) tensor");
        cudnnTensorDescriptor_t d;
        CUDNN_CHECK(cudnnCreateTensorDescriptor(&d));
        CUDNN_CHECK(cudnnSetTensor4dDescriptor(d, CUDNN_TENSOR_NCHW, to_cudnn_dtype(dtype_), static_cast<int>(shape_[0]),
                                               static_cast<int>(shape_[1]), static_cast<int>(shape_[2]),
                                               static_cast<int>(shape_[3])));
        return d;
    }
#endif

    std::string shape_str() const {
        std::ostringstream o;
        o << "(";
        for (size_t i = 0; i < shape_.size(); ++i) o << shape_[i] << (i + 1 < shape_.size() ? ", " : "");
        o << ")";
        return o.str();
    }

private:
    void* d_ptr_ = nullptr;
    std::vector<int64_t> shape_;
    DType dtype_ = DType::kFloat32;
    bool owns_memory_ = true;

    Tensor(void* p, std::vector<int64_t> shape, DType dtype, bool owns) noexcept
        : d_ptr_(p), shape_(std::move(shape)), dtype_(dtype), owns_memory_(owns) {}

    void release() noexcept {
        if (owns_memory_ && d_ptr_) cudaFreeAsync(d_ptr_, nullptr);  // a destructor must not throw
        d_ptr_ = nullptr;
    }
    void copy(void* dst, const void* src, cudaMemcpyKind kind, cudaStream_t stream) const {
        if (stream)
            CUDA_CHECK(cudaMemcpyAsync(dst, src, nbytes(), kind, stream));
        else
            CUDA_CHECK(cudaMemcpy(dst, src, nbytes(), kind));
    }
    int64_t dim(int i) const {
        if (shape_.size() != 4)
            throw std::runtime_error("Tensor: NCHW dimension accessor requires ndim==4, got " + std::to_string(shape_.size()));
        return shape_[static_cast<size_t>(i)];
    }
};

}  // namespace denoiser
