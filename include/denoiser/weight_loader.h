// denoiser::WeightStore — source-compatible with the reference's
// include/denoiser/weight_loader.h:61-101, over the C-ABI store
// (dn_weights_*): the manifest is parsed and every .bin memory-mapped and
// size-checked at construction; get() uploads a tensor to the current
// device on first use and caches it (behind a mutex, as the reference does).
// Exceptions: std::runtime_error for a missing or malformed manifest/.bin,
// std::out_of_range for a missing key.
#pragma once

#include <cstdint>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "denoiser/detail/abi.h"
#include "denoiser/tensor.h"
#include "denoiser_b200.h"

namespace denoiser {

struct LayerEntry {
    std::string name;
    std::vector<int64_t> shape;
    DType dtype;
    std::string file;
};

struct Manifest {
    std::string version;
    DType dtype;
    std::vector<LayerEntry> layers;
    struct Architecture {
        std::string type;
        std::vector<int> enc_channels;
        int num_levels = 0;
        int base_channels = 32;
        int in_channels = 3;
        int out_channels = 3;
        int num_frames = 3;
        bool use_warp = false;
    } architecture;
};

class WeightStore {
public:
    explicit WeightStore(const std::string& manifest_path) {
        const int rc = dn_weights_open(manifest_path.c_str(), &h_);
        if (rc != DN_OK) {
            const std::string msg = dn_last_error();
            if (rc == DN_ERR_NOT_FOUND) throw std::out_of_range(msg);
            throw std::runtime_error(msg);
        }
        try {
            load_manifest();
        } catch (...) {
            dn_weights_close(h_);
            throw;
        }
    }
    ~WeightStore() { dn_weights_close(h_); }
    WeightStore(const WeightStore&) = delete;
    WeightStore& operator=(const WeightStore&) = delete;

    // Device tensor of `name` (uploaded on first use, then cached).
    const Tensor& get(const std::string& name) const {
        std::lock_guard<std::mutex> lock(mu_);
        auto it = cache_.find(name);
        if (it != cache_.end()) return it->second;
        int64_t shape[8];
        int ndim = 0, dt = 0;
        const void* host = nullptr;
        detail::check(dn_weights_info(h_, name.c_str(), shape, &ndim, &dt, &host));
        std::vector<int64_t> s(shape, shape + ndim);
        if (s.empty()) s.push_back(1);
        const DType dtype = dt == 1 ? DType::kFloat16 : DType::kFloat32;
        return cache_.emplace(name, Tensor::from_host(host, s, dtype)).first->second;
    }
    bool contains(const std::string& name) const { return dn_weights_contains(h_, name.c_str()) == 1; }
    const Manifest& manifest() const noexcept { return manifest_; }
    void prefetch_all(cudaStream_t /*stream*/ = nullptr) const {
        for (const auto& l : manifest_.layers) get(l.name);
    }
    size_t device_bytes_allocated() const {
        std::lock_guard<std::mutex> lock(mu_);
        size_t n = 0;
        for (const auto& kv : cache_) n += kv.second.nbytes();
        return n;
    }

    // Path of manifest.json (the models build their engine from it).
    std::string manifest_path() const { return dn_weights_path(h_); }
    // The C-ABI handle, for the layers built from this store.
    const dn_weights* handle() const noexcept { return h_; }

private:
    dn_weights* h_ = nullptr;
    Manifest manifest_;
    mutable std::mutex mu_;
    mutable std::unordered_map<std::string, Tensor> cache_;

    void load_manifest() {
        const char* version = "";
        int dt = 1, enc[16] = {0}, n_enc = 0, out_ch = 3;
        detail::check(dn_weights_meta(h_, &version, &dt, enc, 16, &n_enc, &out_ch));
        manifest_.version = version;
        manifest_.dtype = dt == 1 ? DType::kFloat16 : DType::kFloat32;
        char type[64] = {0};
        int base = 0, levels = 0, in_ch = 0, frames = 0, warp = 0;
        detail::check(dn_weights_arch(h_, type, sizeof(type), &base, &levels, &in_ch, &frames, &warp));
        auto& a = manifest_.architecture;
        a.type = type;
        a.enc_channels.assign(enc, enc + (n_enc < 16 ? n_enc : 16));
        a.num_levels = levels;
        a.base_channels = base;
        a.in_channels = in_ch;
        a.out_channels = out_ch;
        a.num_frames = frames;
        a.use_warp = warp != 0;
        const int n = dn_weights_count(h_);
        for (int i = 0; i < n; ++i) {
            const char* name = nullptr;
            detail::check(dn_weights_name(h_, i, &name));
            int64_t shape[8];
            int ndim = 0, ldt = 0;
            const void* host = nullptr;
            detail::check(dn_weights_info(h_, name, shape, &ndim, &ldt, &host));
            const char* file = "";
            detail::check(dn_weights_file(h_, name, &file));
            manifest_.layers.push_back(
                {name, std::vector<int64_t>(shape, shape + ndim), ldt == 1 ? DType::kFloat16 : DType::kFloat32, file});
        }
    }
};

}  // namespace denoiser
