// Host side of the weight format of the reference project:
// manifest.json (version, dtype, architecture, layers[{name, shape, dtype,
// file}]) + raw little-endian C-contiguous .bin files
// (training/export.py:48-118, src/weight_loader.cc:63-129).
//
// Files are memory-mapped read-only like the reference WeightStore
// (weight_loader.cc:29-58), and, unlike it, every .bin is checked against
// numel(shape) * sizeof(dtype) so a truncated export fails at load time.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace dnb {

// Reference exception semantics: runtime_error for missing/bad files,
// out_of_range for a missing key (tests/test_weight_loader.cc:115-153).
struct IoError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct FormatError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct NotFoundError : std::out_of_range {
    using std::out_of_range::out_of_range;
};

enum class WDType : int { F32 = 0, F16 = 1 };

inline size_t wdtype_size(WDType t) { return t == WDType::F16 ? 2 : 4; }

struct WEntry {
    std::string name;
    std::vector<int64_t> shape;
    WDType dtype = WDType::F16;
    std::string file;
    const void* data = nullptr;  // mapped bytes (null for an empty tensor)
    size_t bytes = 0;
    int64_t numel() const;
};

// Mirrors Manifest::Architecture (include/denoiser/weight_loader.h:30-39)
// with the reference parser's defaults (weight_loader.cc:102-116).
struct ManifestArch {
    std::string type = "nafnet_residual";
    std::vector<int> enc_channels;
    int num_levels = 4;
    int base_channels = 32;
    int in_channels = 3;
    int out_channels = 3;
    int num_frames = 3;
    bool use_warp = false;
};

class HostWeights {
public:
    explicit HostWeights(const std::string& manifest_path);
    ~HostWeights();
    HostWeights(const HostWeights&) = delete;
    HostWeights& operator=(const HostWeights&) = delete;

    bool contains(const std::string& name) const { return index_.count(name) > 0; }
    const WEntry& entry(const std::string& name) const;
    // Values of `name` as float32 (fp16 entries are widened exactly).
    std::vector<float> to_f32(const std::string& name) const;
    const std::vector<WEntry>& entries() const { return entries_; }
    const ManifestArch& arch() const { return arch_; }
    const std::string& version() const { return version_; }
    WDType dtype() const { return dtype_; }
    const std::string& path() const { return path_; }

private:
    struct Mapping {
        void* ptr = nullptr;
        size_t size = 0;
    };
    std::string path_;
    std::string version_ = "1.0";
    WDType dtype_ = WDType::F16;
    ManifestArch arch_;
    std::vector<WEntry> entries_;
    std::unordered_map<std::string, size_t> index_;
    std::vector<Mapping> maps_;
};

WDType parse_wdtype(const std::string& s);

}  // namespace dnb
