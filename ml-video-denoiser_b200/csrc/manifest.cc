#include "manifest.h"

#include <cuda_fp16.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <sstream>

#include "json.h"

namespace dnb {

namespace fs = std::filesystem;

int64_t WEntry::numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return shape.empty() ? 1 : n;
}

WDType parse_wdtype(const std::string& s) {
    if (s == "float16") return WDType::F16;
    if (s == "float32") return WDType::F32;
    throw FormatError("Unknown dtype string: " + s);
}

HostWeights::HostWeights(const std::string& manifest_path) : path_(manifest_path) {
    const fs::path mp(manifest_path);
    if (!fs::exists(mp)) throw IoError("Manifest not found: " + manifest_path);
    std::ifstream f(manifest_path, std::ios::binary);
    if (!f.is_open()) throw IoError("Cannot open manifest: " + manifest_path);
    std::stringstream ss;
    ss << f.rdbuf();
    Json j;
    try {
        j = parse_json(ss.str());
    } catch (const JsonError& e) {
        throw FormatError(e.what());
    }
    if (j.kind != Json::Object) throw FormatError("manifest JSON: top level is not an object");
    try {
        version_ = j.get_string("version", "1.0");
        dtype_ = parse_wdtype(j.get_string("dtype", "float16"));
        if (j.has("architecture")) {
            const Json& a = j.at("architecture");
            arch_.type = a.get_string("type", "nafnet_residual");
            arch_.base_channels = static_cast<int>(a.get_int("base_channels", 32));
            arch_.in_channels = static_cast<int>(a.get_int("in_channels", 3));
            arch_.out_channels = static_cast<int>(a.get_int("out_channels", 3));
            arch_.num_levels = static_cast<int>(a.get_int("num_levels", 4));
            arch_.num_frames = static_cast<int>(a.get_int("num_frames", 3));
            arch_.use_warp = a.get_bool("use_warp", false);
            if (a.has("enc_channels")) {
                for (const Json& c : a.at("enc_channels").arr)
                    arch_.enc_channels.push_back(static_cast<int>(c.num));
            }
        }
        const Json& layers = j.at("layers");
        if (layers.kind != Json::Array) throw FormatError("manifest JSON: 'layers' is not an array");
        for (const Json& l : layers.arr) {
            WEntry e;
            e.name = l.at("name").str;
            e.dtype = parse_wdtype(l.at("dtype").str);
            e.file = l.at("file").str;
            for (const Json& d : l.at("shape").arr) {
                if (d.kind != Json::Number || d.num < 0) throw FormatError("bad shape for " + e.name);
                e.shape.push_back(static_cast<int64_t>(d.num));
            }
            index_[e.name] = entries_.size();
            entries_.push_back(std::move(e));
        }
    } catch (const JsonError& e) {
        throw FormatError(e.what());
    }

    const fs::path base = mp.parent_path();
    maps_.resize(entries_.size());
    for (size_t i = 0; i < entries_.size(); ++i) {
        WEntry& e = entries_[i];
        const std::string bin = (base / e.file).string();
        const int fd = ::open(bin.c_str(), O_RDONLY);
        if (fd == -1)
            throw IoError("Cannot open weight file: " + bin + " (" + std::strerror(errno) + ")");
        struct stat st {};
        if (::fstat(fd, &st) == -1) {
            ::close(fd);
            throw IoError("Cannot stat: " + bin);
        }
        const size_t size = static_cast<size_t>(st.st_size);
        const size_t want = static_cast<size_t>(e.numel()) * wdtype_size(e.dtype);
        if (size != want) {
            ::close(fd);
            throw FormatError("Weight file size mismatch for " + e.name + ": " + bin + " has " +
                              std::to_string(size) + " bytes, shape needs " + std::to_string(want));
        }
        if (size > 0) {
            void* p = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE | MAP_POPULATE, fd, 0);
            if (p == MAP_FAILED) {
                ::close(fd);
                throw IoError("mmap failed for: " + bin);
            }
            maps_[i] = {p, size};
            e.data = p;
            e.bytes = size;
        }
        ::close(fd);
    }
}

HostWeights::~HostWeights() {
    for (auto& m : maps_)
        if (m.ptr) ::munmap(m.ptr, m.size);
}

const WEntry& HostWeights::entry(const std::string& name) const {
    auto it = index_.find(name);
    if (it == index_.end()) throw NotFoundError("WeightStore: layer not found: " + name);
    return entries_[it->second];
}

std::vector<float> HostWeights::to_f32(const std::string& name) const {
    const WEntry& e = entry(name);
    const size_t n = static_cast<size_t>(e.numel());
    std::vector<float> out(n);
    if (!e.data) return out;
    if (e.dtype == WDType::F32) {
        std::memcpy(out.data(), e.data, n * 4);
    } else {
        const __half* h = static_cast<const __half*>(e.data);
        for (size_t i = 0; i < n; ++i) out[i] = __half2float(h[i]);
    }
    return out;
}

}  // namespace dnb
