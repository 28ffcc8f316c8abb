// C-ABI of the host half of WeightStore (include/denoiser/weight_loader.h
// :61-101 of the reference): parse manifest.json, map and validate every .bin,
// look tensors up by name. No device is needed, so format errors surface on
// any host.
#include <cstring>
#include <memory>
#include <new>

#include "capi_internal.h"
#include "manifest.h"
#include "status.h"

using namespace dnb;


extern "C" {

int dn_weights_open(const char* manifest_path, dn_weights** out) {
    if (!manifest_path || !out) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_open: null argument");
    *out = nullptr;
    try {
        auto w = std::make_unique<dn_weights>();
        w->hw = std::make_unique<HostWeights>(manifest_path);
        *out = w.release();
        return DN_OK;
    } catch (const NotFoundError& e) {
        return dn_fail(DN_ERR_NOT_FOUND, e.what());
    } catch (const IoError& e) {
        return dn_fail(DN_ERR_IO, e.what());
    } catch (const FormatError& e) {
        return dn_fail(DN_ERR_FORMAT, e.what());
    } catch (const std::exception& e) {
        return dn_fail(DN_ERR_FORMAT, e.what());
    }
}

void dn_weights_close(dn_weights* w) { delete w; }

int dn_weights_count(const dn_weights* w) {
    if (!w) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_count: null handle");
    return static_cast<int>(w->hw->entries().size());
}

int dn_weights_contains(const dn_weights* w, const char* name) {
    if (!w || !name) return 0;
    return w->hw->contains(name) ? 1 : 0;
}

int dn_weights_info(const dn_weights* w, const char* name, int64_t* shape, int* ndim, int* dtype,
                    const void** host_data) {
    if (!w || !name) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_info: null argument");
    if (!w->hw->contains(name))
        return dn_fail_str(DN_ERR_NOT_FOUND, std::string("WeightStore: layer not found: ") + name);
    const WEntry& e = w->hw->entry(name);
    if (ndim) *ndim = static_cast<int>(e.shape.size());
    if (shape)
        for (size_t i = 0; i < e.shape.size() && i < 8; ++i) shape[i] = e.shape[i];
    if (dtype) *dtype = static_cast<int>(e.dtype);
    if (host_data) *host_data = e.data;
    return DN_OK;
}

int dn_weights_name(const dn_weights* w, int index, const char** name) {
    if (!w || !name) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_name: null argument");
    if (index < 0 || index >= static_cast<int>(w->hw->entries().size()))
        return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_name: index out of range");
    *name = w->hw->entries()[index].name.c_str();
    return DN_OK;
}

int dn_weights_arch(const dn_weights* w, char* type_buf, int type_buf_len, int* base_channels,
                    int* num_levels, int* in_channels, int* num_frames, int* use_warp) {
    if (!w) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_arch: null handle");
    const ManifestArch& a = w->hw->arch();
    if (type_buf && type_buf_len > 0) {
        std::strncpy(type_buf, a.type.c_str(), type_buf_len - 1);
        type_buf[type_buf_len - 1] = '\0';
    }
    if (base_channels) *base_channels = a.base_channels;
    if (num_levels) *num_levels = a.num_levels;
    if (in_channels) *in_channels = a.in_channels;
    if (num_frames) *num_frames = a.num_frames;
    if (use_warp) *use_warp = a.use_warp ? 1 : 0;
    return DN_OK;
}

int dn_weights_meta(const dn_weights* w, const char** version, int* dtype, int* enc_channels, int max_enc,
                    int* n_enc, int* out_channels) {
    if (!w) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_meta: null handle");
    const ManifestArch& a = w->hw->arch();
    if (version) *version = w->hw->version().c_str();
    if (dtype) *dtype = w->hw->dtype() == WDType::F16 ? 1 : 0;
    if (n_enc) *n_enc = static_cast<int>(a.enc_channels.size());
    if (enc_channels)
        for (int i = 0; i < max_enc && i < static_cast<int>(a.enc_channels.size()); ++i) enc_channels[i] = a.enc_channels[i];
    if (out_channels) *out_channels = a.out_channels;
    return DN_OK;
}

int dn_weights_file(const dn_weights* w, const char* name, const char** file) {
    if (!w || !name || !file) return dn_fail(DN_ERR_INVALID_ARG, "dn_weights_file: null argument");
    if (!w->hw->contains(name)) return dn_fail_str(DN_ERR_NOT_FOUND, std::string("weight not found: ") + name);
    *file = w->hw->entry(name).file.c_str();
    return DN_OK;
}

const char* dn_weights_path(const dn_weights* w) { return w ? w->hw->path().c_str() : ""; }

}  // extern "C"
