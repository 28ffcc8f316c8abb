// Status codes of the C-ABI -> the exceptions the reference engine throws.
#pragma once

#include <stdexcept>
#include <string>

#include "denoiser_b200.h"

namespace denoiser::detail {

// DN_ERR_NOT_FOUND -> std::out_of_range (missing weight key),
// DN_ERR_INVALID_ARG -> std::invalid_argument, anything else ->
// std::runtime_error; the message is dn_last_error().
inline void check(int rc) {
    if (rc == DN_OK) return;
    const std::string msg = dn_last_error();
    if (rc == DN_ERR_NOT_FOUND) throw std::out_of_range(msg);
    if (rc == DN_ERR_INVALID_ARG) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

}  // namespace denoiser::detail
