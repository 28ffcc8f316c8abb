// Opaque C-ABI handles shared between the C-ABI translation units.
#pragma once

#include <memory>

#include "manifest.h"

struct dn_weights {
    std::unique_ptr<dnb::HostWeights> hw;
};
