// lwm_host.hpp — host-side pieces shared by the C ABI translation units: the
// thread-local error text and the VarBuilder names of the weight blobs.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/lewm_b200.h"

namespace lwm {

// Stores `message` as this thread's lwm_last_error() text and returns `status`.
lwm_status set_last_error(lwm_status status, const std::string& message);

// One tensor of a weight blob: its VarBuilder path, shape, place in the blob
// and the file it lives in (SkyJEPA: 0 latent model, 1 prober).
struct NamedTensor {
    std::string name;
    std::vector<uint32_t> shape;
    size_t off = 0, n = 0;
    int file = 0;
};

// The blob's tensors in order; returns the element count (0: invalid config).
size_t skyjepa_named_tensors(const lwm_skyjepa_config& c, std::vector<NamedTensor>* out);
size_t lewm_named_tensors(const lwm_lewm_config& c, int names, std::vector<NamedTensor>* out);

}  // namespace lwm
