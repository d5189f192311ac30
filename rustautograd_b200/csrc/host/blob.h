// The plan wire format crossing the C ABI (include/rgc.h). A plan is flattened into one
// little-endian byte string: slots, pinned flags, constants, input and output slots, then the
// steps, with control-flow body plans nested inside their instruction.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "plan.h"

namespace rg {

constexpr uint32_t PLAN_BLOB_VERSION = 1;

std::vector<uint8_t> encode_plan(const Plan& p);
// Throws std::runtime_error on a malformed blob.
Plan decode_plan(const uint8_t* data, size_t len);

}  // namespace rg
