// capi_types.hpp -- definitions of the opaque handles of include/ckks_b200.h,
// shared by the translation units that implement C-ABI entry points.
#pragma once
#include <memory>
#include <string>

#include "ckks_internal.hpp"

namespace ckks {
// records the message ckks_last_error() returns on this thread
void set_last_error(const std::string& msg);
}  // namespace ckks

struct ckks_ctx {
  std::unique_ptr<ckks::Context> c;
};
struct ckks_ct {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};
struct ckks_pt {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};
