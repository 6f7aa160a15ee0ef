// capi_types.hpp -- definitions of the opaque handles of include/ckks_b200.h,
// shared by the translation units that implement C-ABI entry points.
#pragma once
#include <memory>
#include <mutex>
#include <string>
#include <unordered_set>

#include "ckks_internal.hpp"

namespace ckks {
// records the message ckks_last_error() returns on this thread
void set_last_error(const std::string& msg);
}  // namespace ckks

struct ckks_ct;
struct ckks_pt;
struct ckks_block;

// Objects register with their context.  Destroying a context first frees the
// device memory of every object still alive and marks it orphaned, so that
// handles released afterwards (in any order, e.g. by a garbage collector)
// only free their host-side struct.
struct ckks_ctx {
  std::unique_ptr<ckks::Context> c;
  std::mutex mu;
  std::unordered_set<ckks_ct*> cts;
  std::unordered_set<ckks_pt*> pts;
  std::unordered_set<ckks_block*> blocks;
};
struct ckks_ct {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};
struct ckks_pt {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};

namespace ckks {
// frees a block's device resources and detaches it from its context
void block_orphan(ckks_block* b);
}  // namespace ckks
