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
struct ckks_diag;

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
  std::unordered_set<ckks_diag*> diags;
};
struct ckks_ct {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};
struct ckks_pt {
  ckks_ctx* owner = nullptr;
  ckks::DevPoly p;
};
// the encoded BSGS diagonals of one matrix at one level (the reference's
// cached_diagonal_plains): n1 * n2 plaintexts of `limbs` limbs in the
// tile-major layout the inner-sum kernels stream, from the context's
// allocator
struct ckks_diag {
  ckks_ctx* owner = nullptr;
  uint64_t* data = nullptr;
  int limbs = 0, n1 = 0, n2 = 0, batch = 0;
  double scale = 0.0;
};

namespace ckks {
// frees a block's device resources and detaches it from its context
void block_orphan(ckks_block* b);
}  // namespace ckks
