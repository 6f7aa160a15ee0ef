// rotate_noalloc.cu -- EvalRotate for callers that cannot allocate device
// memory.
//
// Who needs it: code that runs where cudaMalloc / cudaFree are not allowed
// or not wanted -- a host thread that must not take the driver's allocation
// locks while other threads launch, or a service with a fixed device-memory
// budget that must not grow per request.  The regular ckks_rotate takes its
// key-switching temporaries from the context's device-memory cache, which
// calls cudaMalloc whenever it needs a block it does not hold; this variant
// takes them from one fixed array compiled into the library instead, and the
// caller supplies input and output buffers.
//
// The array is a file-scope static __device__ array of kScratchBytes
// (128 MiB).  Every GPU that loads the library holds it until the process
// exits.  Host code cannot use the array's name as a device address, so the
// first call on each device looks the address up with cudaGetSymbolAddress
// (with that device current) and caches it; make that first call before any
// stream capture begins.  All calls share the one array and it keeps the
// last call's contents: calls whose work overlaps on the GPU (two streams,
// two host threads, two contexts on one device) race on it.  Nothing in it
// needs to start at zero -- every word a call reads was written earlier in
// that same call.
#include <cstring>
#include <mutex>

#include "../../include/ckks_b200.h"
#include "capi_types.hpp"
#include "ckks_internal.hpp"

namespace {

constexpr size_t kScratchBytes = 128ull << 20;
constexpr size_t kScratchWords = kScratchBytes / sizeof(uint64_t);

static __device__ __align__(256) uint64_t g_rotate_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint64_t* g_scratch_addr[kMaxDevices] = {};

// device address of the scratch array on `device`, looked up once per device
uint64_t* scratch_on(int device) {
  if (device < 0 || device >= kMaxDevices) throw ckks::Error(CKKS_EARG, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[device]) {
    int prev = 0;
    CKKS_CUDA(cudaGetDevice(&prev));
    CKKS_CUDA(cudaSetDevice(device));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rotate_scratch);
    cudaSetDevice(prev);
    if (e != cudaSuccess || p == nullptr)
      throw ckks::Error(CKKS_ECUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[device] = static_cast<uint64_t*>(p);
  }
  return g_scratch_addr[device];
}

}  // namespace

extern "C" int ckks_rotate_noalloc(ckks_ctx* ctx, const uint64_t* in_dev, int limbs, int k, uint64_t* out_dev) {
  try {
    if (!ctx || !ctx->c) throw ckks::Error(CKKS_EARG, "null context");
    ckks::Context& c = *ctx->c;
    if (!in_dev || !out_dev) throw ckks::Error(CKKS_EARG, "null device buffer");
    if (limbs < 1 || limbs > c.L) throw ckks::Error(CKKS_EARG, "limb count outside 1..L");
    // the scratch address and the context's stream belong to the context's
    // device: launching from another current device would hand its kernels
    // the wrong GPU's array
    int cur = -1;
    CKKS_CUDA(cudaGetDevice(&cur));
    if (cur != c.params.device)
      throw ckks::Error(CKKS_EARG, "current device " + std::to_string(cur) + " is not the context's device " +
                                       std::to_string(c.params.device));
    const size_t N = (size_t)c.N, S = (size_t)limbs * N, E = (size_t)limbs + c.Kx(limbs);
    const uint64_t *lo_in = in_dev, *hi_in = in_dev + 2 * S;
    const uint64_t *lo_out = out_dev, *hi_out = out_dev + 2 * S;
    if (lo_in < hi_out && lo_out < hi_in) throw ckks::Error(CKKS_EARG, "output overlaps input");
    const uint32_t g = c.galois(k);
    if (g == 1u) {  // the identity is a copy and needs no scratch
      CKKS_CUDA(cudaMemcpyAsync(out_dev, in_dev, sizeof(uint64_t) * 2 * S, cudaMemcpyDeviceToDevice, c.stream));
      return CKKS_OK;
    }
    const size_t beta = (size_t)c.lt(limbs).beta;
    const size_t need = (beta * E + 2 * E + 2 * (size_t)limbs) * N;
    if (need > kScratchWords)
      throw ckks::Error(CKKS_ECAPACITY, "rotation needs " + std::to_string(need * 8 >> 20) +
                                            " MiB of scratch; the fixed no-allocation array holds " +
                                            std::to_string(kScratchBytes >> 20) + " MiB");
    const uint64_t* key = c.switch_key(g, limbs);
    if (!key) throw ckks::Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(k));
    uint64_t* scratch = scratch_on(c.params.device);
    uint64_t* ext = scratch;                // beta * E limbs
    uint64_t* acc = ext + beta * E * N;     // 2 E limbs
    uint64_t* tmp = acc + 2 * E * N;        // limbs (ModUp copy), then 2 limbs (ModDown conversion)
    ckks::modup_with(c, in_dev + S, limbs, ext, tmp, c.stream);
    ckks::ks_inner(c, ext, limbs, key, g, acc, c.stream);
    ckks::moddown2_with(c, acc, limbs, in_dev, g, nullptr, out_dev, out_dev + S, tmp, c.stream);
    return CKKS_OK;
  } catch (const ckks::Error& e) {
    ckks::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    ckks::set_last_error(e.what());
    return CKKS_EARG;
  }
}
