// k_noalloc.cu — a GroupNorm entry point that allocates no device memory.
//
// di_group_norm_nhwc needs a small scratch buffer for its per-chunk partial sums, which the library
// normally obtains with cudaMalloc on first use.  Some callers cannot allow that: hosts that hand the
// library a pre-sized memory budget and forbid allocation after start-up, code running where an
// allocation would synchronise the device or fail (for example under an external allocator that owns
// all device memory), and real-time paths that must not take the driver's allocation locks.  For them,
// di_group_norm_nhwc_noalloc keeps its scratch in a fixed array compiled into the library (one copy per
// GPU that loads the library, held until the process exits).
//
// Host code cannot use the array's name as a device address (on the host it is only a stand-in), so
// the device address is looked up once per device with cudaGetSymbolAddress and passed to the kernels.
// Under CUDA's lazy module loading that first lookup may load the library's device code, which
// allocates; the same set-up also loads the GroupNorm kernels, so only the first call on a device can
// allocate: callers make it at start-up.
#include <mutex>

#include "di_common.cuh"

namespace di {

int group_norm_nhwc(Ctx* c, int in_dtype, int out_dtype, const void* x1, int C1, const void* x2, int C2, int N,
                    int HW, int G, float eps, const float* gamma, const float* beta, int silu, void* y,
                    void* partial_ws);
size_t gn_nhwc_ws_bytes(int N, int HW, int G);
int gn_nhwc_preload(Ctx* c);

namespace {

// 1 MiB of (sum, sum-of-squares) partials: N * max(1, min(16, HW/256)) * G entries of 8 bytes.
constexpr size_t kNoAllocScratchBytes = 1u << 20;
static __device__ __align__(256) float2 g_gn_scratch[kNoAllocScratchBytes / sizeof(float2)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_gn_scratch on `device` (looked up once per device with that device current).
int scratch_address(Ctx* c, void** out) {
  if (c->device < 0 || c->device >= kMaxDevices) return set_error(c, DI_EUNSUPPORTED, "noalloc: device ordinal");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[c->device]) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gn_scratch);
    // load the GroupNorm kernels now too, so that no later call loads code (and allocates) on this device
    const int pl = e == cudaSuccess ? gn_nhwc_preload(c) : DI_OK;
    cudaSetDevice(prev);
    if (e != cudaSuccess || !p)
      return set_error(c, DI_ECUDA, std::string("noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    if (pl) return pl;
    g_scratch_addr[c->device] = p;
  }
  *out = g_scratch_addr[c->device];
  return DI_OK;
}

}  // namespace

// Called by di_destroy: the next call on `device` looks the address up again, so a module reloaded after
// the context is re-created (for example after a device reset) is never addressed through a stale pointer.
void noalloc_forget(int device) {
  if (device < 0 || device >= kMaxDevices) return;
  std::lock_guard<std::mutex> lk(g_mu);
  g_scratch_addr[device] = nullptr;
}

}  // namespace di

using namespace di;

extern "C" int di_group_norm_nhwc_noalloc(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N,
                                          int HW, int G, float eps, const float* gamma, const float* beta,
                                          int fuse_silu, void* y) {
  Ctx* c = ctx_of(h);
  if (!c || N <= 0 || HW <= 0 || G <= 0) return DI_EINVAL;
  const size_t need = gn_nhwc_ws_bytes(N, HW, G);
  if (need > kNoAllocScratchBytes)
    return set_error(c, DI_EINVAL,
                     "group_norm_nhwc_noalloc: needs " + std::to_string(need) + " bytes of scratch, the fixed maximum is " +
                         std::to_string(kNoAllocScratchBytes) + " (N * max(1, min(16, HW/256)) * G * 8 bytes)");
  void* scratch = nullptr;
  const int r = scratch_address(c, &scratch);
  if (r) return r;
  // Every partial entry the normalise pass reads is written by the statistics pass of the same call, so
  // the array's contents from an earlier call never leak into this one and nothing needs clearing.
  return group_norm_nhwc(c, dtype, dtype, x1, C1, x2, x2 ? C2 : 0, N, HW, G, eps, gamma, beta, fuse_silu, y, scratch);
}
