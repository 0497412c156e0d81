// di_core.cu — context, buffers, submission and error plumbing of the libdi C ABI.
//
// Mirrors the device lifecycle of the reference's WebGPU host: a context per device (requestDevice,
// unet-wgsl.js:64-72) with a sticky fault flag (device.lost / uncapturederror, unet-wgsl.js:73-84),
// buffers (createStorage/createOutput/readBack, wgsl-ops.js:1172-1210) and one queue (the stream).
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "di_common.cuh"

struct di_ctx_s {
  di::Ctx c;
};
struct di_buf_s {
  di_ctx_s* ctx;
  void* ptr;
  size_t bytes;
};

namespace di {

void noalloc_forget(int device);  // k_noalloc.cu

int set_error(Ctx* c, int code, const std::string& msg) {
  if (c) c->last_error = msg;
  return code;
}

int check_launch(Ctx* c, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    c->sticky = 1;
    return set_error(c, DI_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return DI_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz, std::string* err) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = fn(map, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) {
      char buf[256];
      snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) rank=%d base=%p", (int)r, rank, base);
      *err = buf;
    }
    return false;
  }
  return true;
}

}  // namespace di

using di::set_error;

extern "C" {

int di_init(int device_ordinal, di_ctx_t* out) {
  if (!out) return DI_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device_ordinal < 0 || device_ordinal >= n) return DI_ECUDA;
  if (cudaSetDevice(device_ordinal) != cudaSuccess) return DI_ECUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device_ordinal) != cudaSuccess) return DI_ECUDA;
  if (prop.major != 10) return DI_EUNSUPPORTED;  // sm_100a kernels only
  auto* h = new di_ctx_s();
  h->c.device = device_ordinal;
  h->c.num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&h->c.stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete h;
    return DI_ECUDA;
  }
  h->c.own_stream = true;
  if (cudaMalloc(&h->c.d_err, sizeof(int)) != cudaSuccess) {
    cudaStreamDestroy(h->c.stream);
    delete h;
    return DI_ENOMEM;
  }
  cudaMemset(h->c.d_err, 0, sizeof(int));
  cudaDeviceSynchronize();
  *out = h;
  return DI_OK;
}

void di_destroy(di_ctx_t ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->c.device);
  cudaStreamSynchronize(ctx->c.stream);
  if (ctx->c.d_err) cudaFree(ctx->c.d_err);
  if (ctx->c.gn_bar) cudaFree(ctx->c.gn_bar);
  for (auto& w : ctx->c.ws)
    if (w.ptr) cudaFree(w.ptr);
  if (ctx->c.own_stream) cudaStreamDestroy(ctx->c.stream);
  di::noalloc_forget(ctx->c.device);
  delete ctx;
}

int di_set_stream(di_ctx_t ctx, void* s) {
  if (!ctx) return DI_EINVAL;
  // Launches go to `s` verbatim from now on (NULL = the CUDA default stream); the context's own
  // stream, created by di_init, is released the first time a caller supplies one.
  if (ctx->c.own_stream) {
    cudaStreamSynchronize(ctx->c.stream);
    cudaStreamDestroy(ctx->c.stream);
    ctx->c.own_stream = false;
  }
  ctx->c.stream = static_cast<cudaStream_t>(s);
  return DI_OK;
}

void* di_get_stream(di_ctx_t ctx) { return ctx ? static_cast<void*>(ctx->c.stream) : nullptr; }

int di_buf_alloc(di_ctx_t ctx, size_t bytes, di_buf_t* out) {
  if (!ctx || !out) return DI_EINVAL;
  *out = nullptr;
  cudaSetDevice(ctx->c.device);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
    cudaGetLastError();
    return set_error(&ctx->c, DI_ENOMEM, "di_buf_alloc: cudaMalloc failed");
  }
  *out = new di_buf_s{ctx, p, bytes};
  return DI_OK;
}

int di_buf_free(di_buf_t b) {
  if (!b) return DI_EINVAL;
  cudaSetDevice(b->ctx->c.device);
  cudaStreamSynchronize(b->ctx->c.stream);
  cudaFree(b->ptr);
  delete b;
  return DI_OK;
}

void* di_buf_ptr(di_buf_t b) { return b ? b->ptr : nullptr; }
size_t di_buf_size(di_buf_t b) { return b ? b->bytes : 0; }

int di_buf_upload(di_buf_t b, const void* src, size_t bytes, size_t off) {
  if (!b || !src || off + bytes > b->bytes) return DI_EINVAL;
  cudaSetDevice(b->ctx->c.device);
  if (cudaMemcpyAsync(static_cast<char*>(b->ptr) + off, src, bytes, cudaMemcpyHostToDevice, b->ctx->c.stream) !=
      cudaSuccess)
    return set_error(&b->ctx->c, DI_ECUDA, "di_buf_upload failed");
  return cudaStreamSynchronize(b->ctx->c.stream) == cudaSuccess ? DI_OK : DI_ECUDA;
}

int di_buf_download(di_buf_t b, void* dst, size_t bytes, size_t off) {
  if (!b || !dst || off + bytes > b->bytes) return DI_EINVAL;
  cudaSetDevice(b->ctx->c.device);
  if (cudaMemcpyAsync(dst, static_cast<const char*>(b->ptr) + off, bytes, cudaMemcpyDeviceToHost, b->ctx->c.stream) !=
      cudaSuccess)
    return set_error(&b->ctx->c, DI_ECUDA, "di_buf_download failed");
  return cudaStreamSynchronize(b->ctx->c.stream) == cudaSuccess ? DI_OK : DI_ECUDA;
}

int di_wait(di_ctx_t ctx) {
  if (!ctx) return DI_EINVAL;
  cudaError_t e = cudaStreamSynchronize(ctx->c.stream);
  if (e != cudaSuccess) {
    ctx->c.sticky = 1;
    return set_error(&ctx->c, DI_ECUDA, std::string("di_wait: ") + cudaGetErrorString(e));
  }
  return ctx->c.sticky ? DI_EFAULT : DI_OK;
}

const char* di_last_error(di_ctx_t ctx) { return ctx ? ctx->c.last_error.c_str() : "null context"; }

int di_device_fault(di_ctx_t ctx) {
  if (!ctx) return DI_EINVAL;
  int v = 0;
  if (cudaMemcpyAsync(&v, ctx->c.d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->c.stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->c.stream) != cudaSuccess) {
    ctx->c.sticky = 1;
    return DI_ECUDA;
  }
  if (v) ctx->c.sticky = 1;
  return v;
}

int di_clear_fault(di_ctx_t ctx) {
  if (!ctx) return DI_EINVAL;
  cudaMemsetAsync(ctx->c.d_err, 0, sizeof(int), ctx->c.stream);
  ctx->c.sticky = 0;
  ctx->c.last_error.clear();
  return cudaStreamSynchronize(ctx->c.stream) == cudaSuccess ? DI_OK : DI_ECUDA;
}

}  // extern "C"

namespace {
// One thread waits, through the same bounded mbarrier wait every pipeline kernel uses, on a barrier phase
// that nothing completes; after `timeout_ns` it records DEVERR_WAIT_PROBE in the error word and returns.
__global__ void wait_probe_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  di::mbar_init(&bar, 1);
  di::fence_mbar_init();
  di::mbar_wait(&bar, 0, err, di::DEVERR_WAIT_PROBE, timeout_ns);
}
}  // namespace

extern "C" int di_debug_wait_timeout(di_ctx_t ctx, int timeout_us) {
  if (!ctx) return DI_EINVAL;
  if (timeout_us <= 0 || timeout_us > 1000000)
    return set_error(&ctx->c, DI_EINVAL, "di_debug_wait_timeout: timeout_us must be in 1 .. 1000000");
  wait_probe_kernel<<<1, 32, 0, ctx->c.stream>>>(ctx->c.d_err, 1000ull * (unsigned long long)timeout_us);
  return di::check_launch(&ctx->c, "wait_probe_kernel");
}

// Internal accessors used by the other translation units.
namespace di {
Ctx* ctx_of(di_ctx_t h) { return h ? &h->c : nullptr; }

// Library-owned scratch (GroupNorm partials, packed operands of the fp32 op family): one growable
// device buffer per slot.  Growing synchronises the stream first so no queued kernel still reads the
// old buffer.  Callers that capture CUDA graphs size the slots before capture.
void* workspace(Ctx* c, size_t bytes, int slot) {
  if (slot < 0 || slot >= (int)(sizeof(c->ws) / sizeof(c->ws[0]))) return nullptr;
  auto& w = c->ws[slot];
  if (w.bytes >= bytes && w.ptr) return w.ptr;
  cudaStreamSynchronize(c->stream);
  if (w.ptr) cudaFree(w.ptr);
  w.ptr = nullptr;
  w.bytes = 0;
  size_t want = std::max<size_t>(bytes, 1 << 20);
  if (cudaMalloc(&w.ptr, want) != cudaSuccess) {
    cudaGetLastError();
    w.ptr = nullptr;
    return nullptr;
  }
  w.bytes = want;
  return w.ptr;
}
}  // namespace di
