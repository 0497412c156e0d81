// plan.cu — the SD-Turbo U-Net forward (and its ResNet / transformer blocks) as a pre-planned,
// CUDA-graph-replayed sequence of sm_100a kernels.
//
// The reference walks a 5,478-node ONNX graph op by op on every call (Executor.run,
// wgsl-executor.js:1248-1466): per-node uniform-buffer creation, buffer-pool lookups, NCHW fp32.  Here the
// architecture (SD2.1 / SD-Turbo: 320/640/1280/1280 channels, 2 ResNet blocks per level, a transformer
// at the first three levels, head dim 64, cross-attention over a 77x1024 context) is walked once at
// plan time: weights are drawn (or supplied by the caller by parameter name), converted to fp16 and
// packed for the kernels; every activation and scratch buffer is placed; each kernel launch is
// recorded with fixed pointers and TMA descriptors.  The first forward captures the launches into a
// CUDA graph; every later forward is one graph launch.
//
// Data layout in HBM: activations NHWC fp16 (the transformer's token-major [B, H*W, C] is the same
// memory), weights fp16 K-major ([Co][ky][kx][Ci] for 3x3 convs, [out][in] for linears, Q/K/V stacked
// into one [3C, C] matrix, cross-attention K/V stacked into [2C, 1024], GEGLU value/gate rows
// interleaved per 64-column tile), biases and norm affines fp32.
//
// Fusions: GroupNorm apply + SiLU in one pass that also materialises the skip concat; bias, the
// timestep-embedding broadcast and the residual in the conv / linear epilogues; the GEGLU gate in the
// FF up-projection epilogue; the 1x1 shortcut reads the two concat sources directly; every ResNet
// block's time projection in one GEMV; Q/K/V in one GEMM; attention as one flash kernel.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "di_common.cuh"

namespace di {

int gemm_linear(Ctx* c, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
                const float* bias, const void* R, int res_f32, void* Y, int out_f32, int geglu, const float* rowvec,
                int rowvec_div, void* splitk_ws = nullptr, const GnFuse* gnf = nullptr, int gnf_hw = 0, int act = 0);
int gemm_conv3x3(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W, int stride,
                 const void* Wt, int Co, const float* bias, const float* temb, const void* residual, int res_f32,
                 void* y, int out_f32, int temb_ld, void* splitk_ws = nullptr, const GnFuse* gnf = nullptr,
                 int act = 0);
int group_norm_nhwc(Ctx* c, int in_dtype, int out_dtype, const void* x1, int C1, const void* x2, int C2, int N,
                    int HW, int G, float eps, const float* gamma, const float* beta, int silu, void* y,
                    void* partial_ws);
size_t gn_nhwc_ws_bytes(int N, int HW, int G);
bool gn_grid_usable(Ctx* c, int dtype, int N, int HW, int C1, int C2, int G);
size_t gn_grid_ws_bytes(Ctx* c, int N, int HW, int C, int G);
int gn_nhwc_grid_launch(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                        float eps, const float* gamma, const float* beta, int silu, void* y, float2* partial,
                        unsigned* bar);
bool gn_cluster_usable(int dtype, int HW, int C1, int C2, int G);
int gn_nhwc_cluster_launch(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                           float eps, const float* gamma, const float* beta, int silu, void* y);
int gn_apply_with_stats(Ctx* c, const void* x, int C, int N, int HW, const long long* stats, float eps,
                        const float* gamma, const float* beta, int silu, void* y);
int gn_table_nhwc(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G, float eps,
                  const float* gamma, const float* beta, float2* table);
int gn_nhwc_via_table(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                      float eps, const float* gamma, const float* beta, int silu, void* y, float2* table);
int gemm_kernel_count(Ctx* c, int M, int N, int K, int geglu);
int layer_norm(Ctx* c, int in_dtype, int out_dtype, const void* x, const float* g, const float* b, void* y, int rows,
               int D, float eps);
int attention(Ctx* c, int dtype, const void* Q, const void* K, const void* V, void* O, int B, int H, int Sq, int Skv,
              int layout, long long ld_q, long long ld_k, long long ld_v, long long ld_o, int causal = 0);
int gemv(Ctx* c, const float* x, int B, int K, const void* W, int w_f16, const float* bias, int N, int silu_in,
         float* y, int ldy);
int tembed(Ctx* c, const float* t, int B, const float* W1, const float* b1, const float* W2, const float* b2, int Din,
           int Dh, float* hidden, float* y);
int nchw_to_nhwc(Ctx* c, int in_dt, int out_dt, const void* x, void* y, int N, int C, int HW);
int nhwc_to_nchw(Ctx* c, int in_dt, int out_dt, const void* x, void* y, int N, int C, int HW);

// ---------------------------------------------------------------------------------------------
// Seeded synthetic parameters (the build's documented scheme, restated independently of the CPU
// oracle; tests compare the two bit for bit):
//   key = mix64(seed * 0x9E3779B97F4A7C15 + fnv1a64(name)),
//   u_i = (mix64(key + (i+1) * 0x9E3779B97F4A7C15) >> 40) * 2^-24,
//   uniform(b) = (2u - 1) * b in float; normal = Box-Muller (double) on (u_2j, u_2j+1), cos even / sin odd.
// ---------------------------------------------------------------------------------------------
static inline uint64_t smix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static inline uint64_t name_hash(const char* s) {
  uint64_t h = 0xcbf29ce484222325ULL;
  while (*s) { h ^= (unsigned char)*s++; h *= 0x100000001b3ULL; }
  return h;
}
static inline float unit24(uint64_t key, uint64_t i) {
  return (float)(smix(key + (i + 1) * 0x9E3779B97F4A7C15ULL) >> 40) * (1.0f / 16777216.0f);
}
template <typename F>
static void par_for(size_t n, F f) {
  const unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  if (n < (1u << 16) || nt == 1) { for (size_t i = 0; i < n; ++i) f(i); return; }
  std::vector<std::thread> th;
  const size_t per = (n + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t)
    th.emplace_back([=] { for (size_t i = t * per; i < std::min(n, (t + 1) * per); ++i) f(i); });
  for (auto& x : th) x.join();
}
void synth_uniform(uint64_t seed, const char* name, size_t n, float bound, float* out) {
  const uint64_t key = smix(seed * 0x9E3779B97F4A7C15ULL + name_hash(name));
  par_for(n, [&](size_t i) {
    const float u = unit24(key, i);
    const float t = 2.0f * u - 1.0f;
    out[i] = t * bound;
  });
}
void synth_normal(uint64_t seed, const char* name, size_t n, float mean, float stdv, float* out) {
  const uint64_t key = smix(seed * 0x9E3779B97F4A7C15ULL + name_hash(name));
  par_for(n, [&](size_t i) {
    const uint64_t j = i & ~(size_t)1;
    double u1 = (double)unit24(key, j), u2 = (double)unit24(key, j + 1);
    if (u1 < 1.0 / 16777216.0) u1 = 1.0 / 16777216.0;
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double z = (i & 1) ? r * std::sin(6.283185307179586 * u2) : r * std::cos(6.283185307179586 * u2);
    out[i] = (float)((double)mean + (double)stdv * z);
  });
}

namespace {

// Latent NCHW fp32 -> NHWC fp16 padded to Cp channels.  sched (device, may be null) holds the Euler
// scheduler's scaleModelInput factor in sched[0] (scheduler.js:95-101): the value fed to the U-Net is
// float(double(x) * sched[0]), the reference's double multiply and Float32Array store.
__global__ void latent_in_kernel(const float* __restrict__ x, __half* __restrict__ y, int N, int C, int HW, int Cp,
                                 const double* __restrict__ sched) {
  pdl_begin();
  const size_t total = (size_t)N * HW * Cp;
  const double scale = sched ? sched[0] : 1.0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = i % Cp;
    const size_t np = i / Cp;
    const int p = np % HW;
    const size_t n = np / HW;
    const float v = c < C ? (float)__dmul_rn((double)x[(n * C + c) * HW + p], scale) : 0.f;
    y[i] = __float2half_rn(v);
  }
}
// U-Net output NHWC fp16 (Cp channels) -> NCHW fp32 noise prediction.  With `next`, also the Euler step
// of scheduler.js:105-110: next = float(double(x_in) + sched[1] * double(eps)), sched[1] = sigma_{i+1} -
// sigma_i, rounded like the reference (a double product, then a double sum, no fused multiply-add).
__global__ void latent_out_kernel(const __half* __restrict__ x, int Cp, float* __restrict__ y, int N, int C, int HW,
                                  const float* __restrict__ x_in, const double* __restrict__ sched,
                                  float* __restrict__ next) {
  pdl_begin();
  const size_t total = (size_t)N * C * HW;
  const double dt = sched ? sched[1] : 0.0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = i % HW;
    const size_t nc = i / HW;
    const int c = nc % C;
    const size_t n = nc / C;
    const float e = __half2float(x[(n * HW + p) * Cp + c]);
    y[i] = e;
    if (next) next[i] = (float)__dadd_rn((double)x_in[i], __dmul_rn(dt, (double)e));
  }
}
// CLIP text embeddings: x[t, :] = token_embedding[ids[t]] + position_embedding[t % S] (fp16 tables, fp32
// sum).  Ids outside [0, V) are clamped for the read and flagged in the device error word.
__global__ void embed_tokens_kernel(const int* __restrict__ ids, int tokens, int S, const __half* __restrict__ tok,
                                    const __half* __restrict__ pos, int D, int V, float* __restrict__ x,
                                    int* __restrict__ err) {
  pdl_begin();
  const int per = D / 8;
  const size_t total = (size_t)tokens * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per), c = (int)(i % per) * 8;
    int id = ids[t];
    if (id < 0 || id >= V) {
      if (c == 0) atomicOr(err, DEVERR_BOUNDS);
      id = id < 0 ? 0 : V - 1;
    }
    const uint4 a = *reinterpret_cast<const uint4*>(tok + (size_t)id * D + c);
    const uint4 b = *reinterpret_cast<const uint4*>(pos + (size_t)(t % S) * D + c);
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    const __half2* bh = reinterpret_cast<const __half2*>(&b);
    float r[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(ah[k]), g = __half22float2(bh[k]);
      r[2 * k] = f.x + g.x;
      r[2 * k + 1] = f.y + g.y;
    }
    float4* o = reinterpret_cast<float4*>(x + (size_t)t * D + c);
    o[0] = make_float4(r[0], r[1], r[2], r[3]);
    o[1] = make_float4(r[4], r[5], r[6], r[7]);
  }
}
// Row softmax in place on fp16 scores (the scale is folded into the query projection): one 256-thread
// block per row, eight columns per thread per step, fp32 max / sum (block reductions in a fixed order).
__global__ void softmax_rows_f16(__half* __restrict__ s, int cols) {
  pdl_begin();
  __shared__ float red[8];
  __half* row = s + (size_t)blockIdx.x * cols;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  float mx = -INFINITY;
  for (int c = t * 8; c < cols; c += 256 * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      mx = fmaxf(mx, fmaxf(f.x, f.y));
    }
  }
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[wid] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  const float ml = mx * 1.4426950408889634f;
  float sum = 0.f;
  for (int c = t * 8; c < cols; c += 256 * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      sum += exp2f(fmaf(f.x, 1.4426950408889634f, -ml)) + exp2f(fmaf(f.y, 1.4426950408889634f, -ml));
    }
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < 8; ++w) sum += red[w];
  const float inv = 1.0f / sum;
  for (int c = t * 8; c < cols; c += 256 * 8) {
    uint4 u = *reinterpret_cast<const uint4*>(row + c);
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      h[j] = __floats2half2_rn(exp2f(fmaf(f.x, 1.4426950408889634f, -ml)) * inv,
                               exp2f(fmaf(f.y, 1.4426950408889634f, -ml)) * inv);
    }
    *reinterpret_cast<uint4*>(row + c) = u;
  }
}

// Nearest 2x upsample, NHWC, 16-byte vectors (index math of wgsl-ops.js:921-943 with W_out = 2 W_in).
__global__ void upsample2_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, int N, int H, int W, int Cv) {
  pdl_begin();
  const size_t total = (size_t)N * 4 * H * W * Cv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int v = i % Cv;
    size_t r = i / Cv;
    const int ox = r % (2 * W);
    r /= (2 * W);
    const int oy = r % (2 * H);
    const size_t n = r / (2 * H);
    y[i] = x[((n * H + oy / 2) * W + ox / 2) * Cv + v];
  }
}
__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
  pdl_begin();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

}  // namespace

typedef int (*WeightFn)(const char* name, size_t n, float* dst, void* user);

// GroupNorm statistics of a GEMM-produced activation: `ptr` is set at build time when a GroupNorm
// consumer asks for them; the producer's recorded op reads it when it runs (null: no statistics).
struct GnStatSlot {
  long long* ptr = nullptr;
};

struct Act {
  void* p = nullptr;
  int N = 0, H = 0, W = 0, C = 0;
  GnStatSlot* st = nullptr;  // set when a GEMM epilogue can produce this tensor's GroupNorm(32) statistics
  size_t bytes() const { return (size_t)N * H * W * C * 2; }
};

// ---------------------------------------------------------------------------------------------
// Plan: arenas, parameter loading, recorded launches, CUDA graph.
// ---------------------------------------------------------------------------------------------
struct Plan {
  Ctx* c = nullptr;
  uint64_t seed = 0;
  WeightFn wfn = nullptr;
  void* wuser = nullptr;
  cudaStream_t stream = nullptr;  // private stream: graph capture needs a non-legacy stream
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  std::vector<void*> blocks;      // cudaMalloc'd regions
  std::vector<std::function<int()>> ops;
  cudaGraphExec_t gexec = nullptr;
  int launches = 0;               // kernels per forward (recorded ops)
  size_t weight_bytes = 0, act_bytes = 0;
  int err = DI_OK;
  std::string errmsg;

  // split-K partial sums of the GEMM kernel (at most ~2 CTAs per SM x 128x128 fp32 tiles); ops run
  // in stream order, so one buffer serves every launch of the plan
  void* splitk = nullptr;
  static constexpr size_t kSplitKBytes = kSplitKWsBytes;

  // temporary bump arena (reset per block; stream order makes reuse safe)
  char* tmp_base = nullptr;
  size_t tmp_cap = 0, tmp_off = 0, tmp_peak = 0;

  ~Plan() {
    if (gexec) cudaGraphExecDestroy(gexec);
    if (pexec) cudaGraphExecDestroy(pexec);
    for (auto& k : kexec)
      if (k) cudaGraphExecDestroy(k);
    for (auto& e : pev) cudaEventDestroy(e);
    if (stream) { cudaStreamSynchronize(stream); cudaStreamDestroy(stream); }
    if (side) { cudaStreamSynchronize(side); cudaStreamDestroy(side); }
    for (auto& e : fork_ev) cudaEventDestroy(e);
    if (ev_in) cudaEventDestroy(ev_in);
    if (ev_out) cudaEventDestroy(ev_out);
    for (void* b : blocks) cudaFree(b);
  }

  void fail(int code, const std::string& m) {
    if (err == DI_OK) { err = code; errmsg = m; }
  }

  void* dalloc(size_t bytes) {
    if (err) return nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
      cudaGetLastError();
      fail(DI_ENOMEM, "plan: cudaMalloc of " + std::to_string(bytes) + " bytes failed");
      return nullptr;
    }
    blocks.push_back(p);
    return p;
  }
  void* act_alloc(size_t bytes) {
    act_bytes += bytes;
    return dalloc(bytes);
  }
  void* tmp(size_t bytes) {
    const size_t off = (tmp_off + 255) & ~(size_t)255;
    if (off + bytes > tmp_cap) {
      fail(DI_ENOMEM, "plan: temporary arena exhausted");
      return nullptr;
    }
    tmp_off = off + bytes;
    tmp_peak = std::max(tmp_peak, tmp_off);
    return tmp_base + off;
  }
  void tmp_reset() { tmp_off = 0; }

  // kind 0: uniform weight (fan_out > 0) or bias (fan_out == 0); 1: normal(1, 0.02) (norm gamma);
  // 2: normal(0, 0.02) (norm beta).  init_mode picks the uniform bound:
  //   0 torch layer default: +-1/sqrt(fan_in) for weights and biases (the U-Net)
  //   1 Kaiming-uniform weights +-sqrt(6/fan_in), default biases (config 1)
  //   2 Xavier-uniform weights +-sqrt(6/(fan_in+fan_out)), zero biases (config 2)
  int init_mode = 0;
  std::vector<float> host_param(const std::string& name, size_t n, int kind, int fan_in, int fan_out = 0) {
    std::vector<float> h(n);
    if (wfn && wfn(name.c_str(), n, h.data(), wuser) == 0) {
    } else if (kind == 0) {
      float bound = 1.0f / std::sqrt((float)fan_in);
      if (init_mode == 1 && fan_out > 0) bound = std::sqrt(6.0f / (float)fan_in);
      if (init_mode == 2) bound = fan_out > 0 ? std::sqrt(6.0f / (float)(fan_in + fan_out)) : 0.0f;
      if (bound == 0.0f) std::fill(h.begin(), h.end(), 0.0f);
      else synth_uniform(seed, name.c_str(), n, bound, h.data());
    } else {
      synth_normal(seed, name.c_str(), n, kind == 1 ? 1.0f : 0.0f, 0.02f, h.data());
    }
    return h;
  }
  static void round_f16(std::vector<float>& v) {
    par_for(v.size(), [&](size_t i) { v[i] = __half2float(__float2half_rn(v[i])); });
  }
  const float* upload_f32(const std::vector<float>& v) {
    float* d = static_cast<float*>(dalloc(v.size() * 4));
    if (!d) return nullptr;
    cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
    weight_bytes += v.size() * 4;
    return d;
  }
  const void* upload_f16(const std::vector<float>& v) {
    std::vector<__half> h(v.size());
    par_for(v.size(), [&](size_t i) { h[i] = __float2half_rn(v[i]); });
    void* d = dalloc(h.size() * 2);
    if (!d) return nullptr;
    cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
    weight_bytes += h.size() * 2;
    return d;
  }
  // fp32 vector of fp16-rounded parameter values (biases, norm affines)
  const float* vec(const std::string& name, size_t n, int kind, int fan_in) {
    auto h = host_param(name, n, kind, fan_in);
    round_f16(h);
    return upload_f32(h);
  }

  // Per-op metadata: kind (0 tensor-core GEMM / conv, 1 attention, 2 normalisation, 3 other),
  // algorithmic FLOPs and HBM bytes, and how many kernels the op launches.
  struct OpInfo { int kind; double flops, bytes; int kernels; };
  std::vector<OpInfo> info;

  void record(std::function<int()> f, int kind = 3, double flops = 0, double bytes = 0, int kernels = 1) {
    // A plan's weights are written once at build time (and synchronised), so its GEMMs may fetch
    // weight tiles before the programmatic-dependency wait.
    Ctx* cc = c;
    ops.push_back([cc, f = std::move(f)] {
      cc->weights_const = true;
      const int r = f();
      cc->weights_const = false;
      return r;
    });
    info.push_back({kind, flops, bytes, kernels});
    launches += kernels;
  }

  // GroupNorm statistics arena (GnStatSlot): N x 32 groups x 3 int64 per requested tensor, zeroed at the
  // start of every forward (run_ops).
  std::deque<GnStatSlot> stat_slots;
  long long* stats_base = nullptr;
  size_t stats_cap = 0, stats_off = 0;  // in int64 units
  GnStatSlot* new_stat_slot() {
    stat_slots.emplace_back();
    return &stat_slots.back();
  }
  // A zeroed {arrivals, generation} barrier pair for one single-launch GroupNorm site (gn_nhwc_grid).
  // Each site has its own pair, so launches on the plan's side stream could never share one.
  unsigned* gn_bars = nullptr;
  int gn_bar_used = 0, gn_bar_cap = 0;
  unsigned* gn_bar_alloc() {
    if (gn_bar_used == gn_bar_cap) {
      gn_bar_cap = 256;
      gn_bar_used = 0;
      gn_bars = static_cast<unsigned*>(dalloc(sizeof(unsigned) * 2 * gn_bar_cap));
      if (!gn_bars) return nullptr;
      cudaMemset(gn_bars, 0, sizeof(unsigned) * 2 * gn_bar_cap);
    }
    return gn_bars ? gn_bars + 2 * gn_bar_used++ : nullptr;
  }
  long long* stats_alloc(int N) {
    const size_t need = (size_t)N * 32 * 3;
    if (!stats_base) {
      stats_cap = need * 160;
      stats_base = static_cast<long long*>(dalloc(stats_cap * sizeof(long long)));
      if (!stats_base) return nullptr;
    }
    if (stats_off + need > stats_cap) {
      fail(DI_ENOMEM, "plan: GroupNorm statistics arena exhausted");
      return nullptr;
    }
    long long* r = stats_base + stats_off;
    stats_off += need;
    return r;
  }
  // GEMM call with the GroupNorm statistics of its output when a consumer asked for them
  static int with_stats(Ctx* cc, const GnStatSlot* st, int hw, const std::function<int()>& f) {
    cc->gn_stats = st ? st->ptr : nullptr;
    cc->gn_stats_hw = hw;
    const int r = f();
    cc->gn_stats = nullptr;
    return r;
  }

  // Side branch: an op whose inputs are ready well before its consumer runs on a second stream, so
  // the captured graph forks there and joins at the consumer (join(j) before the consumer's launch).
  // The branch has its own split-K buffer; it may not share a temporary with the main chain.
  cudaStream_t side = nullptr;
  void* splitk_side = nullptr;
  std::vector<cudaEvent_t> fork_ev;  // [2j] fork, [2j + 1] join
  // fork_live[j]: branch j was enqueued in the current pass and not joined yet.  A consumer joins only a
  // live branch, and every pass ends by joining the rest (join_all), so a pass over a subset of the ops
  // (profile_kind) that runs a branch without its consumer, or a consumer without its branch, still
  // captures a well-formed graph.
  mutable std::vector<char> fork_live;
  int record_fork(std::function<int()> f, int kind, double flops, double bytes, int kernels) {
    return insert_fork(ops.size(), std::move(f), kind, flops, bytes, kernels);
  }
  // The same, inserted as op `at` (a branch built after the ops that follow it, e.g. the time MLP).
  int insert_fork(size_t at, std::function<int()> f, int kind, double flops, double bytes, int kernels) {
    if (!side) {
      if (cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking) != cudaSuccess) {
        fail(DI_ECUDA, "plan: side stream");
        return -1;
      }
      splitk_side = dalloc(kSplitKBytes);
    }
    const int j = (int)fork_ev.size() / 2;
    fork_ev.resize(fork_ev.size() + 2);
    fork_live.push_back(0);
    cudaEventCreateWithFlags(&fork_ev[2 * j], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&fork_ev[2 * j + 1], cudaEventDisableTiming);
    Ctx* cc = c;
    Plan* self = this;
    ops.insert(ops.begin() + at, [cc, self, j, f = std::move(f)] {
      cudaEventRecord(self->fork_ev[2 * j], cc->stream);
      cudaStreamWaitEvent(self->side, self->fork_ev[2 * j], 0);
      cudaStream_t main_stream = cc->stream;
      cc->stream = self->side;
      cc->weights_const = true;
      const int r = f();
      cc->weights_const = false;
      cc->stream = main_stream;
      cudaEventRecord(self->fork_ev[2 * j + 1], self->side);
      self->fork_live[j] = 1;
      return r;
    });
    info.insert(info.begin() + at, OpInfo{kind, flops, bytes, kernels});
    launches += kernels;
    return j;
  }
  void join(int j) const {
    if (j >= 0 && fork_live[j]) {
      cudaStreamWaitEvent(c->stream, fork_ev[2 * j + 1], 0);
      fork_live[j] = 0;
    }
  }
  void join_all() const {
    for (int j = 0; j < (int)fork_live.size(); ++j) join(j);
  }

  // Device time of the ops of one kind alone: a graph holding only those launches (same buffers, same
  // order) replayed `reps` times between two events; *ms = mean per replay.  Used to time the GEMM
  // kernel inside the step without per-op event nodes.
  cudaGraphExec_t kexec[4] = {nullptr, nullptr, nullptr, nullptr};
  int profile_kind(int kind, int reps, float* ms) {
    if (err) return err;
    if (kind < 0 || kind > 3) return DI_EINVAL;
    if (!gexec) {
      int r = forward();
      if (r) return r;
      cudaStreamSynchronize(stream);
    }
    cudaStream_t saved = c->stream;
    c->stream = stream;
    int r = DI_OK;
    if (!kexec[kind]) {
      cudaGraph_t g = nullptr;
      if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        c->stream = saved;
        return set_error(c, DI_ECUDA, "profile_kind: capture");
      }
      for (size_t i = 0; i < ops.size() && r == DI_OK; ++i)
        if (info[i].kind == kind) r = ops[i]();
      join_all();
      cudaError_t e = cudaStreamEndCapture(stream, &g);
      if (r != DI_OK || e != cudaSuccess || cudaGraphInstantiate(&kexec[kind], g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        c->stream = saved;
        cudaGetLastError();
        return set_error(c, DI_ECUDA, "profile_kind: graph");
      }
      cudaGraphDestroy(g);
    }
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaGraphLaunch(kexec[kind], stream);  // warm
    cudaEventRecord(e0, stream);
    for (int i = 0; i < reps; ++i) cudaGraphLaunch(kexec[kind], stream);
    cudaEventRecord(e1, stream);
    cudaEventSynchronize(e1);
    float t = 0.f;
    cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    c->stream = saved;
    if (cudaGetLastError() != cudaSuccess) return set_error(c, DI_ECUDA, "profile_kind: replay");
    *ms = t / std::max(1, reps);
    return DI_OK;
  }

  // LOG.profile analogue (wgsl-executor.js:1380-1390): a second graph with an event-record node between
  // every op, replayed `reps` times; op_ms[i] = mean device time of op i.
  cudaGraphExec_t pexec = nullptr;
  std::vector<cudaEvent_t> pev;
  int profile(int reps, float* op_ms) {
    if (err) return err;
    if (!gexec) {
      int r = forward();
      if (r) return r;
      cudaStreamSynchronize(stream);
    }
    cudaStream_t saved = c->stream;
    c->stream = stream;
    if (!pexec) {
      pev.resize(ops.size() + 1);
      for (auto& e : pev) cudaEventCreate(&e);
      cudaGraph_t g = nullptr;
      if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        c->stream = saved;
        return set_error(c, DI_ECUDA, "profile: capture");
      }
      int r = DI_OK;
      // External records become event-record nodes of the captured graph (plain records inside a
      // capture only express dependencies).
      cudaEventRecordWithFlags(pev[0], stream, cudaEventRecordExternal);
      for (size_t i = 0; i < ops.size() && r == DI_OK; ++i) {
        r = ops[i]();
        cudaEventRecordWithFlags(pev[i + 1], stream, cudaEventRecordExternal);
      }
      join_all();
      cudaError_t e = cudaStreamEndCapture(stream, &g);
      if (r != DI_OK || e != cudaSuccess || cudaGraphInstantiate(&pexec, g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        c->stream = saved;
        cudaGetLastError();
        return set_error(c, DI_ECUDA, "profile: graph");
      }
      cudaGraphDestroy(g);
    }
    std::vector<double> acc(ops.size(), 0.0);
    for (int rep = 0; rep < reps; ++rep) {
      cudaGraphLaunch(pexec, stream);
      cudaStreamSynchronize(stream);
      for (size_t i = 0; i < ops.size(); ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, pev[i], pev[i + 1]);
        acc[i] += ms;
      }
    }
    c->stream = saved;
    if (cudaGetLastError() != cudaSuccess) return set_error(c, DI_ECUDA, "profile: replay");
    for (size_t i = 0; i < ops.size(); ++i) op_ms[i] = (float)(acc[i] / std::max(1, reps));
    return DI_OK;
  }

  int run_ops() {
    if (stats_off) cudaMemsetAsync(stats_base, 0, stats_off * sizeof(long long), c->stream);
    for (auto& f : ops) {
      int r = f();
      if (r) {
        join_all();
        return r;
      }
    }
    join_all();
    return DI_OK;
  }

  // Enqueue one forward on the plan's stream, ordered after / before the context stream.
  int forward() {
    if (err) return err;
    if (const char* e = getenv("DI_PLAN_LIMIT")) {  // diagnostics: run only the first k ops, eagerly
      const size_t k = std::min<size_t>(ops.size(), (size_t)std::max(0, atoi(e)));
      int r = DI_OK;
      for (size_t i = 0; i < k && r == DI_OK; ++i) r = ops[i]();
      join_all();
      if (r) return r;
      return cudaStreamSynchronize(c->stream) == cudaSuccess ? DI_OK : DI_ECUDA;
    }
    cudaEventRecord(ev_in, c->stream);
    cudaStreamWaitEvent(stream, ev_in, 0);
    cudaStream_t saved = c->stream;
    c->stream = stream;
    int r = DI_OK;
    if (!gexec) {
      // One eager pass first: it validates every launch outside capture and performs the one-time
      // per-kernel attribute set-up, so the captured pass issues kernel launches only.
      r = run_ops();
      if (r == DI_OK && cudaStreamSynchronize(stream) != cudaSuccess) r = set_error(c, DI_ECUDA, "plan: eager pass");
      if (r != DI_OK) {
        c->stream = saved;
        return r;
      }
      cudaGraph_t g = nullptr;
      if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        c->stream = saved;
        return set_error(c, DI_ECUDA, "plan: begin capture failed");
      }
      r = run_ops();
      cudaError_t e = cudaStreamEndCapture(stream, &g);
      if (r == DI_OK && e == cudaSuccess) {
        if (cudaGraphInstantiate(&gexec, g, 0) != cudaSuccess) r = set_error(c, DI_ECUDA, "plan: instantiate");
      } else if (r == DI_OK) {
        r = set_error(c, DI_ECUDA, std::string("plan: capture failed: ") + cudaGetErrorString(e));
      }
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
    }
    if (r == DI_OK && cudaGraphLaunch(gexec, stream) != cudaSuccess) r = set_error(c, DI_ECUDA, "plan: graph launch");
    c->stream = saved;
    cudaEventRecord(ev_out, stream);
    cudaStreamWaitEvent(c->stream, ev_out, 0);
    return r;
  }

  bool init(Ctx* ctx, uint64_t sd, WeightFn f, void* u, size_t tmp_bytes) {
    c = ctx;
    seed = sd;
    wfn = f;
    wuser = u;
    if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) return false;
    cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
    splitk = dalloc(kSplitKBytes);
    tmp_cap = tmp_bytes;
    tmp_base = static_cast<char*>(dalloc(tmp_bytes));
    act_bytes += tmp_bytes;
    return tmp_base != nullptr;
  }

  // ---------------------------------------------------------------------------------------------
  // Layer builders (parameter names follow diffusers' UNet2DConditionModel).
  // ---------------------------------------------------------------------------------------------
  // 3x3 conv weight packed [Co][ky][kx][Cin_padded]; input channels beyond Ci are zero.
  const void* conv_weight(const std::string& name, int Co, int Ci, int Cip, int Cop) {
    auto w = host_param(name, (size_t)Co * Ci * 9, 0, Ci * 9, Co * 9);
    std::vector<float> pk((size_t)Cop * 9 * Cip, 0.0f);
    par_for((size_t)Co, [&](size_t co) {
      for (int ci = 0; ci < Ci; ++ci)
        for (int t = 0; t < 9; ++t) pk[(co * 9 + t) * Cip + ci] = w[(co * Ci + ci) * 9 + t];
    });
    return upload_f16(pk);
  }
  const float* bias_padded(const std::string& name, int Co, int Cop, int fan_in) {
    auto b = host_param(name, Co, 0, fan_in);
    round_f16(b);
    b.resize(Cop, 0.0f);
    return upload_f32(b);
  }

  // Chain plans (the VAE decoder: every op reads only its immediate input) take activations from a ring
  // of `act_ring` buffers instead of one allocation each.
  std::vector<void*> act_ring;
  size_t act_ring_bytes = 0, act_ring_next = 0;
  Act new_act(int N, int H, int W, int C) {
    Act a;
    a.N = N; a.H = H; a.W = W; a.C = C;
    if (!act_ring.empty()) {
      if (a.bytes() > act_ring_bytes) {
        fail(DI_ENOMEM, "plan: activation ring too small");
        a.p = nullptr;
        return a;
      }
      a.p = act_ring[act_ring_next++ % act_ring.size()];
      return a;
    }
    a.p = act_alloc(a.bytes());
    return a;
  }

  Act conv3x3(const std::string& pre, const Act& x, int Co, int stride, const Act* x2 = nullptr) {
    const int Ci = x.C + (x2 ? x2->C : 0);
    const void* w = conv_weight(pre + ".weight", Co, Ci, Ci, Co);
    const float* b = bias_padded(pre + ".bias", Co, Co, Ci * 9);
    Act y = new_act(x.N, x.H / stride, x.W / stride, Co);
    y.st = new_stat_slot();
    Ctx* cc = c;
    const Act xx = x;
    const void* p2 = x2 ? x2->p : nullptr;
    const int C2 = x2 ? x2->C : 0;
    void* sk = splitk;
    record([=] {
      return with_stats(cc, y.st, y.H * y.W, [&] {
        return gemm_conv3x3(cc, DI_F16, xx.p, xx.C, p2, C2, xx.N, xx.H, xx.W, stride, w, Co, b, nullptr, nullptr, 0,
                            y.p, 0, Co, sk);
      });
    },
           0, 2.0 * y.N * y.H * y.W * Co * 9 * Ci, (double)x.bytes() + 18.0 * Co * Ci + (double)y.bytes(), gemm_kernel_count(c, y.N * y.H * y.W, Co, 9 * Ci, 0));
    return y;
  }

  Act upsample(const Act& x) {
    Act y = new_act(x.N, x.H * 2, x.W * 2, x.C);
    Ctx* cc = c;
    const Act xx = x;
    record([=] {
      const size_t total = (size_t)xx.N * 4 * xx.H * xx.W * (xx.C / 8);
      launch_k(upsample2_kernel, (int)std::min<size_t>((total + 255) / 256, 16 * cc->num_sms), 256, 0, cc->stream,
          static_cast<const uint4*>(xx.p), static_cast<uint4*>(y.p), xx.N, xx.H, xx.W, xx.C / 8);
      return check_launch(cc, "upsample2");
    }, 3, 0, 5.0 * x.bytes());
    return y;
  }

  // GroupNorm statistics of concat(x1, x2) as a per-(image, channel) affine table for a consumer GEMM
  // that normalises its operand as it loads it (GnFuse): no normalised tensor is written.
  const float2* gn_tab(const std::string& pre, const Act& x1, const Act* x2, float eps) {
    const int C = x1.C + (x2 ? x2->C : 0), HW = x1.H * x1.W;
    const float* g = vec(pre + ".weight", C, 1, 1);
    const float* b = vec(pre + ".bias", C, 2, 1);
    float2* tab = static_cast<float2*>(tmp(sizeof(float2) * (size_t)x1.N * C));
    Ctx* cc = c;
    const Act a = x1;
    const void* p2 = x2 ? x2->p : nullptr;
    const int C2 = x2 ? x2->C : 0;
    record([=] { return gn_table_nhwc(cc, DI_F16, a.p, a.C, p2, C2, a.N, HW, 32, eps, g, b, tab); }, 2, 0,
           (double)x1.N * HW * C * 2, 1);
    return tab;
  }

  // A consumer GEMM's view of GroupNorm(+SiLU)(concat(x1, x2)).  gn_mode 0: two-pass GroupNorm into a
  // temporary (per-chunk partials); 1: cluster statistics table + elementwise normalise into a
  // temporary; 2: statistics table only, the consumer normalises its operand as it loads it (GnFuse).
  struct GnOp {
    const void* x1;
    int C1;
    const void* x2;
    int C2;
    const float2* tab;  // non-null: fused (raw inputs above)
    int silu;
  };
  int gn_mode = [] {  // diagnostics: DI_GN_MODE selects the GroupNorm strategy
    const char* e = getenv("DI_GN_MODE");
    return (e && e[0] >= '0' && e[0] <= '2') ? e[0] - '0' : 1;
  }();
  // DI_GN_STATS=1: GroupNorm statistics from the producing GEMM's epilogue (exact fixed-point atomics)
  // instead of a statistics kernel.  Off by default: measured slower on B200 at batch 1 (208 vs 233
  // steps/s) and at batch 64 (177 vs 183 images/s); the epilogue and split-K reduce work it adds
  // outweighs the launch it removes.
  bool use_stats = [] {
    const char* e = getenv("DI_GN_STATS");
    return e && e[0] == '1';
  }();
  GnOp gn_op(const std::string& pre, const Act& x1, const Act* x2, float eps, int silu) {
    const int C = x1.C + (x2 ? x2->C : 0);
    if (use_stats && gn_mode == 1 && !x2 && x1.st && C % 32 == 0 && C >= 256 && (x1.H * x1.W) % 32 == 0) {
      // statistics from the producer GEMM's epilogue: one normalising pass, no statistics kernel
      if (!x1.st->ptr) x1.st->ptr = stats_alloc(x1.N);
      const int HW = x1.H * x1.W;
      const float* g = vec(pre + ".weight", C, 1, 1);
      const float* b = vec(pre + ".bias", C, 2, 1);
      void* y = tmp((size_t)x1.N * HW * C * 2);
      Ctx* cc = c;
      const Act a = x1;
      const long long* st = x1.st->ptr;
      record([=] { return gn_apply_with_stats(cc, a.p, C, a.N, HW, st, eps, g, b, silu, y); }, 2, 0,
             2.0 * x1.N * HW * C * 2, 1);
      return GnOp{y, C, nullptr, 0, nullptr, 0};
    }
    if (gn_mode == 2) return GnOp{x1.p, x1.C, x2 ? x2->p : nullptr, x2 ? x2->C : 0, gn_tab(pre, x1, x2, eps), silu};
    // mode 0 also for large tensors: its statistics pass spreads each image over up to 128 CTAs, the
    // table path over one 16-CTA cluster (latency-optimal for the U-Net's small maps only)
    const size_t tensor_bytes = (size_t)x1.N * x1.H * x1.W * C * 2;
    if (gn_mode == 0 || tensor_bytes > (16u << 20)) return GnOp{gn(pre, x1, x2, eps, silu), C, nullptr, 0, nullptr, 0};
    const int HW = x1.H * x1.W;
    const float* g = vec(pre + ".weight", C, 1, 1);
    const float* b = vec(pre + ".bias", C, 2, 1);
    void* y = tmp((size_t)x1.N * HW * C * 2);
    if (gn_cluster_usable(DI_F16, HW, x1.C, x2 ? x2->C : 0, 32)) {
      // one launch per image cluster: slice in shared memory, statistics folded through DSMEM
      Ctx* cc = c;
      const Act a = x1;
      const void* p2 = x2 ? x2->p : nullptr;
      const int C2 = x2 ? x2->C : 0;
      record([=] {
        const int r = gn_nhwc_cluster_launch(cc, DI_F16, a.p, a.C, p2, C2, a.N, HW, 32, eps, g, b, silu, y);
        return r == 1 ? set_error(cc, DI_EUNSUPPORTED, "gn_nhwc_cluster: shape or alignment no longer accepted") : r;
      }, 2, 0, 2.0 * x1.N * HW * C * 2, 1);
      return GnOp{y, C, nullptr, 0, nullptr, 0};
    }
    if (gn_grid_usable(c, DI_F16, x1.N, HW, x1.C, x2 ? x2->C : 0, 32)) {
      // one launch: statistics, grid barrier and normalise (gn_nhwc_grid; opt-in, DI_GN_GRID=1)
      float2* part = static_cast<float2*>(tmp(gn_grid_ws_bytes(c, x1.N, HW, C, 32)));
      unsigned* bar = gn_bar_alloc();
      Ctx* cc = c;
      const Act a = x1;
      const void* p2 = x2 ? x2->p : nullptr;
      const int C2 = x2 ? x2->C : 0;
      record([=] {
        const int r = gn_nhwc_grid_launch(cc, DI_F16, a.p, a.C, p2, C2, a.N, HW, 32, eps, g, b, silu, y, part, bar);
        return r == 1 ? set_error(cc, DI_EUNSUPPORTED, "gn_nhwc_grid: shape or alignment no longer accepted") : r;
      }, 2, 0, 2.0 * x1.N * HW * C * 2, 1);
      return GnOp{y, C, nullptr, 0, nullptr, 0};
    }
    float2* tab = static_cast<float2*>(tmp(sizeof(float2) * (size_t)x1.N * C));
    Ctx* cc = c;
    const Act a = x1;
    const void* p2 = x2 ? x2->p : nullptr;
    const int C2 = x2 ? x2->C : 0;
    record([=] { return gn_nhwc_via_table(cc, DI_F16, a.p, a.C, p2, C2, a.N, HW, 32, eps, g, b, silu, y, tab); }, 2, 0,
           3.0 * x1.N * HW * C * 2, 2);
    return GnOp{y, C, nullptr, 0, nullptr, 0};
  }

  // GroupNorm(+SiLU) of concat(x1, x2) into a temporary.
  void* gn(const std::string& pre, const Act& x1, const Act* x2, float eps, int silu) {
    const int C = x1.C + (x2 ? x2->C : 0), HW = x1.H * x1.W;
    const float* g = vec(pre + ".weight", C, 1, 1);
    const float* b = vec(pre + ".bias", C, 2, 1);
    void* y = tmp((size_t)x1.N * HW * C * 2);
    void* part = tmp(gn_nhwc_ws_bytes(x1.N, HW, 32));
    Ctx* cc = c;
    const Act a = x1;
    const void* p2 = x2 ? x2->p : nullptr;
    const int C2 = x2 ? x2->C : 0;
    record([=] { return group_norm_nhwc(cc, DI_F16, DI_F16, a.p, a.C, p2, C2, a.N, HW, 32, eps, g, b, silu, y,
                                        part); },
           2, 0, 3.0 * x1.N * HW * C * 2, 2);
    return y;
  }

  // Linear on token rows: Y[M, N] = X[M, K] W^T (+b) (+R).
  const void* lin_weight(const std::string& name, int N, int K) {
    return upload_f16(host_param(name, (size_t)N * K, 0, K, N));
  }
  void linear(const void* X, int M, int K, const void* W, int N, const float* b, const void* R, void* Y,
              const void* X2 = nullptr, int K1 = 0, const float2* gtab = nullptr, int gsilu = 0, int ghw = 0,
              const GnStatSlot* st = nullptr, int st_hw = 0) {
    Ctx* cc = c;
    void* sk = splitk;
    record([=] {
      const GnFuse f{gtab, gsilu};
      return with_stats(cc, st, st_hw, [&] {
        return gemm_linear(cc, DI_F16, X, X2 ? K1 : K, X2, M, K, W, N, b, R, 0, Y, 0, 0, nullptr, 1, sk,
                           gtab ? &f : nullptr, ghw);
      });
    },
           0, 2.0 * M * N * K, 2.0 * ((double)M * K + (double)N * K + (double)M * N * (R ? 2 : 1)), gemm_kernel_count(c, M, N, K, 0));
  }

  // ResnetBlock2D on concat(x1, x2): gn1+silu -> conv1 (+b1 +time proj) -> gn2+silu -> conv2 (+b2 + shortcut).
  struct TimeSlice { int off, C; };
  std::vector<float> tproj_w, tproj_b;  // concatenated time projections (host staging)
  int tproj_rows = 0;
  float* temb_all = nullptr;            // [B, tproj_rows] fp32, computed once per forward
  int tproj_ld = 0;

  Act resnet(const std::string& pre, const Act& x1, const Act* x2, int Co, float eps = 1e-5f, bool temb = true) {
    tmp_reset();
    const int Ci = x1.C + (x2 ? x2->C : 0);
    // 1x1 shortcut when the channel count changes: it reads only the block input, so it runs on the side
    // branch while gn1 -> conv1 -> gn2 run on the main chain; conv2 joins it for the residual add
    const void* res = x1.p;
    int fork = -1;
    static const bool fork_ok = [] {  // diagnostics: DI_PLAN_FORK=0 keeps the shortcut on the main chain
      const char* e = getenv("DI_PLAN_FORK");
      return !(e && e[0] == '0');
    }();
    if (Ci != Co && !fork_ok) {
      const void* ws = lin_weight(pre + ".conv_shortcut.weight", Co, Ci);
      const float* bs = vec(pre + ".conv_shortcut.bias", Co, 0, Ci);
      void* s = tmp((size_t)x1.N * x1.H * x1.W * Co * 2);
      linear(x1.p, x1.N * x1.H * x1.W, Ci, ws, Co, bs, nullptr, s, x2 ? x2->p : nullptr, x1.C);
      res = s;
    } else if (Ci != Co) {
      const void* ws = lin_weight(pre + ".conv_shortcut.weight", Co, Ci);
      const float* bs = vec(pre + ".conv_shortcut.bias", Co, 0, Ci);
      const int M = x1.N * x1.H * x1.W;
      void* s = tmp((size_t)M * Co * 2);
      Ctx* cc = c;
      Plan* self = this;
      const void* xa = x1.p;
      const void* xb = x2 ? x2->p : nullptr;
      const int K1 = x1.C;
      fork = record_fork([=] {
        return gemm_linear(cc, DI_F16, xa, xb ? K1 : Ci, xb, M, Ci, ws, Co, bs, nullptr, 0, s, 0, 0, nullptr, 1,
                           self->splitk_side);
      }, 0, 2.0 * M * Co * Ci, 2.0 * ((double)M * Ci + (double)Co * Ci + (double)M * Co), gemm_kernel_count(c, M, Co, Ci, 0));
      res = s;
    }
    const GnOp g1 = gn_op(pre + ".norm1", x1, x2, eps, 1);
    // time projection rows appended to the shared GEMV
    if (temb) {
      auto w = host_param(pre + ".time_emb_proj.weight", (size_t)Co * 1280, 0, 1280, Co);
      auto b = host_param(pre + ".time_emb_proj.bias", Co, 0, 1280);
      round_f16(w);
      round_f16(b);
      tproj_w.insert(tproj_w.end(), w.begin(), w.end());
      tproj_b.insert(tproj_b.end(), b.begin(), b.end());
    }
    const int toff = tproj_rows;
    if (temb) tproj_rows += Co;
    const bool join_temb = temb && !temb_seen;  // the first reader of the time projections
    if (temb) temb_seen = true;
    const void* w1 = conv_weight(pre + ".conv1.weight", Co, Ci, Ci, Co);
    const float* b1 = bias_padded(pre + ".conv1.bias", Co, Co, Ci * 9);
    Act h;
    h.N = x1.N; h.H = x1.H; h.W = x1.W; h.C = Co;
    h.p = tmp(h.bytes());
    h.st = new_stat_slot();
    Ctx* cc = c;
    const int N = x1.N, H = x1.H, W = x1.W;
    Plan* self = this;
    void* sk = splitk;
    record([=] {
      if (join_temb) self->join(self->temb_fork);
      const GnFuse f{g1.tab, g1.silu};
      return with_stats(cc, h.st, H * W, [&] {
        return gemm_conv3x3(cc, DI_F16, g1.x1, g1.C1, g1.x2, g1.C2, N, H, W, 1, w1, Co, b1,
                            temb ? self->temb_all + toff : nullptr, nullptr, 0, h.p, 0, self->tproj_ld, sk,
                            g1.tab ? &f : nullptr);
      });
    },
           0, 2.0 * N * H * W * Co * 9 * Ci, 2.0 * ((double)N * H * W * (Ci + Co) + 9.0 * Co * Ci), gemm_kernel_count(c, N * H * W, Co, 9 * Ci, 0));
    const GnOp g2 = gn_op(pre + ".norm2", h, nullptr, eps, 1);
    const void* w2 = conv_weight(pre + ".conv2.weight", Co, Co, Co, Co);
    const float* b2 = bias_padded(pre + ".conv2.bias", Co, Co, Co * 9);
    Act y = new_act(N, H, W, Co);
    y.st = new_stat_slot();
    record([=] {
      self->join(fork);
      const GnFuse f{g2.tab, g2.silu};
      return with_stats(cc, y.st, H * W, [&] {
        return gemm_conv3x3(cc, DI_F16, g2.x1, g2.C1, g2.x2, g2.C2, N, H, W, 1, w2, Co, b2, nullptr, res, 0, y.p, 0,
                            Co, sk, g2.tab ? &f : nullptr);
      });
    },
           0, 2.0 * N * H * W * Co * 9 * Co, 2.0 * ((double)N * H * W * 3 * Co + 9.0 * Co * Co), gemm_kernel_count(c, N * H * W, Co, 9 * Co, 0));
    return y;
  }

  // Transformer2DModel (linear proj_in/out) + BasicTransformerBlock; ctx16 = [N, Sk, Cctx] fp16.
  // LayerNorm(x) . W^T + b as one GEMM on the raw rows x (the GEMM folds the normalisation, Ctx::ln_c1):
  // W'[n][k] = f16(f16(W[n][k]) * gamma[k]), c1[n] = sum_k W'[n][k], b'[n] = b[n] + sum_k f16(W[n][k]) * beta[k].
  // y = rstd * (x . W'^T - mean * c1) + b' is LayerNorm(x) . W^T + b with the LayerNorm output kept in fp32.
  // Opt-in (DI_LN_FOLD=1): parity-green, but measured slower in the step (236.8 vs 263.7 steps/s, one-wave
  // GEMMs only; 227.3 when folded everywhere) than the separate LayerNorm kernel.
  bool ln_fold_on = [] {
    const char* e = getenv("DI_LN_FOLD");
    return e && e[0] == '1';
  }();
  struct LnFold { const void* W; const float* c1; const float* b; };
  LnFold ln_fold(std::vector<float> W, const std::vector<float>* bias, int N, int K, const std::string& norm) {
    auto g = host_param(norm + ".weight", K, 1, 1);
    auto be = host_param(norm + ".bias", K, 2, 1);
    round_f16(g);
    round_f16(be);
    round_f16(W);
    std::vector<float> wp(W.size()), c1(N), b2(N);
    for (int n = 0; n < N; ++n) {
      double bs = bias ? (*bias)[n] : 0.0;
      for (int k = 0; k < K; ++k) {
        const float w = W[(size_t)n * K + k];
        wp[(size_t)n * K + k] = w * g[k];
        bs += (double)w * be[k];
      }
      b2[n] = (float)bs;
    }
    round_f16(wp);
    for (int n = 0; n < N; ++n) {
      double cs = 0.0;
      for (int k = 0; k < K; ++k) cs += wp[(size_t)n * K + k];
      c1[n] = (float)cs;
    }
    return LnFold{upload_f16(wp), upload_f32(c1), upload_f32(b2)};
  }
  // The fold pays only when the GEMM runs as one tile per CTA (BN = 256 bound); otherwise the plan keeps the
  // LayerNorm kernel.
  bool ln_fits(int M, int N) const { return (long long)((M + 127) / 128) * ((N + 255) / 256) <= c->num_sms; }
  void linear_ln(const void* X, int M, int K, const LnFold& f, int N, void* Y, int geglu) {
    Ctx* cc = c;
    void* sk = splitk;
    record([=] {
      cc->ln_c1 = f.c1;
      cc->ln_eps = 1e-5f;
      const int r = gemm_linear(cc, DI_F16, X, K, nullptr, M, K, f.W, N, f.b, nullptr, 0, Y, 0, geglu, nullptr, 1, sk,
                                nullptr, 0, 0);
      cc->ln_c1 = nullptr;
      return r;
    }, 0, 2.0 * M * N * K, 2.0 * ((double)M * K + (double)N * K + (double)M * (geglu ? N / 2 : N)), 1);
  }

  Act transformer(const std::string& pre, const Act& x, const void* ctx16, int Sk, int Cctx) {
    tmp_reset();
    const int N = x.N, HW = x.H * x.W, C = x.C, M = N * HW, heads = C / 64;
    const std::string tb = pre + ".transformer_blocks.0";
    const GnOp gx = gn_op(pre + ".norm", x, nullptr, 1e-6f, 0);
    const void* wpi = lin_weight(pre + ".proj_in.weight", C, C);
    const float* bpi = vec(pre + ".proj_in.bias", C, 0, C);
    void* h0 = tmp((size_t)M * C * 2);
    linear(gx.x1, M, C, wpi, C, bpi, nullptr, h0, nullptr, 0, gx.tab, 0, HW);
    Ctx* cc = c;
    // --- self attention ---
    const float* g1 = vec(tb + ".norm1.weight", C, 1, 1);
    const float* be1 = vec(tb + ".norm1.bias", C, 2, 1);
    std::vector<float> wqkv;
    for (const char* nm : {".attn1.to_q.weight", ".attn1.to_k.weight", ".attn1.to_v.weight"}) {
      auto w = host_param(tb + nm, (size_t)C * C, 0, C, C);
      wqkv.insert(wqkv.end(), w.begin(), w.end());
    }
    void* qkv = tmp((size_t)M * 3 * C * 2);
    if (ln_fold_on && ln_fits(M, 3 * C)) {
      linear_ln(h0, M, C, ln_fold(wqkv, nullptr, 3 * C, C, tb + ".norm1"), 3 * C, qkv, 0);
    } else {
      void* n1 = tmp((size_t)M * C * 2);
      record([=] { return layer_norm(cc, DI_F16, DI_F16, h0, g1, be1, n1, M, C, 1e-5f); }, 2, 0, 4.0 * M * C);
      linear(n1, M, C, upload_f16(wqkv), 3 * C, nullptr, nullptr, qkv);
    }
    void* o1 = tmp((size_t)M * C * 2);
    record([=] {
      const char* base = static_cast<const char*>(qkv);
      return attention(cc, DI_F16, base, base + (size_t)C * 2, base + (size_t)2 * C * 2, o1, N, heads, HW, HW, 0,
                       3 * C, 3 * C, 3 * C, C);
    }, 1, 4.0 * N * heads * HW * (double)HW * 64, 2.0 * 4 * M * C);
    const void* wo1 = lin_weight(tb + ".attn1.to_out.0.weight", C, C);
    const float* bo1 = vec(tb + ".attn1.to_out.0.bias", C, 0, C);
    void* h1 = tmp((size_t)M * C * 2);
    linear(o1, M, C, wo1, C, bo1, h0, h1);
    // --- cross attention ---
    const float* g2 = vec(tb + ".norm2.weight", C, 1, 1);
    const float* be2 = vec(tb + ".norm2.bias", C, 2, 1);
    void* q2 = tmp((size_t)M * C * 2);
    if (ln_fold_on && ln_fits(M, C)) {
      linear_ln(h1, M, C, ln_fold(host_param(tb + ".attn2.to_q.weight", (size_t)C * C, 0, C, C), nullptr, C, C,
                                  tb + ".norm2"), C, q2, 0);
    } else {
      void* n2 = tmp((size_t)M * C * 2);
      record([=] { return layer_norm(cc, DI_F16, DI_F16, h1, g2, be2, n2, M, C, 1e-5f); }, 2, 0, 4.0 * M * C);
      const void* wq2 = lin_weight(tb + ".attn2.to_q.weight", C, C);
      linear(n2, M, C, wq2, C, nullptr, nullptr, q2);
    }
    std::vector<float> wkv;
    for (const char* nm : {".attn2.to_k.weight", ".attn2.to_v.weight"}) {
      auto w = host_param(tb + nm, (size_t)C * Cctx, 0, Cctx, C);
      wkv.insert(wkv.end(), w.begin(), w.end());
    }
    void* o2 = tmp((size_t)M * C * 2);
    if (batch_ctx_kv) {
      // K / V rows appended to the plan's single context projection (finish_ctx_kv); this block reads its
      // columns [off, off + 2C) of the [N*Sk, ctxkv_rows] result
      const int off = ctxkv_rows;
      ctxkv_w.insert(ctxkv_w.end(), wkv.begin(), wkv.end());
      ctxkv_rows += 2 * C;
      Plan* self = this;
      const bool join_ctx = !ctx_seen;  // the first reader of the context projection
      ctx_seen = true;
      record([=] {
        if (join_ctx) self->join(self->ctx_fork);
        const __half* base = self->ctxkv + off;
        const long long ld = self->ctxkv_rows;
        return attention(cc, DI_F16, q2, base, base + C, o2, N, heads, HW, Sk, 0, C, ld, ld, C);
      }, 1, 4.0 * N * heads * HW * (double)Sk * 64, 2.0 * (2.0 * M * C + 2.0 * N * Sk * C));
    } else {
      const void* Wkv = upload_f16(wkv);
      void* kv = tmp((size_t)N * Sk * 2 * C * 2);
      linear(ctx16, N * Sk, Cctx, Wkv, 2 * C, nullptr, nullptr, kv);
      record([=] {
        const char* base = static_cast<const char*>(kv);
        return attention(cc, DI_F16, q2, base, base + (size_t)C * 2, o2, N, heads, HW, Sk, 0, C, 2 * C, 2 * C, C);
      }, 1, 4.0 * N * heads * HW * (double)Sk * 64, 2.0 * (2.0 * M * C + 2.0 * N * Sk * C));
    }
    const void* wo2 = lin_weight(tb + ".attn2.to_out.0.weight", C, C);
    const float* bo2 = vec(tb + ".attn2.to_out.0.bias", C, 0, C);
    void* h2 = tmp((size_t)M * C * 2);
    linear(o2, M, C, wo2, C, bo2, h1, h2);
    // --- GEGLU feed-forward ---
    const float* g3 = vec(tb + ".norm3.weight", C, 1, 1);
    const float* be3 = vec(tb + ".norm3.bias", C, 2, 1);
    const int F = 4 * C;
    auto wff = host_param(tb + ".ff.net.0.proj.weight", (size_t)2 * F * C, 0, C, 2 * F);
    auto bff = host_param(tb + ".ff.net.0.proj.bias", (size_t)2 * F, 0, C);
    round_f16(bff);
    std::vector<float> wp((size_t)2 * F * C), bp(2 * F);
    for (int t = 0; t < F / 64; ++t) {
      for (int r = 0; r < 64; ++r) {
        std::memcpy(&wp[(size_t)(128 * t + r) * C], &wff[(size_t)(64 * t + r) * C], sizeof(float) * C);
        std::memcpy(&wp[(size_t)(128 * t + 64 + r) * C], &wff[(size_t)(F + 64 * t + r) * C], sizeof(float) * C);
        bp[128 * t + r] = bff[64 * t + r];
        bp[128 * t + 64 + r] = bff[F + 64 * t + r];
      }
    }
    void* g = tmp((size_t)M * F * 2);
    if (ln_fold_on && ln_fits(M, 2 * 4 * C)) {
      linear_ln(h2, M, C, ln_fold(wp, &bp, 2 * F, C, tb + ".norm3"), 2 * F, g, 1);
    } else {
      void* n3 = tmp((size_t)M * C * 2);
      record([=] { return layer_norm(cc, DI_F16, DI_F16, h2, g3, be3, n3, M, C, 1e-5f); }, 2, 0, 4.0 * M * C);
      const void* Wff = upload_f16(wp);
      const float* Bff = upload_f32(bp);
      record([=] { return gemm_linear(cc, DI_F16, n3, C, nullptr, M, C, Wff, 2 * F, Bff, nullptr, 0, g, 0, 1, nullptr,
                                      1, splitk); },
             0, 2.0 * M * 2 * F * C, 2.0 * ((double)M * C + 2.0 * F * C + (double)M * F), gemm_kernel_count(c, M, 2 * F, C, 1));
    }
    const void* wf2 = lin_weight(tb + ".ff.net.2.weight", C, F);
    const float* bf2 = vec(tb + ".ff.net.2.bias", C, 0, F);
    void* h3 = tmp((size_t)M * C * 2);
    linear(g, M, F, wf2, C, bf2, h2, h3);
    // --- proj_out + block residual ---
    const void* wpo = lin_weight(pre + ".proj_out.weight", C, C);
    const float* bpo = vec(pre + ".proj_out.bias", C, 0, C);
    Act y = new_act(N, x.H, x.W, C);
    y.st = new_stat_slot();
    linear(h3, M, C, wpo, C, bpo, x.p, y.p, nullptr, 0, nullptr, 0, 0, y.st, HW);
    return y;
  }

  // Builds the time-projection GEMV once every ResNet block has appended its rows; `at` is the op
  // index it must run at (right after the timestep embedding).
  // The VAE's mid-block attention (diffusers Attention: GroupNorm(32, 1e-6), one head of C channels,
  // biased q / k / v / out projections, residual).  Per image: S = q k^T (the 1/sqrt(C) scale folded into
  // the query projection), an fp16 row softmax, O = P V with V^T = Wv a^T from one GEMM (the v bias is
  // folded into the out-projection bias: softmax rows sum to one), then out-projection + residual.
  Act vae_attention(const std::string& pre, const Act& x) {
    tmp_reset();
    const int N = x.N, HW = x.H * x.W, C = x.C, M = N * HW;
    if (HW % 64 || C % 64) {
      fail(DI_EUNSUPPORTED, "vae attention: H*W and C must be multiples of 64");
      return x;
    }
    const int saved_mode = gn_mode;
    gn_mode = 1;  // V^T = Wv a^T takes the normalised activations as its B operand: materialise them
    const GnOp g = gn_op(pre + ".group_norm", x, nullptr, 1e-6f, 0);
    gn_mode = saved_mode;
    const float scale = 1.0f / std::sqrt((float)C);
    auto wq = host_param(pre + ".to_q.weight", (size_t)C * C, 0, C, C);
    auto bq = host_param(pre + ".to_q.bias", C, 0, C);
    round_f16(wq);
    round_f16(bq);
    for (auto& v : wq) v *= scale;
    for (auto& v : bq) v *= scale;
    const void* Wq = upload_f16(wq);
    const float* Bq = upload_f32(bq);
    const void* Wk = lin_weight(pre + ".to_k.weight", C, C);
    const float* Bk = vec(pre + ".to_k.bias", C, 0, C);
    auto wv = host_param(pre + ".to_v.weight", (size_t)C * C, 0, C, C);
    auto bv = host_param(pre + ".to_v.bias", C, 0, C);
    auto wo = host_param(pre + ".to_out.0.weight", (size_t)C * C, 0, C, C);
    auto bo = host_param(pre + ".to_out.0.bias", C, 0, C);
    round_f16(wv);
    round_f16(bv);
    round_f16(wo);
    round_f16(bo);
    for (int o = 0; o < C; ++o) {  // bo' = bo + Wo bv
      double acc = bo[o];
      for (int k = 0; k < C; ++k) acc += (double)wo[(size_t)o * C + k] * bv[k];
      bo[o] = (float)acc;
    }
    const void* Wv = upload_f16(wv);
    const void* Wo = upload_f16(wo);
    const float* Bo = upload_f32(bo);
    void* q = tmp((size_t)M * C * 2);
    void* k = tmp((size_t)M * C * 2);
    void* vt = tmp((size_t)C * HW * 2);
    void* sc = tmp((size_t)HW * HW * 2);
    void* o = tmp((size_t)M * C * 2);
    if (err) return x;
    linear(g.x1, M, C, Wq, C, Bq, nullptr, q, nullptr, 0, g.tab, 0, HW);
    linear(g.x1, M, C, Wk, C, Bk, nullptr, k, nullptr, 0, g.tab, 0, HW);
    Ctx* cc = c;
    void* sk = splitk;
    for (int n = 0; n < N; ++n) {
      const size_t off = (size_t)n * HW * C * 2;
      const char* qn = static_cast<const char*>(q) + off;
      const char* kn = static_cast<const char*>(k) + off;
      const char* an = static_cast<const char*>(g.x1) + off;
      char* on = static_cast<char*>(o) + off;
      const float2* tab = g.tab ? g.tab + (size_t)n * C : nullptr;
      // these three GEMMs take activations as their B operand: no weight-tile fetch before the dependency wait
      record([=] {
        cc->weights_const = false;
        return gemm_linear(cc, DI_F16, qn, C, nullptr, HW, C, kn, HW, nullptr, nullptr, 0, sc, 0, 0, nullptr, 1, sk);
      },
             1, 2.0 * HW * HW * C, 2.0 * (2.0 * HW * C + (double)HW * HW), gemm_kernel_count(cc, HW, HW, C, 0));
      record([=] {
        launch_k(softmax_rows_f16, HW, 256, 0, cc->stream, static_cast<__half*>(sc), HW);
        return check_launch(cc, "softmax_rows_f16");
      }, 1, 0, 4.0 * HW * HW);
      record([=] {
        cc->weights_const = false;
        const GnFuse f{tab, 0};
        return gemm_linear(cc, DI_F16, Wv, C, nullptr, C, C, an, HW, nullptr, nullptr, 0, vt, 0, 0, nullptr, 1, sk,
                           tab ? &f : nullptr, HW);
      }, 0, 2.0 * C * HW * C, 2.0 * (2.0 * C * C + (double)HW * C), gemm_kernel_count(cc, C, HW, C, 0));
      record([=] {
        cc->weights_const = false;
        return gemm_linear(cc, DI_F16, sc, HW, nullptr, HW, HW, vt, C, nullptr, nullptr, 0, on, 0, 0, nullptr, 1, sk);
      },
             1, 2.0 * HW * HW * C, 2.0 * ((double)HW * HW + 2.0 * C * HW), gemm_kernel_count(cc, HW, C, HW, 0));
    }
    Act y = new_act(N, x.H, x.W, C);
    linear(o, M, C, Wo, C, Bo, x.p, y.p);
    return y;
  }

  // Cross-attention K / V of every transformer from one GEMM over the (step-invariant) context:
  // [N*Sk, Cctx] x [ctxkv_rows, Cctx]^T, inserted as op `at`, instead of one small GEMM per block.
  bool batch_ctx_kv = false;
  std::vector<float> ctxkv_w;
  int ctxkv_rows = 0;
  __half* ctxkv = nullptr;
  // The step's prologue work whose results are needed only later (the time MLP and the ResNets' time
  // projections, first read by the first conv1 epilogue; the context K / V projection, first read by the
  // first cross-attention) runs on the side branch beside conv_in and the first GroupNorms / convs.
  // DI_PLAN_PREFORK=0 keeps it on the main chain (diagnostics).
  static bool prefork_ok() {
    static const bool on = [] {
      const char* e = getenv("DI_PLAN_PREFORK");
      return !(e && e[0] == '0');
    }();
    return on;
  }
  int temb_fork = -1, ctx_fork = -1;  // side branches joined by the first consumer (resnet / transformer)
  bool temb_seen = false, ctx_seen = false;

  // Inserts op `at`: the context K / V projection of every transformer block, one GEMM.
  void finish_ctx_kv(size_t at, const void* ctx16, int rows, int Cctx) {
    const void* W = upload_f16(ctxkv_w);
    ctxkv = static_cast<__half*>(act_alloc(sizeof(__half) * (size_t)rows * ctxkv_rows));
    Ctx* cc = c;
    const int N = ctxkv_rows;
    __half* out = ctxkv;
    const double flops = 2.0 * rows * N * Cctx;
    const double bytes = 2.0 * ((double)rows * Cctx + (double)N * Cctx + (double)rows * N);
    const int kern = gemm_kernel_count(c, rows, N, Cctx, 0);
    if (prefork_ok()) {
      Plan* self = this;
      ctx_fork = insert_fork(at, [=] {
        return gemm_linear(cc, DI_F16, ctx16, Cctx, nullptr, rows, Cctx, W, N, nullptr, nullptr, 0, out, 0, 0,
                           nullptr, 1, self->splitk_side);
      }, 0, flops, bytes, kern);
    } else {
      void* sk = splitk;
      info.insert(info.begin() + at, OpInfo{0, flops, bytes, kern});
      launches += kern;
      ops.insert(ops.begin() + at, [=] {
        cc->weights_const = true;
        const int r = gemm_linear(cc, DI_F16, ctx16, Cctx, nullptr, rows, Cctx, W, N, nullptr, nullptr, 0, out, 0, 0,
                                  nullptr, 1, sk);
        cc->weights_const = false;
        return r;
      });
    }
    ctxkv_w.clear();
    ctxkv_w.shrink_to_fit();
  }

  // Inserts op `at`: `pre` (the time MLP writing `temb`, `pre_kernels` launches) followed by one GEMV
  // computing every ResNet's time projection from it.
  void finish_time_proj(size_t at, const float* temb, int B, std::function<int()> pre, double pre_flops,
                        double pre_bytes, int pre_kernels) {
    const void* W = upload_f16(tproj_w);
    const float* b = upload_f32(tproj_b);
    temb_all = static_cast<float*>(act_alloc(sizeof(float) * (size_t)B * tproj_rows));
    tproj_ld = tproj_rows;
    Ctx* cc = c;
    const int rows = tproj_rows;
    float* out = temb_all;
    auto f = [=] {
      int r = pre();
      for (int b0 = 0; b0 < B && r == DI_OK; b0 += 8) {
        const int nb = std::min(8, B - b0);
        r = gemv(cc, temb + (size_t)b0 * 1280, nb, 1280, W, 1, b, rows, 1, out + (size_t)b0 * rows, rows);
      }
      return r;
    };
    const double flops = pre_flops + 2.0 * B * rows * 1280, bytes = pre_bytes + 2.0 * rows * 1280;
    const int kern = pre_kernels + (B + 7) / 8;
    if (prefork_ok()) {
      temb_fork = insert_fork(at, f, 3, flops, bytes, kern);
    } else {
      info.insert(info.begin() + at, OpInfo{3, flops, bytes, kern});
      ops.insert(ops.begin() + at, f);
      launches += kern;
    }
    tproj_w.clear();
    tproj_w.shrink_to_fit();
  }
};

// ---------------------------------------------------------------------------------------------
// The three plans.
// ---------------------------------------------------------------------------------------------
struct UNetPlan {
  Plan P;
  int B = 1, H = 64, W = 64, Sk = 77;
  float* latent = nullptr;  // [B,4,H,W] fp32 NCHW (input)
  float* tvals = nullptr;   // [B] fp32
  float* ctx32 = nullptr;   // [B,Sk,1024] fp32
  float* out = nullptr;     // [B,4,H,W] fp32 NCHW
  float* next = nullptr;    // [B,4,H,W] fp32 NCHW: the Euler step latent + dt * out
  double* sched = nullptr;  // device {scaleModelInput factor, sigma_{i+1} - sigma_i}; {1, 0} by default
  float* ext_ctx = nullptr; // when set before building: the text-encoder output used as ctx32
  double gflop = 0;
};

static size_t unet_tmp_bytes(int B, int H, int W) {
  // largest block working set: the 64x64 transformer (GEGLU hidden 4C plus QKV 3C and six C-wide temps)
  const size_t M = (size_t)B * H * W;
  return M * 320 * 2 * (16 + 3 + 8) + (size_t)B * 77 * 2 * 1280 * 2 + (64 << 20);
}

static int build_unet(UNetPlan* u) {
  Plan& P = u->P;
  const int B = u->B, H = u->H, W = u->W, Sk = u->Sk;
  Ctx* cc = P.c;
  void* sk = P.splitk;
  u->latent = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 4 * H * W));
  u->tvals = static_cast<float*>(P.act_alloc(sizeof(float) * B));
  u->ctx32 = u->ext_ctx ? u->ext_ctx : static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * Sk * 1024));
  u->out = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 4 * H * W));
  u->next = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 4 * H * W));
  u->sched = static_cast<double*>(P.act_alloc(2 * sizeof(double)));
  __half* ctx16 = static_cast<__half*>(P.act_alloc(sizeof(__half) * (size_t)B * Sk * 1024));
  if (P.err) return P.err;
  {
    const double s0[2] = {1.0, 0.0};
    cudaMemcpy(u->sched, s0, sizeof s0, cudaMemcpyHostToDevice);
  }
  const double* sched = u->sched;
  // inputs: ctx fp32 -> fp16, latent NCHW fp32 -> NHWC fp16 padded to 64 channels
  {
    const float* src = u->ctx32;
    const size_t n = (size_t)B * Sk * 1024;
    P.record([=] {
      launch_k(f32_to_f16_kernel, (int)std::min<size_t>((n + 255) / 256, 1024), 256, 0, cc->stream, src, ctx16, n);
      return check_launch(cc, "ctx_to_f16");
    }, 3, 0, 6.0 * n);
  }
  Act lat;
  lat.N = B; lat.H = H; lat.W = W; lat.C = 64;
  lat.p = P.act_alloc(lat.bytes());
  {
    const float* src = u->latent;
    void* dst = lat.p;
    P.record([=] {
      const size_t n = (size_t)B * H * W * 64;
      launch_k(latent_in_kernel, (int)std::min<size_t>((n + 255) / 256, 4096), 256, 0, cc->stream, 
          src, static_cast<__half*>(dst), B, 4, H * W, 64, sched);
      return check_launch(cc, "latent_in");
    }, 3, 0, (double)B * H * W * (16 + 128));
  }
  // timestep embedding (fp32 weights, fp16-rounded values)
  float* temb = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 1280));
  float* thid = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 1280));
  std::function<int()> temb_fn;
  {
    auto w1 = P.host_param("time_embedding.linear_1.weight", (size_t)1280 * 320, 0, 320, 1280);
    Plan::round_f16(w1);
    const float* W1 = P.upload_f32(w1);
    const float* b1 = P.vec("time_embedding.linear_1.bias", 1280, 0, 320);
    auto w2 = P.host_param("time_embedding.linear_2.weight", (size_t)1280 * 1280, 0, 1280, 1280);
    Plan::round_f16(w2);
    const float* W2 = P.upload_f32(w2);
    const float* b2 = P.vec("time_embedding.linear_2.bias", 1280, 0, 1280);
    const float* tv = u->tvals;
    // run, with the time projections, as one op (finish_time_proj) on the plan's side branch
    temb_fn = [=] {
      for (int b0 = 0; b0 < B; b0 += 8) {
        const int nb = std::min(8, B - b0);
        int r = tembed(cc, tv + b0, nb, W1, b1, W2, b2, 320, 1280, thid + (size_t)b0 * 1280, temb + (size_t)b0 * 1280);
        if (r) return r;
      }
      return DI_OK;
    };
  }
  const size_t tproj_at = P.ops.size();
  P.batch_ctx_kv = true;

  // conv_in: 4 (padded to 64) -> 320
  Act h;
  {
    const void* w = P.conv_weight("conv_in.weight", 320, 4, 64, 320);
    const float* b = P.bias_padded("conv_in.bias", 320, 320, 36);
    h = P.new_act(B, H, W, 320);
    h.st = P.new_stat_slot();
    const Act x = lat;
    const Act y = h;
    P.record([=] {
      return Plan::with_stats(cc, y.st, H * W, [&] {
        return gemm_conv3x3(cc, DI_F16, x.p, 64, nullptr, 0, B, H, W, 1, w, 320, b, nullptr, nullptr, 0, y.p, 0, 320,
                            sk);
      });
    },
             0, 2.0 * B * H * W * 320 * 9 * 4, (double)B * H * W * (128 + 640), gemm_kernel_count(cc, B * H * W, 320, 9 * 64, 0));
  }
  const int ch[4] = {320, 640, 1280, 1280};
  std::vector<Act> skips{h};
  for (int i = 0; i < 4; ++i) {
    const std::string pre = "down_blocks." + std::to_string(i);
    for (int j = 0; j < 2; ++j) {
      h = P.resnet(pre + ".resnets." + std::to_string(j), h, nullptr, ch[i]);
      if (i < 3) h = P.transformer(pre + ".attentions." + std::to_string(j), h, ctx16, Sk, 1024);
      skips.push_back(h);
    }
    if (i < 3) {
      P.tmp_reset();
      h = P.conv3x3(pre + ".downsamplers.0.conv", h, ch[i], 2);
      skips.push_back(h);
    }
  }
  h = P.resnet("mid_block.resnets.0", h, nullptr, 1280);
  h = P.transformer("mid_block.attentions.0", h, ctx16, Sk, 1024);
  h = P.resnet("mid_block.resnets.1", h, nullptr, 1280);
  const int rch[4] = {1280, 1280, 640, 320};
  for (int i = 0; i < 4; ++i) {
    const std::string pre = "up_blocks." + std::to_string(i);
    for (int j = 0; j < 3; ++j) {
      Act s = skips.back();
      skips.pop_back();
      h = P.resnet(pre + ".resnets." + std::to_string(j), h, &s, rch[i]);
      if (i > 0) h = P.transformer(pre + ".attentions." + std::to_string(j), h, ctx16, Sk, 1024);
    }
    if (i < 3) {
      P.tmp_reset();
      h = P.conv3x3(pre + ".upsamplers.0.conv", P.upsample(h), rch[i], 1);
    }
  }
  // conv_norm_out + SiLU, conv_out 320 -> 4 (padded to 16)
  P.tmp_reset();
  const Plan::GnOp go = P.gn_op("conv_norm_out", h, nullptr, 1e-5f, 1);
  {
    const void* w = P.conv_weight("conv_out.weight", 4, 320, 320, 16);
    const float* b = P.bias_padded("conv_out.bias", 4, 16, 320 * 9);
    void* y16 = P.act_alloc((size_t)B * H * W * 16 * 2);
    P.record([=] {
      const GnFuse f{go.tab, go.silu};
      return gemm_conv3x3(cc, DI_F16, go.x1, 320, nullptr, 0, B, H, W, 1, w, 16, b, nullptr, nullptr, 0, y16, 0, 16, sk,
                          go.tab ? &f : nullptr);
    },
             0, 2.0 * B * H * W * 4 * 9 * 320, (double)B * H * W * (640 + 32), gemm_kernel_count(cc, B * H * W, 16, 9 * 320, 0));
    float* out = u->out;
    float* next = u->next;
    const float* x_in = u->latent;
    P.record([=] {
      const size_t n = (size_t)B * 4 * H * W;
      launch_k(latent_out_kernel, (int)std::min<size_t>((n + 255) / 256, 1024), 256, 0, cc->stream,
          static_cast<const __half*>(y16), 16, out, B, 4, H * W, x_in, sched, next);
      return check_launch(cc, "latent_out");
    }, 3, 0, (double)B * H * W * (32 + 16 + 32));
  }
  P.finish_time_proj(tproj_at, temb, B, temb_fn, 2.0 * B * 1280 * (320 + 1280), 4.0 * 1280 * (320 + 1280),
                     2 * ((B + 7) / 8));
  P.finish_ctx_kv(tproj_at + 1, ctx16, B * Sk, 1024);  // after the time MLP on the side branch
  cudaDeviceSynchronize();
  return P.err;
}

// Config-1 ResNet block: fp32 NCHW in / out (fused-resnet.js drop-in, plus the timestep add).
struct ResPlan {
  Plan P;
  int N = 1, C = 320, H = 64, W = 64, Tdim = 1280;
  float* x = nullptr;      // [N,C,H,W]
  float* temb = nullptr;   // [N,Tdim]
  float* y = nullptr;      // [N,C,H,W]
};

static int build_resnet(ResPlan* r, float eps, int temb_silu) {
  Plan& P = r->P;
  const int N = r->N, C = r->C, H = r->H, W = r->W, HW = H * W, T = r->Tdim;
  Ctx* cc = P.c;
  void* sk = P.splitk;
  r->x = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * C * HW));
  r->temb = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * T));
  r->y = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * C * HW));
  float* xh = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * C * HW));   // NHWC fp32 copy of x
  float* yh = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * C * HW));   // NHWC fp32 result
  void* a = P.act_alloc((size_t)N * HW * C * 2);
  void* hbuf = P.act_alloc((size_t)N * HW * C * 2);
  void* part = P.act_alloc(gn_nhwc_ws_bytes(N, HW, 32));
  float* tp = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)N * C));
  if (P.err) return P.err;
  auto up32 = [&](const std::string& nm, size_t n, int kind, int fan, int fan_out = 0) {
    return P.upload_f32(P.host_param(nm, n, kind, fan, fan_out));
  };
  const float* G1 = up32("norm1.weight", C, 1, 1);
  const float* Be1 = up32("norm1.bias", C, 2, 1);
  const void* W1 = P.conv_weight("conv1.weight", C, C, C, C);
  const float* B1 = up32("conv1.bias", C, 0, 9 * C);
  const float* Wt = up32("time_emb_proj.weight", (size_t)C * T, 0, T, C);
  const float* Bt = up32("time_emb_proj.bias", C, 0, T);
  const float* G2 = up32("norm2.weight", C, 1, 1);
  const float* Be2 = up32("norm2.bias", C, 2, 1);
  const void* W2 = P.conv_weight("conv2.weight", C, C, C, C);
  const float* B2 = up32("conv2.bias", C, 0, 9 * C);
  const float* x = r->x;
  const float* te = r->temb;
  float* y = r->y;
  const double act = (double)N * HW * C;
  const double conv_flops = 2.0 * act * C * 9;
  P.record([=] { return nchw_to_nhwc(cc, DI_F32, DI_F32, x, xh, N, C, HW); }, 3, 0, 8.0 * act);
  P.record([=] { return group_norm_nhwc(cc, DI_F32, DI_F16, xh, C, nullptr, 0, N, HW, 32, eps, G1, Be1, 1, a, part); },
           2, 0, 10.0 * act, 2);
  P.record([=] { return gemv(cc, te, N, T, Wt, 0, Bt, C, temb_silu, tp, C); }, 3, 2.0 * N * C * T, 4.0 * C * T);
  P.record([=] { return gemm_conv3x3(cc, DI_F16, a, C, nullptr, 0, N, H, W, 1, W1, C, B1, tp, nullptr, 0, hbuf, 0, C, sk); },
           0, conv_flops, 4.0 * act + 18.0 * C * C, gemm_kernel_count(cc, N * HW, C, 9 * C, 0));
  P.record([=] { return group_norm_nhwc(cc, DI_F16, DI_F16, hbuf, C, nullptr, 0, N, HW, 32, eps, G2, Be2, 1, a, part); },
           2, 0, 6.0 * act, 2);
  P.record([=] { return gemm_conv3x3(cc, DI_F16, a, C, nullptr, 0, N, H, W, 1, W2, C, B2, nullptr, xh, 1, yh, 1, C, sk); },
           0, conv_flops, 10.0 * act + 18.0 * C * C, gemm_kernel_count(cc, N * HW, C, 9 * C, 0));
  P.record([=] { return nhwc_to_nchw(cc, DI_F32, DI_F32, yh, y, N, C, HW); }, 3, 0, 8.0 * act);
  cudaDeviceSynchronize();
  return P.err;
}

// Config-2 transformer block: token-major fp16 hidden [B,S,C] and context [B,Sk,Cctx].
struct TBPlan {
  Plan P;
  int B = 2, S = 1024, C = 640, Sk = 77, Cctx = 1024;
  void* hidden = nullptr;  // fp16 [B,S,C]
  void* ctx = nullptr;     // fp16 [B,Sk,Cctx]
  void* out = nullptr;     // fp16 [B,S,C]
};

static int build_tblock(TBPlan* t) {
  Plan& P = t->P;
  Act x;
  x.N = t->B; x.H = t->S; x.W = 1; x.C = t->C;
  x.p = P.act_alloc(x.bytes());
  t->hidden = x.p;
  t->ctx = P.act_alloc((size_t)t->B * t->Sk * t->Cctx * 2);
  if (P.err) return P.err;
  Act y = P.transformer("block", x, t->ctx, t->Sk, t->Cctx);
  t->out = y.p;
  cudaDeviceSynchronize();
  return P.err;
}

}  // namespace di

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------
using namespace di;

// SD VAE decoder (diffusers AutoencoderKL.decode: post_quant_conv + Decoder, block_out_channels
// 128/256/512/512, 3 ResNets per up block, GroupNorm 32 eps 1e-6, one mid-block attention), the graph
// vae-wgsl.js:99-118 runs (latent / 0.18215 first).  Latent [B,4,h,w] fp32 NCHW -> image [B,3,8h,8w].
struct VaePlan {
  Plan P;
  int B = 1, h = 64, w = 64;
  float* latent = nullptr;  // [B,4,h,w] fp32 NCHW (input)
  float* image = nullptr;   // [B,3,8h,8w] fp32 NCHW (output)
};

static size_t vae_ring_bytes(int B, int h, int w) {  // largest activation: 256 channels at 8h x 8w
  return (size_t)B * 64 * h * w * 256 * 2;
}
static size_t vae_tmp_bytes(int B, int h, int w) {
  // largest ResNet working set: GroupNorm output (256 ch) + conv1 output, GroupNorm output and shortcut
  // (128 ch each) at 8h x 8w; attention at h x w (q, k, o, V^T, scores) is smaller for the U-Net's sizes
  const size_t px = (size_t)B * 64 * h * w;
  const size_t resnet = px * (256 + 3 * 128) * 2 + (size_t)B * 256 * 16;
  const size_t hw = (size_t)h * w;
  const size_t attn = (size_t)B * hw * 512 * 2 * 4 + hw * 512 * 2 + hw * hw * 2 + (size_t)B * 512 * 16;
  return std::max(resnet, attn) + (64 << 20);
}

static int build_vae(VaePlan* v) {
  Plan& P = v->P;
  const int B = v->B, h = v->h, w = v->w;
  Ctx* cc = P.c;
  void* sk = P.splitk;
  v->latent = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 4 * h * w));
  v->image = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)B * 3 * 64 * h * w));
  for (int i = 0; i < 3; ++i) P.act_ring.push_back(P.act_alloc(vae_ring_bytes(B, h, w)));
  P.act_ring_bytes = vae_ring_bytes(B, h, w);
  if (P.err) return P.err;
  // latent NCHW fp32 -> NHWC fp16 padded to 64 channels
  Act lat = P.new_act(B, h, w, 64);
  {
    const float* src = v->latent;
    void* dst = lat.p;
    P.record([=] {
      const size_t n = (size_t)B * h * w * 64;
      launch_k(latent_in_kernel, (int)std::min<size_t>((n + 255) / 256, 4096), 256, 0, cc->stream, src,
               static_cast<__half*>(dst), B, 4, h * w, 64, nullptr);
      return check_launch(cc, "vae latent_in");
    }, 3, 0, (double)B * h * w * (16 + 128));
  }
  // post_quant_conv (1x1, 4 -> 4) with the 1/0.18215 latent scaling folded into its weight; channels
  // padded to 64 (zero rows / columns) so conv_in reads a 64-channel input
  Act z = P.new_act(B, h, w, 64);
  {
    auto wq = P.host_param("post_quant_conv.weight", 16, 0, 4, 4);
    auto bq = P.host_param("post_quant_conv.bias", 4, 0, 4);
    Plan::round_f16(wq);
    Plan::round_f16(bq);
    std::vector<float> wp(64 * 64, 0.0f), bp(64, 0.0f);
    for (int o = 0; o < 4; ++o) {
      for (int i = 0; i < 4; ++i) wp[o * 64 + i] = wq[o * 4 + i] / 0.18215f;
      bp[o] = bq[o];
    }
    P.linear(lat.p, B * h * w, 64, P.upload_f16(wp), 64, P.upload_f32(bp), nullptr, z.p);
  }
  // conv_in 4 (padded 64) -> 512
  Act x;
  {
    const void* wt = P.conv_weight("decoder.conv_in.weight", 512, 4, 64, 512);
    const float* bt = P.bias_padded("decoder.conv_in.bias", 512, 512, 4 * 9);
    x = P.new_act(B, h, w, 512);
    x.st = P.new_stat_slot();
    const Act zz = z, xx = x;
    P.record([=] {
      return Plan::with_stats(cc, xx.st, h * w, [&] {
        return gemm_conv3x3(cc, DI_F16, zz.p, 64, nullptr, 0, B, h, w, 1, wt, 512, bt, nullptr, nullptr, 0, xx.p, 0,
                            512, sk);
      });
    },
             0, 2.0 * B * h * w * 512 * 9 * 4, (double)B * h * w * (128 + 1024), gemm_kernel_count(cc, B * h * w, 512, 9 * 64, 0));
  }
  // mid block
  x = P.resnet("decoder.mid_block.resnets.0", x, nullptr, 512, 1e-6f, false);
  x = P.vae_attention("decoder.mid_block.attentions.0", x);
  x = P.resnet("decoder.mid_block.resnets.1", x, nullptr, 512, 1e-6f, false);
  // up blocks
  const int chans[4] = {512, 512, 256, 128};
  for (int i = 0; i < 4; ++i) {
    for (int j = 0; j < 3; ++j)
      x = P.resnet("decoder.up_blocks." + std::to_string(i) + ".resnets." + std::to_string(j), x, nullptr, chans[i],
                   1e-6f, false);
    if (i < 3) {
      P.tmp_reset();
      x = P.conv3x3("decoder.up_blocks." + std::to_string(i) + ".upsamplers.0.conv", P.upsample(x), chans[i], 1);
    }
  }
  // conv_norm_out + SiLU, conv_out 128 -> 3 (padded to 16), NHWC fp16 -> NCHW fp32
  P.tmp_reset();
  const Plan::GnOp go = P.gn_op("decoder.conv_norm_out", x, nullptr, 1e-6f, 1);
  const int H = x.H, W = x.W;
  {
    const void* wt = P.conv_weight("decoder.conv_out.weight", 3, 128, 128, 16);
    const float* bt = P.bias_padded("decoder.conv_out.bias", 3, 16, 128 * 9);
    void* y16 = P.tmp((size_t)B * H * W * 16 * 2);
    P.record([=] {
      const GnFuse f{go.tab, go.silu};
      return gemm_conv3x3(cc, DI_F16, go.x1, 128, nullptr, 0, B, H, W, 1, wt, 16, bt, nullptr, nullptr, 0, y16, 0, 16, sk,
                          go.tab ? &f : nullptr);
    }, 0, 2.0 * B * H * W * 3 * 9 * 128, (double)B * H * W * (256 + 32), gemm_kernel_count(cc, B * H * W, 16, 9 * 128, 0));
    float* out = v->image;
    P.record([=] {
      const size_t n = (size_t)B * 3 * H * W;
      launch_k(latent_out_kernel, (int)std::min<size_t>((n + 255) / 256, 8192), 256, 0, cc->stream,
               static_cast<const __half*>(y16), 16, out, B, 3, H * W, nullptr, nullptr, nullptr);
      return check_launch(cc, "vae image_out");
    }, 3, 0, (double)B * H * W * (32 + 12));
  }
  cudaDeviceSynchronize();
  return P.err;
}

// OpenCLIP ViT-H text encoder as SD2.x / SD-Turbo use it (HF CLIPTextModel names): token + position
// embeddings, `layers` pre-LN blocks (causal multi-head self-attention with biased q/k/v/out projections,
// MLP 1024 -> 4096 -> 1024 with erf GELU), final LayerNorm.  The reference runs this model through ONNX
// Runtime (text-encoder.js:69-174); its output is last_hidden_state [B, 77, 1024].
// The residual stream stays fp32 (the GEMM epilogues add the residual in fp32 and write fp32);
// LayerNorm outputs, q/k/v, attention output and the MLP hidden are fp16.
struct TextPlan {
  Plan P;
  int B = 1, S = 77, layers = 24;
  int* ids = nullptr;          // [B,S] int32 token ids (input)
  float* hidden = nullptr;     // [B,S,1024] fp32 (output)
  float* ext_hidden = nullptr; // when set before building: write the output here (the U-Net's context)
};

static constexpr int kTextD = 1024, kTextHeads = 16, kTextF = 4096, kTextVocab = 49408, kTextPos = 77;

static size_t text_tmp_bytes(int, int) { return 1u << 20; }

static int build_text(TextPlan* t) {
  Plan& P = t->P;
  const int B = t->B, S = t->S, D = kTextD, F = kTextF, M = B * S;
  Ctx* cc = P.c;
  void* sk = P.splitk;
  t->ids = static_cast<int*>(P.act_alloc(sizeof(int) * (size_t)M));
  t->hidden = t->ext_hidden ? t->ext_hidden : static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)M * D));
  float* x = static_cast<float*>(P.act_alloc(sizeof(float) * (size_t)M * D));
  __half* n = static_cast<__half*>(P.act_alloc(2 * (size_t)M * D));
  __half* qkv = static_cast<__half*>(P.act_alloc(2 * (size_t)M * 3 * D));
  __half* o = static_cast<__half*>(P.act_alloc(2 * (size_t)M * D));
  __half* mid = static_cast<__half*>(P.act_alloc(2 * (size_t)M * F));
  if (P.err) return P.err;
  {
    const void* tok = P.upload_f16(P.host_param("text_model.embeddings.token_embedding.weight",
                                                (size_t)kTextVocab * D, 2, 1));
    const void* pos = P.upload_f16(P.host_param("text_model.embeddings.position_embedding.weight",
                                                (size_t)kTextPos * D, 2, 1));
    const int* ids = t->ids;
    P.record([=] {
      const size_t total = (size_t)M * (D / 8);
      launch_k(embed_tokens_kernel, (int)std::min<size_t>((total + 255) / 256, 4096), 256, 0, cc->stream, ids, M, S,
               static_cast<const __half*>(tok), static_cast<const __half*>(pos), D, kTextVocab, x, cc->d_err);
      return check_launch(cc, "embed_tokens");
    }, 3, 0, (double)M * D * (2 + 2 + 4));
  }
  for (int l = 0; l < t->layers; ++l) {
    const std::string pre = "text_model.encoder.layers." + std::to_string(l);
    const float* g1 = P.vec(pre + ".layer_norm1.weight", D, 1, 1);
    const float* b1 = P.vec(pre + ".layer_norm1.bias", D, 2, 1);
    P.record([=] { return layer_norm(cc, DI_F32, DI_F16, x, g1, b1, n, M, D, 1e-5f); }, 2, 0, 6.0 * M * D);
    std::vector<float> wqkv, bqkv;
    for (const char* nm : {".self_attn.q_proj", ".self_attn.k_proj", ".self_attn.v_proj"}) {
      auto w = P.host_param(pre + nm + ".weight", (size_t)D * D, 0, D, D);
      auto b = P.host_param(pre + nm + ".bias", D, 0, D);
      wqkv.insert(wqkv.end(), w.begin(), w.end());
      bqkv.insert(bqkv.end(), b.begin(), b.end());
    }
    Plan::round_f16(bqkv);
    const void* Wqkv = P.upload_f16(wqkv);
    const float* Bqkv = P.upload_f32(bqkv);
    P.linear(n, M, D, Wqkv, 3 * D, Bqkv, nullptr, qkv);
    P.record([=] {
      return attention(cc, DI_F16, qkv, qkv + D, qkv + 2 * D, o, B, kTextHeads, S, S, 0, 3 * D, 3 * D, 3 * D, D, 1);
    }, 1, 2.0 * B * kTextHeads * (double)S * (S + 1) * 64, 2.0 * 4 * M * D);
    const void* Wo = P.lin_weight(pre + ".self_attn.out_proj.weight", D, D);
    const float* Bo = P.vec(pre + ".self_attn.out_proj.bias", D, 0, D);
    P.record([=] { return gemm_linear(cc, DI_F16, o, D, nullptr, M, D, Wo, D, Bo, x, 1, x, 1, 0, nullptr, 1, sk); },
             0, 2.0 * M * D * D, 2.0 * ((double)M * D + (double)D * D) + 8.0 * M * D, gemm_kernel_count(cc, M, D, D, 0));
    const float* g2 = P.vec(pre + ".layer_norm2.weight", D, 1, 1);
    const float* b2 = P.vec(pre + ".layer_norm2.bias", D, 2, 1);
    P.record([=] { return layer_norm(cc, DI_F32, DI_F16, x, g2, b2, n, M, D, 1e-5f); }, 2, 0, 6.0 * M * D);
    const void* W1 = P.lin_weight(pre + ".mlp.fc1.weight", F, D);
    const float* B1 = P.vec(pre + ".mlp.fc1.bias", F, 0, D);
    P.record([=] {
      return gemm_linear(cc, DI_F16, n, D, nullptr, M, D, W1, F, B1, nullptr, 0, mid, 0, 0, nullptr, 1, sk, nullptr, 0,
                         2);
    }, 0, 2.0 * M * F * D, 2.0 * ((double)M * D + (double)F * D + (double)M * F), gemm_kernel_count(cc, M, F, D, 0));
    const void* W2 = P.lin_weight(pre + ".mlp.fc2.weight", D, F);
    const float* B2 = P.vec(pre + ".mlp.fc2.bias", D, 0, F);
    P.record([=] { return gemm_linear(cc, DI_F16, mid, F, nullptr, M, F, W2, D, B2, x, 1, x, 1, 0, nullptr, 1, sk); },
             0, 2.0 * M * D * F, 2.0 * ((double)M * F + (double)D * F) + 8.0 * M * D, gemm_kernel_count(cc, M, D, F, 0));
  }
  const float* gf = P.vec("text_model.final_layer_norm.weight", D, 1, 1);
  const float* bf = P.vec("text_model.final_layer_norm.bias", D, 2, 1);
  float* out = t->hidden;
  P.record([=] { return layer_norm(cc, DI_F32, DI_F32, x, gf, bf, out, M, D, 1e-5f); }, 2, 0, 8.0 * M * D);
  cudaDeviceSynchronize();
  return P.err;
}

// Batched one-step text-to-image (config 5): text encoder -> U-Net (scaleModelInput fused into its input
// conversion, the Euler step into its output conversion) -> VAE decoder; the text encoder writes the
// U-Net's context directly.  The VAE decodes in chunks of up to 8 images (its 512x512 maps are 0.5 GB per
// image at 256 channels): each chunk's latent is copied into the VAE plan's input and its image out to
// the pipeline's image buffer.  Three plans (CUDA graphs) replayed in order on the context stream.
struct T2IPlan {
  TextPlan text;
  UNetPlan unet;
  VaePlan vae;
  int vae_chunk = 1;
  float* image = nullptr;  // [B,3,8h,8w] fp32
  float sigma0 = 0.f;
};

struct di_unet_s { UNetPlan u; };
struct di_text_s { TextPlan t; };
struct di_t2i_s { T2IPlan p; };

// Euler-discrete sigmas of scheduler.js:27-89 for n inference steps ("trailing" timesteps, the last sigma
// 0): double arithmetic rounded to float at each Float32Array store, Math.round as floor(x + 0.5).
static void euler_sigmas(int n, float* sig_out, float* ts_out) {
  std::vector<float> betas(1000), alphas(1000), sig(1000);
  const double b0 = std::sqrt(0.00085), b1 = std::sqrt(0.012);
  for (int i = 0; i < 1000; ++i) {
    const double v = b0 + (b1 - b0) * (i / 999.0);
    betas[i] = (float)(v * v);
  }
  double prod = 1.0;
  for (int i = 0; i < 1000; ++i) {
    prod *= 1.0 - (double)betas[i];
    alphas[i] = (float)prod;
  }
  for (int i = 0; i < 1000; ++i) sig[i] = (float)std::sqrt((1.0 - (double)alphas[i]) / (double)alphas[i]);
  const double step = 1000.0 / n;
  for (int i = 0; i < n; ++i) {
    const float t = (float)std::floor(1000.0 - (i + 1) * step + step + 0.5) - 1.0f;
    ts_out[i] = t;
    double v;
    if (t <= 0) v = sig[0];
    else if (t >= 999) v = sig[999];
    else {
      const int k = (int)std::floor((double)t);
      const double f = (double)t - k;
      v = (double)sig[k] * (1 - f) + (double)sig[k + 1] * f;
    }
    sig_out[i] = (float)v;
  }
  sig_out[n] = 0.0f;
}
struct di_vae_s { VaePlan v; };
struct di_resnet_s { ResPlan r; };
struct di_tblock_s { TBPlan t; };

extern "C" {

DI_API void di_synth_uniform(uint64_t seed, const char* name, size_t n, float bound, float* out) {
  synth_uniform(seed, name, n, bound, out);
}
DI_API int di_euler_sigmas(int n, float* sigmas, float* timesteps) {
  if (n <= 0 || !sigmas || !timesteps) return DI_EINVAL;
  euler_sigmas(n, sigmas, timesteps);
  return DI_OK;
}
DI_API void di_synth_normal(uint64_t seed, const char* name, size_t n, float mean, float stdv, float* out) {
  synth_normal(seed, name, n, mean, stdv, out);
}

DI_API int di_unet_create(di_ctx_t h, int B, int H, int W, int ctx_len, uint64_t seed, di_weight_fn fn, void* user,
                          di_unet_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || B <= 0 || H <= 0 || W <= 0 || ctx_len <= 0 || (H % 8) || (W % 8))
    return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_unet_s();
  s->u.B = B; s->u.H = H; s->u.W = W; s->u.Sk = ctx_len;
  cudaSetDevice(c->device);
  if (!s->u.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, unet_tmp_bytes(B, H, W))) {
    delete s;
    return set_error(c, DI_ENOMEM, "unet: init");
  }
  int r = build_unet(&s->u);
  if (r) {
    std::string m = s->u.P.errmsg;
    delete s;
    return set_error(c, r, "unet build: " + m);
  }
  *out = s;
  return DI_OK;
}

// Scheduler on the device: the U-Net scales its latent input by `in_scale` (scaleModelInput) and writes
// next = latent + dt * eps (the Euler step) beside the noise prediction.  Defaults 1 and 0.
DI_API int di_unet_sched(di_unet_t u, double in_scale, double dt, float** next) {
  if (!u) return DI_EINVAL;
  const double v[2] = {in_scale, dt};
  Ctx* c = u->u.P.c;
  if (cudaMemcpyAsync(u->u.sched, v, sizeof v, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      cudaStreamSynchronize(c->stream) != cudaSuccess)
    return set_error(c, DI_ECUDA, "unet sched: copy");
  if (next) *next = u->u.next;
  return DI_OK;
}

DI_API int di_unet_io(di_unet_t u, float** latent, float** t, float** ctx, float** out) {
  if (!u) return DI_EINVAL;
  if (latent) *latent = u->u.latent;
  if (t) *t = u->u.tvals;
  if (ctx) *ctx = u->u.ctx32;
  if (out) *out = u->u.out;
  return DI_OK;
}

DI_API int di_unet_info(di_unet_t u, int* launches, size_t* weight_bytes, size_t* act_bytes) {
  if (!u) return DI_EINVAL;
  if (launches) *launches = u->u.P.launches;
  if (weight_bytes) *weight_bytes = u->u.P.weight_bytes;
  if (act_bytes) *act_bytes = u->u.P.act_bytes;
  return DI_OK;
}

DI_API int di_unet_ops(di_unet_t u, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels) {
  if (!u || !n_ops) return DI_EINVAL;
  const auto& I = u->u.P.info;
  *n_ops = (int)I.size();
  for (size_t i = 0; i < I.size(); ++i) {
    if (kinds) kinds[i] = I[i].kind;
    if (flops) flops[i] = I[i].flops;
    if (bytes) bytes[i] = I[i].bytes;
    if (kernels) kernels[i] = I[i].kernels;
  }
  return DI_OK;
}

DI_API int di_unet_profile(di_unet_t u, int reps, float* op_ms) {
  if (!u || !op_ms || reps <= 0) return DI_EINVAL;
  return u->u.P.profile(reps, op_ms);
}

DI_API int di_unet_profile_kind(di_unet_t u, int kind, int reps, float* ms) {
  if (!u || !ms || reps <= 0) return DI_EINVAL;
  return u->u.P.profile_kind(kind, reps, ms);
}

DI_API int di_unet_forward(di_unet_t u) {
  if (!u) return DI_EINVAL;
  return u->u.P.forward();
}

DI_API int di_unet_forward_host(di_unet_t u, const float* latent, const float* t, const float* ctx, float* out) {
  if (!u || !latent || !t || !ctx || !out) return DI_EINVAL;
  UNetPlan& p = u->u;
  Ctx* c = p.P.c;
  const size_t nl = (size_t)p.B * 4 * p.H * p.W, nc = (size_t)p.B * p.Sk * 1024;
  cudaMemcpyAsync(p.latent, latent, nl * 4, cudaMemcpyHostToDevice, c->stream);
  cudaMemcpyAsync(p.tvals, t, p.B * 4, cudaMemcpyHostToDevice, c->stream);
  cudaMemcpyAsync(p.ctx32, ctx, nc * 4, cudaMemcpyHostToDevice, c->stream);
  int r = p.P.forward();
  if (r) return r;
  cudaMemcpyAsync(out, p.out, nl * 4, cudaMemcpyDeviceToHost, c->stream);
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return set_error(c, DI_ECUDA, "unet forward_host sync");
  return DI_OK;
}

DI_API void di_unet_destroy(di_unet_t u) { delete u; }

// ---- text encoder -----------------------------------------------------------------------------
DI_API int di_text_create(di_ctx_t h, int B, int S, int layers, uint64_t seed, di_weight_fn fn, void* user,
                          di_text_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || B <= 0 || S <= 0 || S > kTextPos || layers <= 0) return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_text_s();
  s->t.B = B; s->t.S = S; s->t.layers = layers;
  cudaSetDevice(c->device);
  if (!s->t.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, text_tmp_bytes(B, S))) {
    delete s;
    return set_error(c, DI_ENOMEM, "text encoder: init");
  }
  int r = build_text(&s->t);
  if (r) {
    std::string m = s->t.P.errmsg;
    delete s;
    return set_error(c, r, "text encoder build: " + m);
  }
  *out = s;
  return DI_OK;
}
DI_API int di_text_io(di_text_t t, int** ids, float** hidden) {
  if (!t) return DI_EINVAL;
  if (ids) *ids = t->t.ids;
  if (hidden) *hidden = t->t.hidden;
  return DI_OK;
}
DI_API int di_text_info(di_text_t t, int* launches, size_t* weight_bytes, size_t* act_bytes) {
  if (!t) return DI_EINVAL;
  if (launches) *launches = t->t.P.launches;
  if (weight_bytes) *weight_bytes = t->t.P.weight_bytes;
  if (act_bytes) *act_bytes = t->t.P.act_bytes;
  return DI_OK;
}
DI_API int di_text_ops(di_text_t t, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels) {
  if (!t || !n_ops) return DI_EINVAL;
  const auto& I = t->t.P.info;
  *n_ops = (int)I.size();
  for (size_t i = 0; i < I.size(); ++i) {
    if (kinds) kinds[i] = I[i].kind;
    if (flops) flops[i] = I[i].flops;
    if (bytes) bytes[i] = I[i].bytes;
    if (kernels) kernels[i] = I[i].kernels;
  }
  return DI_OK;
}
DI_API int di_text_forward(di_text_t t) { return t ? t->t.P.forward() : DI_EINVAL; }
DI_API int di_text_forward_host(di_text_t t, const int* ids, float* hidden) {
  if (!t || !ids || !hidden) return DI_EINVAL;
  TextPlan& p = t->t;
  Ctx* c = p.P.c;
  const size_t n = (size_t)p.B * p.S;
  for (size_t i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= kTextVocab) return set_error(c, DI_EINVAL, "text encoder: token id out of range");
  cudaMemcpyAsync(p.ids, ids, n * 4, cudaMemcpyHostToDevice, c->stream);
  int r = p.P.forward();
  if (r) return r;
  cudaMemcpyAsync(hidden, p.hidden, n * kTextD * 4, cudaMemcpyDeviceToHost, c->stream);
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return set_error(c, DI_ECUDA, "text forward_host sync");
  return DI_OK;
}
DI_API void di_text_destroy(di_text_t t) { delete t; }

// ---- one-step text-to-image (config 5) --------------------------------------------------------
DI_API int di_t2i_create(di_ctx_t h, int B, int lh, int lw, int text_layers, uint64_t seed, di_weight_fn fn,
                         void* user, di_t2i_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || B <= 0 || lh <= 0 || lw <= 0 || (lh % 8) || (lw % 8) || text_layers <= 0) return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_t2i_s();
  T2IPlan& p = s->p;
  cudaSetDevice(c->device);
  auto fail = [&](int r, const std::string& what) {
    delete s;
    return set_error(c, r, what);
  };
  p.unet.B = B; p.unet.H = lh; p.unet.W = lw; p.unet.Sk = kTextPos;
  if (!p.unet.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, unet_tmp_bytes(B, lh, lw)))
    return fail(DI_ENOMEM, "t2i: unet init");
  // the U-Net plan owns the shared buffers: the context the text encoder writes, the decoded images
  p.unet.ext_ctx = static_cast<float*>(p.unet.P.act_alloc(sizeof(float) * (size_t)B * kTextPos * kTextD));
  p.image = static_cast<float*>(p.unet.P.act_alloc(sizeof(float) * (size_t)B * 3 * 64 * lh * lw));
  int r = build_unet(&p.unet);
  if (r) return fail(r, "t2i unet build: " + p.unet.P.errmsg);
  p.text.B = B; p.text.S = kTextPos; p.text.layers = text_layers; p.text.ext_hidden = p.unet.ext_ctx;
  if (!p.text.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, text_tmp_bytes(B, kTextPos)))
    return fail(DI_ENOMEM, "t2i: text init");
  r = build_text(&p.text);
  if (r) return fail(r, "t2i text build: " + p.text.P.errmsg);
  p.vae_chunk = 1;
  for (int k = std::min(B, 8); k >= 1; --k)
    if (B % k == 0) { p.vae_chunk = k; break; }
  p.vae.B = p.vae_chunk; p.vae.h = lh; p.vae.w = lw;
  if (!p.vae.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, vae_tmp_bytes(p.vae_chunk, lh, lw)))
    return fail(DI_ENOMEM, "t2i: vae init");
  r = build_vae(&p.vae);
  if (r) return fail(r, "t2i vae build: " + p.vae.P.errmsg);
  // one-step schedule: t = 999, scaleModelInput by 1/sqrt(sigma0^2 + 1), Euler step dt = 0 - sigma0
  float sig[2], ts[1];
  euler_sigmas(1, sig, ts);
  p.sigma0 = sig[0];
  std::vector<float> tv(B, ts[0]);
  cudaMemcpy(p.unet.tvals, tv.data(), sizeof(float) * B, cudaMemcpyHostToDevice);
  const double s0 = sig[0];
  const double v[2] = {1.0 / std::sqrt(s0 * s0 + 1.0), (double)sig[1] - s0};
  cudaMemcpy(p.unet.sched, v, sizeof v, cudaMemcpyHostToDevice);
  *out = s;
  return DI_OK;
}
DI_API int di_t2i_io(di_t2i_t t, int** ids, float** latent, float** image, float** ctx, float** eps) {
  if (!t) return DI_EINVAL;
  if (ids) *ids = t->p.text.ids;
  if (latent) *latent = t->p.unet.latent;
  if (image) *image = t->p.image;
  if (ctx) *ctx = t->p.unet.ctx32;
  if (eps) *eps = t->p.unet.out;
  return DI_OK;
}
DI_API int di_t2i_info(di_t2i_t t, int* launches, size_t* weight_bytes, size_t* act_bytes, float* sigma0) {
  if (!t) return DI_EINVAL;
  const T2IPlan& p = t->p;
  const int chunks = p.unet.B / p.vae_chunk;
  if (launches) *launches = p.text.P.launches + p.unet.P.launches + chunks * p.vae.P.launches;
  if (weight_bytes) *weight_bytes = p.text.P.weight_bytes + p.unet.P.weight_bytes + p.vae.P.weight_bytes;
  if (act_bytes) *act_bytes = p.text.P.act_bytes + p.unet.P.act_bytes + p.vae.P.act_bytes;
  if (sigma0) *sigma0 = p.sigma0;
  return DI_OK;
}
// stage -1: the whole pipeline; 0 text encoder, 1 U-Net + scheduler, 2 VAE decoder.
DI_API int di_t2i_forward(di_t2i_t t, int stage) {
  if (!t || stage < -1 || stage > 2) return DI_EINVAL;
  T2IPlan& p = t->p;
  int r = DI_OK;
  if (stage == -1 || stage == 0) r = p.text.P.forward();
  if (r == DI_OK && (stage == -1 || stage == 1)) r = p.unet.P.forward();
  if (r == DI_OK && (stage == -1 || stage == 2)) {
    Ctx* c = p.unet.P.c;
    const int k = p.vae_chunk;
    const size_t lat = (size_t)4 * p.vae.h * p.vae.w, img = (size_t)3 * 64 * p.vae.h * p.vae.w;
    for (int b0 = 0; r == DI_OK && b0 < p.unet.B; b0 += k) {
      if (cudaMemcpyAsync(p.vae.latent, p.unet.next + b0 * lat, k * lat * 4, cudaMemcpyDeviceToDevice,
                          c->stream) != cudaSuccess)
        return set_error(c, DI_ECUDA, "t2i: latent chunk copy");
      r = p.vae.P.forward();
      if (r == DI_OK && cudaMemcpyAsync(p.image + b0 * img, p.vae.image, k * img * 4, cudaMemcpyDeviceToDevice,
                                        c->stream) != cudaSuccess)
        return set_error(c, DI_ECUDA, "t2i: image chunk copy");
    }
  }
  return r;
}
DI_API int di_t2i_forward_host(di_t2i_t t, const int* ids, const float* latent, float* image) {
  if (!t || !ids || !latent || !image) return DI_EINVAL;
  T2IPlan& p = t->p;
  Ctx* c = p.unet.P.c;
  const int B = p.unet.B;
  const size_t nid = (size_t)B * kTextPos, nl = (size_t)B * 4 * p.unet.H * p.unet.W;
  const size_t ni = (size_t)B * 3 * 64 * p.unet.H * p.unet.W;
  for (size_t i = 0; i < nid; ++i)
    if (ids[i] < 0 || ids[i] >= kTextVocab) return set_error(c, DI_EINVAL, "t2i: token id out of range");
  cudaMemcpyAsync(p.text.ids, ids, nid * 4, cudaMemcpyHostToDevice, c->stream);
  cudaMemcpyAsync(p.unet.latent, latent, nl * 4, cudaMemcpyHostToDevice, c->stream);
  int r = di_t2i_forward(t, -1);
  if (r) return r;
  cudaMemcpyAsync(image, p.image, ni * 4, cudaMemcpyDeviceToHost, c->stream);
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return set_error(c, DI_ECUDA, "t2i forward_host sync");
  return DI_OK;
}
DI_API void di_t2i_destroy(di_t2i_t t) { delete t; }

DI_API int di_vae_create(di_ctx_t h, int B, int lh, int lw, uint64_t seed, di_weight_fn fn, void* user, di_vae_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || B <= 0 || lh <= 0 || lw <= 0 || (lh * lw) % 64) return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_vae_s();
  s->v.B = B; s->v.h = lh; s->v.w = lw;
  if (!s->v.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, vae_tmp_bytes(B, lh, lw))) {
    delete s;
    return set_error(c, DI_ENOMEM, "vae: allocation");
  }
  int r = build_vae(&s->v);
  if (r) {
    std::string m = s->v.P.errmsg;
    delete s;
    return set_error(c, r, "vae build: " + m);
  }
  *out = s;
  return DI_OK;
}
DI_API int di_vae_io(di_vae_t v, float** latent, float** image) {
  if (!v) return DI_EINVAL;
  if (latent) *latent = v->v.latent;
  if (image) *image = v->v.image;
  return DI_OK;
}
DI_API int di_vae_info(di_vae_t v, int* launches, size_t* weight_bytes, size_t* act_bytes) {
  if (!v) return DI_EINVAL;
  if (launches) *launches = v->v.P.launches;
  if (weight_bytes) *weight_bytes = v->v.P.weight_bytes;
  if (act_bytes) *act_bytes = v->v.P.act_bytes;
  return DI_OK;
}
DI_API int di_vae_ops(di_vae_t v, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels) {
  if (!v || !n_ops) return DI_EINVAL;
  const auto& I = v->v.P.info;
  *n_ops = (int)I.size();
  for (size_t i = 0; i < I.size(); ++i) {
    if (kinds) kinds[i] = I[i].kind;
    if (flops) flops[i] = I[i].flops;
    if (bytes) bytes[i] = I[i].bytes;
    if (kernels) kernels[i] = I[i].kernels;
  }
  return DI_OK;
}
DI_API int di_vae_profile_kind(di_vae_t v, int kind, int reps, float* ms) {
  if (!v || !ms || reps <= 0) return DI_EINVAL;
  return v->v.P.profile_kind(kind, reps, ms);
}
DI_API int di_vae_forward(di_vae_t v) { return v ? v->v.P.forward() : DI_EINVAL; }
DI_API int di_vae_forward_host(di_vae_t v, const float* latent, float* image) {
  if (!v || !latent || !image) return DI_EINVAL;
  VaePlan& p = v->v;
  Ctx* c = p.P.c;
  const size_t nl = (size_t)p.B * 4 * p.h * p.w, ni = (size_t)p.B * 3 * 64 * p.h * p.w;
  cudaMemcpyAsync(p.latent, latent, nl * 4, cudaMemcpyHostToDevice, c->stream);
  int r = p.P.forward();
  if (r) return r;
  cudaMemcpyAsync(image, p.image, ni * 4, cudaMemcpyDeviceToHost, c->stream);
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return set_error(c, DI_ECUDA, "vae forward_host sync");
  return DI_OK;
}
DI_API void di_vae_destroy(di_vae_t v) { delete v; }
// Diagnostics: copy bytes of activation-ring buffer `idx` (idx < 0: the temporary arena) to the host.
DI_API int di_vae_debug_copy(di_vae_t v, int idx, size_t off, void* dst, size_t bytes) {
  if (!v || !dst) return DI_EINVAL;
  Plan& P = v->v.P;
  const char* src = idx < 0 ? P.tmp_base : (idx < (int)P.act_ring.size() ? static_cast<const char*>(P.act_ring[idx]) : nullptr);
  if (!src) return DI_EINVAL;
  cudaStreamSynchronize(P.c->stream);
  return cudaMemcpy(dst, src + off, bytes, cudaMemcpyDeviceToHost) == cudaSuccess ? DI_OK : DI_ECUDA;
}

DI_API int di_resnet_block_create(di_ctx_t h, int N, int C, int H, int W, int Tdim, uint64_t seed, float eps,
                                  int temb_silu, di_weight_fn fn, void* user, di_resnet_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || N <= 0 || C % 64 || Tdim <= 0) return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_resnet_s();
  s->r.N = N; s->r.C = C; s->r.H = H; s->r.W = W; s->r.Tdim = Tdim;
  if (!s->r.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, 1 << 20)) { delete s; return DI_ENOMEM; }
  s->r.P.init_mode = 1;  // Kaiming-uniform weights
  int r = build_resnet(&s->r, eps, temb_silu);
  if (r) { std::string m = s->r.P.errmsg; delete s; return set_error(c, r, "resnet build: " + m); }
  *out = s;
  return DI_OK;
}
DI_API int di_resnet_block_io(di_resnet_t r, float** x, float** temb, float** y) {
  if (!r) return DI_EINVAL;
  if (x) *x = r->r.x;
  if (temb) *temb = r->r.temb;
  if (y) *y = r->r.y;
  return DI_OK;
}
DI_API int di_resnet_block_run(di_resnet_t r) { return r ? r->r.P.forward() : DI_EINVAL; }
DI_API void di_resnet_block_destroy(di_resnet_t r) { delete r; }

DI_API int di_transformer_block_create(di_ctx_t h, int B, int S, int C, int Sk, int Cctx, uint64_t seed,
                                       di_weight_fn fn, void* user, di_tblock_t* out) {
  Ctx* c = ctx_of(h);
  if (!c || !out || B <= 0 || S <= 0 || C % 64 || Cctx % 64 || Sk <= 0) return DI_EINVAL;
  *out = nullptr;
  auto* s = new di_tblock_s();
  s->t.B = B; s->t.S = S; s->t.C = C; s->t.Sk = Sk; s->t.Cctx = Cctx;
  const size_t M = (size_t)B * S;
  if (!s->t.P.init(c, seed, reinterpret_cast<WeightFn>(fn), user, M * C * 2 * 27 + (size_t)B * Sk * 2 * C * 2 + (16 << 20))) {
    delete s;
    return DI_ENOMEM;
  }
  s->t.P.init_mode = 2;  // Xavier-uniform weights, zero biases
  int r = build_tblock(&s->t);
  if (r) { std::string m = s->t.P.errmsg; delete s; return set_error(c, r, "transformer build: " + m); }
  *out = s;
  return DI_OK;
}
DI_API int di_transformer_block_io(di_tblock_t t, void** hidden, void** ctx, void** out) {
  if (!t) return DI_EINVAL;
  if (hidden) *hidden = t->t.hidden;
  if (ctx) *ctx = t->t.ctx;
  if (out) *out = t->t.out;
  return DI_OK;
}
DI_API int di_transformer_block_run(di_tblock_t t) { return t ? t->t.P.forward() : DI_EINVAL; }
DI_API void di_transformer_block_destroy(di_tblock_t t) { delete t; }

}  // extern "C"
