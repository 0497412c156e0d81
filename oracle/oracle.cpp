// oracle.cpp — TEST INFRASTRUCTURE ONLY (never linked into, or called by, the product path).
//
// A float32 C++17 restatement of the reference's (abgnydn/draw-instant) WGSL kernels and of its
// JavaScript scheduler / weight plumbing.  It is the parity checker for the sm_100a kernels in
// libdi.so: the pytest suite, __graft_entry__.smoke() and bench.py's CPU baseline leg are the only
// callers.  Each function cites the reference file:line it follows.  OpenMP is used across host
// cores; reductions keep the reference's formulas (sum / sum-of-squares variance, max-subtract
// softmax) but their summation order is sequential per output, not the WGSL tree order.
//
// Parity pins: scheduler timesteps (scheduler.js:4-5), the f16->f32 bit conversion, and the
// numeric cases of wgsl-ops-test.js (regenerated as fixtures by tests/golden/make_golden.py).
// The fused-block outputs have no golden vectors in the reference (its own tests compare naive vs
// fused WGSL on unseeded random data), so their parity is pinned only through these formulas.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <vector>
#include <string>
#include <algorithm>
#include <chrono>
#include <unordered_map>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ------------------------------------------------------------------------------------------
// Seeded synthetic generator (the build's own documented scheme; restated independently in the
// product's host code, checked bit-for-bit by tests/test_generator.py).
//   key     = mix64(seed * 0x9E3779B97F4A7C15 + fnv1a64(name))
//   u_i     = (mix64(key + (i+1) * 0x9E3779B97F4A7C15) >> 40) * 2^-24      (exact in float)
//   uniform = (2u - 1) * bound, evaluated in float
//   normal  = Box-Muller in double on (u_{2j}, u_{2j+1}), cos for even i, sin for odd i
// ------------------------------------------------------------------------------------------
inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
inline uint64_t fnv1a64(const char* s) {
  uint64_t h = 0xcbf29ce484222325ULL;
  for (; *s; ++s) { h ^= (uint8_t)*s; h *= 0x100000001b3ULL; }
  return h;
}
inline uint64_t stream_key(uint64_t seed, const char* name) {
  return mix64(seed * 0x9E3779B97F4A7C15ULL + fnv1a64(name));
}
inline float unit_u(uint64_t key, uint64_t i) {
  return (float)(mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL) >> 40) * (1.0f / 16777216.0f);
}

void gen_uniform(uint64_t seed, const char* name, size_t n, float bound, float* out) {
  const uint64_t key = stream_key(seed, name);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    const float u = unit_u(key, (uint64_t)i);
    const float t = 2.0f * u - 1.0f;  // exact: u has 24 fractional bits
    out[i] = t * bound;
  }
}
void gen_normal(uint64_t seed, const char* name, size_t n, float mean, float stdv, float* out) {
  const uint64_t key = stream_key(seed, name);
  const double two_pi = 6.283185307179586;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    const uint64_t j = (uint64_t)i & ~1ULL;
    double u1 = (double)unit_u(key, j);
    double u2 = (double)unit_u(key, j + 1);
    if (u1 < 1.0 / 16777216.0) u1 = 1.0 / 16777216.0;
    double r = std::sqrt(-2.0 * std::log(u1));
    double z = (i & 1) ? r * std::sin(two_pi * u2) : r * std::cos(two_pi * u2);
    out[i] = (float)((double)mean + (double)stdv * z);
  }
}

// IEEE binary16 -> binary32, restating wgsl-unet.js:23-47 (subnormals renormalised, Inf/NaN kept).
inline float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  int32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) bits = sign;
    else {
      while ((mant & 0x400) == 0) { mant <<= 1; exp -= 1; }
      exp += 1; mant &= 0x3ff;
      bits = sign | ((uint32_t)(exp + 112) << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((uint32_t)(exp + 112) << 23) | (mant << 13);
  }
  float f; std::memcpy(&f, &bits, 4); return f;
}
// binary32 -> binary16, round to nearest even (the rounding the fp16 weight arena uses).
inline uint16_t f2h(float f) {
  uint32_t x; std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);           // rounds to >= 65520 -> Inf
  if (ax < 0x38800000u) {                                              // result subnormal or zero
    if (ax < 0x33000000u) return (uint16_t)sign;                       // < 2^-25 -> 0
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126 - e;                                    // value = q * 2^-24
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112;
  uint32_t m = ax & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(sign | q);
}
inline float round_h(float f) { return h2f(f2h(f)); }

inline float silu(float x) { return x / (1.0f + std::exp(-x)); }
// Abramowitz-Stegun 7.1.26, as in wgsl-ops.js:77-81.
inline float erf_as(float x) {
  float t = 1.0f / (1.0f + 0.3275911f * std::fabs(x));
  float y = 1.0f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t
                    + 0.254829592f) * t * std::exp(-x * x);
  return x >= 0.0f ? y : -y;
}
inline float gelu_erf(float x) { return x * 0.5f * (1.0f + erf_as(x * 0.70710678f)); }   // wgsl-ops.js:69
inline float gelu_tanh(float x) {                                                          // fused-block.js:68-75
  return 0.5f * x * (1.0f + std::tanh(0.7978845608f * (x + 0.044715f * x * x * x)));
}

// ------------------------------------------------------------------------------------------
// Dense helpers (row-major).  y[M,N] = x[M,K] . w[N,K]^T + b  (torch Linear layout, W is [out,in]).
// ------------------------------------------------------------------------------------------
void linear(const float* x, const float* w, const float* b, float* y, int M, int N, int K) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < M; ++m) {
    const float* xr = x + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const float* wr = w + (size_t)n * K;
      float s = 0.0f;
#pragma omp simd reduction(+ : s)
      for (int k = 0; k < K; ++k) s += xr[k] * wr[k];
      y[(size_t)m * N + n] = s + (b ? b[n] : 0.0f);
    }
  }
}

// Conv2d NCHW, square kernel, symmetric pad, square stride — the index math of wgsl-ops.js:584-698
// (iy = oy*S + ky - PAD) evaluated as im2col + GEMM per image.
void conv2d(const float* x, const float* w, const float* b, float* y, int N, int Ci, int H, int W,
            int Co, int K, int S, int PAD) {
  const int Ho = (H + 2 * PAD - K) / S + 1, Wo = (W + 2 * PAD - K) / S + 1;
  const int P = Ho * Wo, KD = Ci * K * K;
  std::vector<float> col((size_t)KD * P);
  for (int n = 0; n < N; ++n) {
    const float* xn = x + (size_t)n * Ci * H * W;
#pragma omp parallel for schedule(static)
    for (int kd = 0; kd < KD; ++kd) {
      const int ci = kd / (K * K), kk = kd % (K * K), ky = kk / K, kx = kk % K;
      float* cr = col.data() + (size_t)kd * P;
      for (int oy = 0; oy < Ho; ++oy)
        for (int ox = 0; ox < Wo; ++ox) {
          const int iy = oy * S + ky - PAD, ix = ox * S + kx - PAD;
          cr[oy * Wo + ox] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xn[((size_t)ci * H + iy) * W + ix] : 0.0f;
        }
    }
    float* yn = y + (size_t)n * Co * P;
#pragma omp parallel for schedule(static)
    for (int co = 0; co < Co; ++co) {
      float* yr = yn + (size_t)co * P;
      const float bias = b ? b[co] : 0.0f;
      std::vector<float> acc(P, 0.0f);
      const float* wr = w + (size_t)co * KD;
      for (int kd = 0; kd < KD; ++kd) {
        const float wv = wr[kd];
        const float* cr = col.data() + (size_t)kd * P;
        for (int p = 0; p < P; ++p) acc[p] += wv * cr[p];
      }
      for (int p = 0; p < P; ++p) yr[p] = acc[p] + bias;
    }
  }
}

// GroupNorm NCHW — wgsl-ops.js:390-458: mean = sum/gs, var = sumsq/gs - mean^2 (clamped >= 0 when
// `clamp`), inv = 1/sqrt(var + eps); the fused-groupnorm.js:145-227 / fused-resnet.js:121-166 variant
// does not clamp.  Optional SiLU epilogue (fused-resnet.js:160-161).
void group_norm(const float* x, const float* g, const float* bt, float* y, int N, int C, int HW, int G,
                float eps, int do_silu, int clamp) {
  const int cpg = C / G;
  const size_t gs = (size_t)cpg * HW;
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; ++n)
    for (int gi = 0; gi < G; ++gi) {
      const size_t base = ((size_t)n * C + (size_t)gi * cpg) * HW;
      float s = 0.0f, s2 = 0.0f;
      for (size_t i = 0; i < gs; ++i) { const float v = x[base + i]; s += v; s2 += v * v; }
      const float mean = s / (float)gs;
      float var = s2 / (float)gs - mean * mean;
      if (clamp) var = std::max(var, 0.0f);
      const float inv = 1.0f / std::sqrt(var + eps);
      for (size_t i = 0; i < gs; ++i) {
        const int c = gi * cpg + (int)(i / HW);
        float v = (x[base + i] - mean) * inv * g[c] + bt[c];
        y[base + i] = do_silu ? silu(v) : v;
      }
    }
}

// LayerNorm over the last dim, eps from caller (1e-5 in wgsl-ops.js:780 / fused-block-full.js:70).
void layer_norm(const float* x, const float* g, const float* b, float* y, int rows, int D, float eps) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * D;
    float s = 0.0f, s2 = 0.0f;
    for (int i = 0; i < D; ++i) { s += xr[i]; s2 += xr[i] * xr[i]; }
    const float mean = s / (float)D;
    const float var = std::max(s2 / (float)D - mean * mean, 0.0f);
    const float inv = 1.0f / std::sqrt(var + eps);
    for (int i = 0; i < D; ++i) y[(size_t)r * D + i] = (xr[i] - mean) * inv * g[i] + b[i];
  }
}

// Scaled-dot-product attention with full-row softmax — fused-attn.js:199-307 and
// fused-cross-attn.js:112-173: scores = q.k * 1/sqrt(d), m = max, e = exp(s - m), p = e / sum, o = p.V.
// Element (b, s, h, d) of Q/K/V/O lives at b*sb + s*ss + h*sh + d (strides in elements), which covers
// both the token-major [B,S,H*64] and the head-major [B,H,S,64] layouts.
struct AttnStrides { long long sb, ss, sh; };
void attention_rows(const float* q, const float* k, const float* v, float* o, int B, int H, int Sq, int Skv,
                    int D, AttnStrides qs, AttnStrides ks, AttnStrides os, const int* rows, int nrows,
                    bool causal = false) {
  const float scale = 1.0f / std::sqrt((float)D);
  const long long total = (long long)B * H * (rows ? nrows : Sq);
#pragma omp parallel for schedule(dynamic, 16)
  for (long long idx = 0; idx < total; ++idx) {
    const int per = rows ? nrows : Sq;
    const int bh = (int)(idx / per), qi = rows ? rows[idx % per] : (int)(idx % per);
    const int b = bh / H, h = bh % H;
    const int nk = causal ? std::min(Skv, qi + 1) : Skv;  // causal: keys 0..qi (CLIP text attention)
    std::vector<float> sc(nk);
    const float* qr = q + b * qs.sb + (long long)qi * qs.ss + h * qs.sh;
    float m = -3.4e38f;
    for (int j = 0; j < nk; ++j) {
      const float* kr = k + b * ks.sb + (long long)j * ks.ss + h * ks.sh;
      float d = 0.0f;
#pragma omp simd reduction(+ : d)
      for (int x = 0; x < D; ++x) d += qr[x] * kr[x];
      sc[j] = d * scale;
      m = std::max(m, sc[j]);
    }
    float sum = 0.0f;
    for (int j = 0; j < nk; ++j) { sc[j] = std::exp(sc[j] - m); sum += sc[j]; }
    const float inv = 1.0f / sum;
    float* orow = o + b * os.sb + (long long)qi * os.ss + h * os.sh;
    for (int x = 0; x < D; ++x) {
      float acc = 0.0f;
      for (int j = 0; j < nk; ++j) acc += sc[j] * inv * v[b * ks.sb + (long long)j * ks.ss + h * ks.sh + x];
      orow[x] = acc;
    }
  }
}

// Sinusoidal timestep embedding, fused-tembed.js:73-101: freq_i = exp(-ln(1e4) * i / half),
// emb = [cos(t f) || sin(t f)] (cos first, no frequency shift).
void sinusoid(float t, int dim, float* out) {
  const int half = dim / 2;
  const float LOG = (float)std::log(10000.0);
  for (int i = 0; i < dim; ++i) {
    const int fi = i < half ? i : i - half;
    const float freq = std::exp(-LOG * (float)fi / (float)half);
    const float arg = t * freq;
    out[i] = i < half ? std::cos(arg) : std::sin(arg);
  }
}

// ------------------------------------------------------------------------------------------
// SD2.1-architecture U-Net (SD-Turbo), NCHW fp32, weights drawn from the seeded generator and
// rounded through fp16 (the ONNX fp16 weights of the reference, converted by f16BytesToF32).
// ------------------------------------------------------------------------------------------
// Parameters by diffusers name.  kind 0 = uniform weight (fan_out > 0) or bias (fan_out == 0), 1 = norm
// gamma ~ N(1, 0.02), 2 = norm beta ~ N(0, 0.02).  mode selects the uniform bound: 0 torch layer default
// +-1/sqrt(fan_in) (weights and biases); 1 Kaiming-uniform weights +-sqrt(6/fan_in); 2 Xavier-uniform
// weights +-sqrt(6/(fan_in+fan_out)) with zero biases.  Only the most recent tensors are kept alive (each
// layer uses its parameters right after fetching them), which bounds host memory for the full U-Net.
double g_param_seconds = 0.0;  // time spent drawing parameters (excluded from CPU-baseline timings)

struct Params {
  uint64_t seed;
  bool fp16_round;
  int mode = 0;
  std::vector<std::vector<float>> store;
  size_t next = 0;
  std::unordered_map<std::string, std::vector<float>>* cache = nullptr;  // keep every tensor (repeat runs)
  const float* get(const std::string& name, size_t n, int kind, int fan_in, int fan_out = 0) {
    if (cache) {
      auto it = cache->find(name);
      if (it != cache->end() && it->second.size() == n) return it->second.data();
    }
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<float>* slotp;
    if (cache) {
      slotp = &(*cache)[name];
    } else {
      if (store.size() < 64) store.emplace_back();
      slotp = &store[next++ % 64];
    }
    std::vector<float>& slot = *slotp;
    slot.assign(n, 0.0f);
    float* p = slot.data();
    const char* nm = name.c_str();
    if (kind == 0) {
      float bound = 1.0f / std::sqrt((float)fan_in);
      if (mode == 1 && fan_out > 0) bound = std::sqrt(6.0f / (float)fan_in);
      if (mode == 2) bound = fan_out > 0 ? std::sqrt(6.0f / (float)(fan_in + fan_out)) : 0.0f;
      if (bound != 0.0f) gen_uniform(seed, nm, n, bound, p);
    } else if (kind == 1) {
      gen_normal(seed, nm, n, 1.0f, 0.02f, p);
    } else {
      gen_normal(seed, nm, n, 0.0f, 0.02f, p);
    }
    if (fp16_round) {
#pragma omp parallel for schedule(static)
      for (long long i = 0; i < (long long)n; ++i) p[i] = round_h(p[i]);
    }
    g_param_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return p;
  }
};

std::unordered_map<uint64_t, std::unordered_map<std::string, std::vector<float>>> g_unet_cache;

struct Tensor4 { int N, C, H, W; std::vector<float> d; size_t size() const { return (size_t)N * C * H * W; } };

Tensor4 t4(int N, int C, int H, int W) { Tensor4 t{N, C, H, W, {}}; t.d.assign((size_t)N * C * H * W, 0.0f); return t; }

Tensor4 conv_p(Params& P, const std::string& pre, const Tensor4& x, int Co, int K, int S) {
  const int fan = x.C * K * K;
  const float* w = P.get(pre + ".weight", (size_t)Co * fan, 0, fan, Co * K * K);
  const float* b = P.get(pre + ".bias", Co, 0, fan);
  const int pad = K / 2;
  Tensor4 y = t4(x.N, Co, (x.H + 2 * pad - K) / S + 1, (x.W + 2 * pad - K) / S + 1);
  conv2d(x.d.data(), w, b, y.d.data(), x.N, x.C, x.H, x.W, Co, K, S, pad);
  return y;
}
Tensor4 gn_p(Params& P, const std::string& pre, const Tensor4& x, float eps, bool act) {
  const float* g = P.get(pre + ".weight", x.C, 1, 1);
  const float* b = P.get(pre + ".bias", x.C, 2, 1);
  Tensor4 y = t4(x.N, x.C, x.H, x.W);
  group_norm(x.d.data(), g, b, y.d.data(), x.N, x.C, x.H * x.W, 32, eps, act ? 1 : 0, 1);
  return y;
}

// diffusers ResnetBlock2D: h = conv1(silu(gn1(x))) + proj(silu(temb)); h = conv2(silu(gn2(h)));
// out = shortcut(x) + h (1x1 conv shortcut when channels change).
Tensor4 resnet(Params& P, const std::string& pre, const Tensor4& x, const std::vector<float>& temb_silu,
               int Co) {
  Tensor4 h = gn_p(P, pre + ".norm1", x, 1e-5f, true);
  h = conv_p(P, pre + ".conv1", h, Co, 3, 1);
  {
    const int TD = (int)(temb_silu.size() / x.N);
    const float* w = P.get(pre + ".time_emb_proj.weight", (size_t)Co * TD, 0, TD, Co);
    const float* b = P.get(pre + ".time_emb_proj.bias", Co, 0, TD);
    std::vector<float> tp((size_t)x.N * Co);
    linear(temb_silu.data(), w, b, tp.data(), x.N, Co, TD);
    const int HW = h.H * h.W;
    for (int n = 0; n < h.N; ++n)
      for (int c = 0; c < Co; ++c)
        for (int i = 0; i < HW; ++i) h.d[((size_t)n * Co + c) * HW + i] += tp[(size_t)n * Co + c];
  }
  h = gn_p(P, pre + ".norm2", h, 1e-5f, true);
  h = conv_p(P, pre + ".conv2", h, Co, 3, 1);
  if (x.C != Co) {
    Tensor4 s = conv_p(P, pre + ".conv_shortcut", x, Co, 1, 1);
    for (size_t i = 0; i < h.size(); ++i) h.d[i] += s.d[i];
  } else {
    for (size_t i = 0; i < h.size(); ++i) h.d[i] += x.d[i];
  }
  return h;
}

std::vector<float> linear_p(Params& P, const std::string& pre, const std::vector<float>& x, int M, int K,
                            int N, bool bias) {
  const float* w = P.get(pre + ".weight", (size_t)N * K, 0, K, N);
  const float* b = bias ? P.get(pre + ".bias", N, 0, K) : nullptr;
  std::vector<float> y((size_t)M * N);
  linear(x.data(), w, b, y.data(), M, N, K);
  return y;
}
std::vector<float> ln_p(Params& P, const std::string& pre, const std::vector<float>& x, int rows, int D) {
  const float* g = P.get(pre + ".weight", D, 1, 1);
  const float* b = P.get(pre + ".bias", D, 2, 1);
  std::vector<float> y(x.size());
  layer_norm(x.data(), g, b, y.data(), rows, D, 1e-5f);
  return y;
}

// Multi-head attention block (diffusers Attention, head dim 64): to_q/k/v without bias, to_out with bias.
std::vector<float> attn_p(Params& P, const std::string& pre, const std::vector<float>& x, int B, int S, int C,
                          const std::vector<float>* ctx, int Sk, int Cctx) {
  const std::vector<float>& kv = ctx ? *ctx : x;
  const int Skv = ctx ? Sk : S, Ck = ctx ? Cctx : C;
  std::vector<float> q = linear_p(P, pre + ".to_q", x, B * S, C, C, false);
  std::vector<float> k = linear_p(P, pre + ".to_k", kv, B * Skv, Ck, C, false);
  std::vector<float> v = linear_p(P, pre + ".to_v", kv, B * Skv, Ck, C, false);
  std::vector<float> o((size_t)B * S * C);
  const int H = C / 64;
  AttnStrides qs{(long long)S * C, C, 64}, ks{(long long)Skv * C, C, 64};
  attention_rows(q.data(), k.data(), v.data(), o.data(), B, H, S, Skv, 64, qs, ks, qs, nullptr, 0);
  return linear_p(P, pre + ".to_out.0", o, B * S, C, C, true);
}

// BasicTransformerBlock (SD2.1): self-attn, cross-attn, GEGLU feed-forward, each pre-LN + residual.
void basic_block(Params& P, const std::string& pre, std::vector<float>& h, int B, int S, int C,
                 const std::vector<float>& ctx, int Sk, int Cctx) {
  {
    auto n = ln_p(P, pre + ".norm1", h, B * S, C);
    auto a = attn_p(P, pre + ".attn1", n, B, S, C, nullptr, 0, 0);
    for (size_t i = 0; i < h.size(); ++i) h[i] += a[i];
  }
  {
    auto n = ln_p(P, pre + ".norm2", h, B * S, C);
    auto a = attn_p(P, pre + ".attn2", n, B, S, C, &ctx, Sk, Cctx);
    for (size_t i = 0; i < h.size(); ++i) h[i] += a[i];
  }
  {
    auto n = ln_p(P, pre + ".norm3", h, B * S, C);
    const int F = 4 * C;
    auto pr = linear_p(P, pre + ".ff.net.0.proj", n, B * S, C, 2 * F, true);
    std::vector<float> g((size_t)B * S * F);
    for (long long r = 0; r < (long long)B * S; ++r)
      for (int j = 0; j < F; ++j) g[r * F + j] = pr[r * 2 * F + j] * gelu_erf(pr[r * 2 * F + F + j]);
    auto o = linear_p(P, pre + ".ff.net.2", g, B * S, F, C, true);
    for (size_t i = 0; i < h.size(); ++i) h[i] += o[i];
  }
}

// Transformer2DModel with linear proj_in / proj_out (SD2.1), GroupNorm(32, eps 1e-6).
Tensor4 transformer(Params& P, const std::string& pre, const Tensor4& x, const std::vector<float>& ctx, int Sk,
                    int Cctx) {
  const int B = x.N, C = x.C, S = x.H * x.W;
  Tensor4 n = gn_p(P, pre + ".norm", x, 1e-6f, false);
  std::vector<float> tok((size_t)B * S * C);
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C; ++c)
      for (int s = 0; s < S; ++s) tok[((size_t)b * S + s) * C + c] = n.d[((size_t)b * C + c) * S + s];
  auto h = linear_p(P, pre + ".proj_in", tok, B * S, C, C, true);
  basic_block(P, pre + ".transformer_blocks.0", h, B, S, C, ctx, Sk, Cctx);
  auto o = linear_p(P, pre + ".proj_out", h, B * S, C, C, true);
  Tensor4 y = t4(B, C, x.H, x.W);
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C; ++c)
      for (int s = 0; s < S; ++s)
        y.d[((size_t)b * C + c) * S + s] = o[((size_t)b * S + s) * C + c] + x.d[((size_t)b * C + c) * S + s];
  return y;
}

Tensor4 concat_c(const Tensor4& a, const Tensor4& b) {
  Tensor4 y = t4(a.N, a.C + b.C, a.H, a.W);
  const size_t HW = (size_t)a.H * a.W;
  for (int n = 0; n < a.N; ++n) {
    std::memcpy(&y.d[(size_t)n * y.C * HW], &a.d[(size_t)n * a.C * HW], sizeof(float) * a.C * HW);
    std::memcpy(&y.d[((size_t)n * y.C + a.C) * HW], &b.d[(size_t)n * b.C * HW], sizeof(float) * b.C * HW);
  }
  return y;
}
Tensor4 upsample2(const Tensor4& x) {  // nearest, wgsl-ops.js:921-943 index math
  Tensor4 y = t4(x.N, x.C, x.H * 2, x.W * 2);
  for (int n = 0; n < x.N; ++n)
    for (int c = 0; c < x.C; ++c)
      for (int oy = 0; oy < y.H; ++oy)
        for (int ox = 0; ox < y.W; ++ox)
          y.d[(((size_t)n * x.C + c) * y.H + oy) * y.W + ox] =
              x.d[(((size_t)n * x.C + c) * x.H + (oy * x.H) / y.H) * x.W + (ox * x.W) / y.W];
  return y;
}

}  // namespace

extern "C" {

// ---- generator / conversion -------------------------------------------------------------------
void o_gen_uniform(uint64_t seed, const char* name, size_t n, float bound, float* out) {
  gen_uniform(seed, name, n, bound, out);
}
void o_gen_normal(uint64_t seed, const char* name, size_t n, float mean, float stdv, float* out) {
  gen_normal(seed, name, n, mean, stdv, out);
}
void o_f16_to_f32(const uint16_t* h, float* f, size_t n) { for (size_t i = 0; i < n; ++i) f[i] = h2f(h[i]); }
void o_f32_to_f16(const float* f, uint16_t* h, size_t n) { for (size_t i = 0; i < n; ++i) h[i] = f2h(f[i]); }

// ---- scheduler.js restatement (JS double semantics, Float32Array stores) ------------------------
static float js_round_f32(double x) { return (float)std::floor(x + 0.5); }
void o_sched_timesteps(int n, float* out) {  // scheduler.js:69-77
  const double step = 1000.0 / n;
  for (int i = 0; i < n; ++i) out[i] = js_round_f32(1000.0 - (i + 1) * step + step) - 1.0f;
}
void o_sched_sigmas(int n, float* out /* n+1 */) {  // scheduler.js:27-59, 79-89
  std::vector<float> betas(1000), alphas(1000), sig(1000);
  const double s = std::sqrt(0.00085), e = std::sqrt(0.012);
  for (int i = 0; i < 1000; ++i) { double t = i / 999.0; double v = s + (e - s) * t; betas[i] = (float)(v * v); }
  double acc = 1.0;
  for (int i = 0; i < 1000; ++i) { acc *= 1.0 - (double)betas[i]; alphas[i] = (float)acc; }
  for (int i = 0; i < 1000; ++i) sig[i] = (float)std::sqrt((1.0 - (double)alphas[i]) / (double)alphas[i]);
  std::vector<float> ts(n);
  o_sched_timesteps(n, ts.data());
  for (int i = 0; i < n; ++i) {
    double t = ts[i];
    double v;
    if (t <= 0) v = sig[0];
    else if (t >= 999) v = sig[999];
    else { int k = (int)std::floor(t); double f = t - k; v = (double)sig[k] * (1 - f) + (double)sig[k + 1] * f; }
    out[i] = (float)v;
  }
  out[n] = 0.0f;
}
void o_sched_scale_input(const float* x, float* y, size_t n, float sigma) {  // scheduler.js:95-101
  const double s = sigma, inv = 1.0 / std::sqrt(s * s + 1.0);
  for (size_t k = 0; k < n; ++k) y[k] = (float)((double)x[k] * inv);
}
void o_sched_step(const float* x, const float* eps, float* y, size_t n, float sig_i, float sig_next) {
  const double dt = (double)sig_next - (double)sig_i;  // scheduler.js:105-110
  for (size_t k = 0; k < n; ++k) y[k] = (float)((double)x[k] + dt * (double)eps[k]);
}
void o_noise_latent(int B, int H, int W, int seed, float sigma, float* out) {  // scheduler.js:117-134
  const size_t n = (size_t)B * 4 * H * W;
  int32_t st = seed ? seed : 1;
  auto rnd = [&]() {
    st = (int32_t)((uint32_t)st * 1664525u + 1013904223u);
    return (double)(uint32_t)st / 4294967296.0;
  };
  for (size_t i = 0; i < n; i += 2) {
    double u1 = std::max(rnd(), 1e-9), u2 = rnd();
    double r = std::sqrt(-2.0 * std::log(u1));
    out[i] = (float)(r * std::cos(2.0 * M_PI * u2) * sigma);
    if (i + 1 < n) out[i + 1] = (float)(r * std::sin(2.0 * M_PI * u2) * sigma);
  }
}

// ---- wgsl-ops.js families (fp32, the reference's NCHW / cfg conventions) -----------------------
// unary op codes: 0 Sigmoid 1 Sqrt 2 Neg 3 Abs 4 Sin 5 Cos 6 Exp 7 Log 8 SiLU 9 GELU 10 Erf (wgsl-ops.js:58-72)
void o_unary(int op, const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    float r = 0;
    switch (op) {
      case 0: r = 1.0f / (1.0f + std::exp(-v)); break;
      case 1: r = std::sqrt(std::max(v, 0.0f)); break;
      case 2: r = -v; break;
      case 3: r = std::fabs(v); break;
      case 4: r = std::sin(v); break;
      case 5: r = std::cos(v); break;
      case 6: r = std::exp(v); break;
      case 7: r = std::log(std::max(v, 1e-12f)); break;
      case 8: r = silu(v); break;
      case 9: r = gelu_erf(v); break;
      case 10: r = erf_as(v); break;
    }
    y[i] = r;
  }
}
static float bin(int op, float a, float b) {  // wgsl-ops.js:130-134; 0 Add 1 Sub 2 Mul 3 Div 4 Pow 5 Max 6 Min
  switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    case 3: return a / b;
    case 4: {
      float p = std::pow(std::fabs(a), b);
      bool neg = a < 0.0f && (b - std::floor(b)) == 0.0f && (((int)b) & 1) == 1;
      return neg ? -p : p;
    }
    case 5: return std::max(a, b);
    default: return std::min(a, b);
  }
}
void o_binary(int op, const float* a, size_t na, const float* b, size_t nb, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = bin(op, a[i % na], b[i % nb]);  // wgsl-ops.js:147-151
}
static void bcast_index(const uint32_t* cfg, uint32_t i, uint32_t idx[4]) {
  uint32_t rem = i; idx[0] = idx[1] = idx[2] = idx[3] = 0;
  const uint32_t rank = cfg[0];
  if (rank >= 4) { idx[3] = rem % cfg[7]; rem /= cfg[7]; }
  if (rank >= 3) { idx[2] = rem % cfg[6]; rem /= cfg[6]; }
  if (rank >= 2) { idx[1] = rem % cfg[5]; rem /= cfg[5]; }
  idx[0] = rem;
}
void o_binary_bcast(int op, const float* a, const float* b, float* y, const uint32_t* cfg) {  // :156-201
  for (uint32_t i = 0; i < cfg[16]; ++i) {
    uint32_t idx[4]; bcast_index(cfg, i, idx);
    uint32_t ao = 0, bo = 0;
    for (int d = 0; d < 4; ++d) { ao += idx[d] * cfg[8 + d]; bo += idx[d] * cfg[12 + d]; }
    y[i] = bin(op, a[ao], b[bo]);
  }
}
void o_affine_bcast(const float* a, const float* g, const float* bt, float* y, const uint32_t* cfg) {  // :206-248
  for (uint32_t i = 0; i < cfg[16]; ++i) {
    uint32_t idx[4]; bcast_index(cfg, i, idx);
    uint32_t ao = 0, bo = 0;
    for (int d = 0; d < 4; ++d) { ao += idx[d] * cfg[8 + d]; bo += idx[d] * cfg[12 + d]; }
    y[i] = a[ao] * g[bo] + bt[bo];
  }
}
void o_softmax(const float* x, float* y, uint32_t inner, uint32_t rows) {  // :266-283
  for (uint32_t r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * inner;
    float m = -1e30f;
    for (uint32_t j = 0; j < inner; ++j) m = std::max(m, xr[j]);
    float s = 0.0f;
    for (uint32_t j = 0; j < inner; ++j) s += std::exp(xr[j] - m);
    const float inv = 1.0f / s;
    for (uint32_t j = 0; j < inner; ++j) y[(size_t)r * inner + j] = std::exp(xr[j] - m) * inv;
  }
}
void o_instance_norm(const float* x, const float* g, const float* b, float* y, uint32_t C, uint32_t HW,
                     uint32_t N) {  // :307-372, eps hard-coded 1e-5
  std::vector<float> gg(C), bb(C);
  for (uint32_t c = 0; c < C; ++c) { gg[c] = g[c]; bb[c] = b[c]; }
  group_norm(x, gg.data(), bb.data(), y, (int)N, (int)C, (int)HW, (int)C, 1e-5f, 0, 1);
}
void o_group_norm(const float* x, const float* g, const float* b, float* y, int N, int C, int HW, int G,
                  float eps, int do_silu, int clamp) {
  group_norm(x, g, b, y, N, C, HW, G, eps, do_silu, clamp);
}
void o_layer_norm(const float* x, const float* g, const float* b, float* y, int rows, int D, float eps) {
  layer_norm(x, g, b, y, rows, D, eps);
}
void o_matmul(const float* A, const float* Bm, float* Y, int M, int N, int K, int bBatched, int batch) {
  // wgsl-ops.js:477-556: Y[z] = A[z] . B[z or 0], B row-major [K,N].
#pragma omp parallel for collapse(2) schedule(static)
  for (int z = 0; z < batch; ++z)
    for (int r = 0; r < M; ++r) {
      const float* a = A + ((size_t)z * M + r) * K;
      const float* bz = Bm + (bBatched ? (size_t)z * K * N : 0);
      float* yr = Y + ((size_t)z * M + r) * N;
      for (int c = 0; c < N; ++c) {
        float s = 0.0f;
        for (int k = 0; k < K; ++k) s += a[k] * bz[(size_t)k * N + c];
        yr[c] = s;
      }
    }
}
void o_gemm(const float* A, const float* Bm, const float* C, float* Y, int M, int N, int K, int transB) {
  // wgsl-ops.js:821-897: Y = A.B (+C[col]); transB=1 reads B as [N,K].
#pragma omp parallel for schedule(static)
  for (int r = 0; r < M; ++r)
    for (int c = 0; c < N; ++c) {
      float s = 0.0f;
      for (int k = 0; k < K; ++k) s += A[(size_t)r * K + k] * (transB ? Bm[(size_t)c * K + k] : Bm[(size_t)k * N + c]);
      Y[(size_t)r * N + c] = s + C[c];
    }
}
void o_conv(const float* x, const float* w, const float* b, float* y, int N, int Ci, int H, int W, int Co,
            int K, int S, int PAD) {
  conv2d(x, w, b, y, N, Ci, H, W, Co, K, S, PAD);
}
void o_resize_nearest(const float* x, float* y, const uint32_t* cfg) {  // :921-943, cfg[8]
  const uint32_t Hi = cfg[1], Wi = cfg[2], Ho = cfg[3], Wo = cfg[4], n = cfg[5];
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t ox = i % Wo, t = i / Wo, oy = t % Ho, oc = t / Ho;
    y[i] = x[(oc * Hi + (oy * Hi) / Ho) * Wi + (ox * Wi) / Wo];
  }
}
void o_reduce_mean(const float* x, float* y, uint32_t inner, uint32_t rows) {  // :958-973
  for (uint32_t r = 0; r < rows; ++r) {
    float s = 0.0f;
    for (uint32_t j = 0; j < inner; ++j) s += x[(size_t)r * inner + j];
    y[r] = s / (float)inner;
  }
}
void o_transpose(const float* x, float* y, const uint32_t* cfg) {  // :993-1032, cfg u32[20]
  for (uint32_t i = 0; i < cfg[16]; ++i) {
    uint32_t o[4]; bcast_index(cfg, i, o);
    uint32_t in[4] = {0, 0, 0, 0};
    for (uint32_t k = 0; k < cfg[0]; ++k) in[cfg[12 + k]] = o[k];
    uint32_t off = 0;
    for (int d = 0; d < 4; ++d) off += in[d] * cfg[8 + d];
    y[i] = x[off];
  }
}
void o_pow_scalar(const float* x, float* y, size_t n, float e) {  // :1050-1075
  const float ei = std::floor(e);
  const bool isInt = std::fabs(e - ei) < 1e-6f;
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    if (v < 0.0f && !isInt) { y[i] = 0.0f; continue; }
    const float s = (v < 0.0f && (((int)ei) & 1) == 1) ? -1.0f : 1.0f;
    y[i] = s * std::pow(std::fabs(v), e);
  }
}
void o_slice(const float* x, float* y, const uint32_t* cfg) {  // :1092-1124
  for (uint32_t i = 0; i < cfg[16]; ++i) {
    uint32_t o[4]; bcast_index(cfg, i, o);
    uint32_t off = 0;
    for (int d = 0; d < 4; ++d) off += (cfg[12 + d] + o[d]) * cfg[8 + d];
    y[i] = x[off];
  }
}
void o_concat_copy(const float* x, float* y, const uint32_t* cfg) {  // :1142-1157, cfg[4]
  for (uint32_t i = 0; i < cfg[3]; ++i) y[(i / cfg[0]) * cfg[1] + cfg[2] + i % cfg[0]] = x[i];
}

// ---- fused blocks ------------------------------------------------------------------------------
void o_attention(const float* q, const float* k, const float* v, float* o, int B, int H, int Sq, int Skv,
                 int layout /*0: [B,S,H,64] token-major, 1: [B,H,S,64] head-major*/, const int* rows, int nrows) {
  AttnStrides qs, ks;
  if (layout == 0) { qs = {(long long)Sq * H * 64, H * 64, 64}; ks = {(long long)Skv * H * 64, H * 64, 64}; }
  else { qs = {(long long)H * Sq * 64, 64, (long long)Sq * 64}; ks = {(long long)H * Skv * 64, 64, (long long)Skv * 64}; }
  attention_rows(q, k, v, o, B, H, Sq, Skv, 64, qs, ks, qs, rows, nrows);
}
void o_attention_causal(const float* q, const float* k, const float* v, float* o, int B, int H, int S, int layout) {
  AttnStrides st;
  if (layout == 0) st = {(long long)S * H * 64, H * 64, 64};
  else st = {(long long)H * S * 64, 64, (long long)S * 64};
  attention_rows(q, k, v, o, B, H, S, S, 64, st, st, st, nullptr, 0, true);
}

// fused-tembed.js:73-130: y = W2 . silu(W1 . [cos||sin](t f) + b1) + b2, W row-major [out,in].
void o_tembed(const float* t, int B, const float* W1, const float* b1, const float* W2, const float* b2,
              int Din, int Dh, float* out) {
  std::vector<float> e((size_t)B * Din), h((size_t)B * Dh);
  for (int b = 0; b < B; ++b) sinusoid(t[b], Din, &e[(size_t)b * Din]);
  linear(e.data(), W1, b1, h.data(), B, Dh, Din);
  for (auto& v : h) v = silu(v);
  linear(h.data(), W2, b2, out, B, Dh, Dh);
}

// Config-1 ResNet block (fused-resnet.js:121-208 plus the timestep add it omits, fused-resnet.js:9-12):
// y = conv2(silu(GN2(conv1(silu(GN1(x))) + Wt.temb + bt))) + x, GN(32, eps), NCHW fp32.
void o_resnet_block(const float* x, const float* temb, int N, int C, int H, int W, int Tdim,
                    const float* g1, const float* be1, const float* w1, const float* bb1,
                    const float* wt, const float* bt,
                    const float* g2, const float* be2, const float* w2, const float* bb2, float eps,
                    int temb_silu, float* y) {
  const size_t n = (size_t)N * C * H * W;
  std::vector<float> a(n), b(n);
  group_norm(x, g1, be1, a.data(), N, C, H * W, 32, eps, 1, 1);
  conv2d(a.data(), w1, bb1, b.data(), N, C, H, W, C, 3, 1, 1);
  std::vector<float> ts((size_t)N * Tdim), tp((size_t)N * C);
  for (size_t i = 0; i < ts.size(); ++i) ts[i] = temb_silu ? silu(temb[i]) : temb[i];
  linear(ts.data(), wt, bt, tp.data(), N, C, Tdim);
  for (int nn = 0; nn < N; ++nn)
    for (int c = 0; c < C; ++c)
      for (int i = 0; i < H * W; ++i) b[((size_t)nn * C + c) * H * W + i] += tp[(size_t)nn * C + c];
  group_norm(b.data(), g2, be2, a.data(), N, C, H * W, 32, eps, 1, 1);
  conv2d(a.data(), w2, bb2, y, N, C, H, W, C, 3, 1, 1);
  for (size_t i = 0; i < n; ++i) y[i] += x[i];
}

// Config-2 SD2.1 transformer block (Transformer2DModel with one BasicTransformerBlock), token-major
// hidden [B,S,C] in and out; weights by name from the seeded generator (fp16-rounded when asked).
void o_transformer_block(const float* hidden, const float* ctx, int B, int S, int C, int Sk, int Cctx,
                         uint64_t seed, int fp16_weights, float* out) {
  Params P{seed, fp16_weights != 0, 2, {}, 0};  // Xavier-uniform weights, zero biases (config 2)
  Tensor4 x = t4(B, C, S, 1);
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s)
      for (int c = 0; c < C; ++c) x.d[((size_t)b * C + c) * S + s] = hidden[((size_t)b * S + s) * C + c];
  std::vector<float> cv(ctx, ctx + (size_t)B * Sk * Cctx);
  Tensor4 y = transformer(P, "block", x, cv, Sk, Cctx);
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s)
      for (int c = 0; c < C; ++c) out[((size_t)b * S + s) * C + c] = y.d[((size_t)b * C + c) * S + s];
}

// Config-4 U-Net forward (SD2.1 / SD-Turbo layout: 320/640/1280/1280, 2 resnets per level, transformer
// at the first three levels, head dim 64, cross-attn dim 1024).  latent [B,4,H,W] NCHW, t per image,
// ctx [B,Sk,1024]; out [B,4,H,W].
void o_unet_forward(const float* latent, const float* tvals, const float* ctx, int B, int H, int W, int Sk,
                    uint64_t seed, float* out) {
  Params P{seed, true, 0, {}, 0, &g_unet_cache[seed]};
  const int ch[4] = {320, 640, 1280, 1280};
  const int Cctx = 1024;
  std::vector<float> cv(ctx, ctx + (size_t)B * Sk * Cctx);
  // time embedding
  std::vector<float> e((size_t)B * 320);
  for (int b = 0; b < B; ++b) sinusoid(tvals[b], 320, &e[(size_t)b * 320]);
  auto t1 = linear_p(P, "time_embedding.linear_1", e, B, 320, 1280, true);
  for (auto& v : t1) v = silu(v);
  auto temb = linear_p(P, "time_embedding.linear_2", t1, B, 1280, 1280, true);
  std::vector<float> temb_s = temb;
  for (auto& v : temb_s) v = silu(v);

  Tensor4 x = t4(B, 4, H, W);
  std::memcpy(x.d.data(), latent, sizeof(float) * x.size());
  Tensor4 h = conv_p(P, "conv_in", x, 320, 3, 1);
  std::vector<Tensor4> skips;
  skips.push_back(h);
  for (int i = 0; i < 4; ++i) {
    for (int j = 0; j < 2; ++j) {
      const std::string pre = "down_blocks." + std::to_string(i);
      h = resnet(P, pre + ".resnets." + std::to_string(j), h, temb_s, ch[i]);
      if (i < 3) h = transformer(P, pre + ".attentions." + std::to_string(j), h, cv, Sk, Cctx);
      skips.push_back(h);
    }
    if (i < 3) {
      h = conv_p(P, "down_blocks." + std::to_string(i) + ".downsamplers.0.conv", h, ch[i], 3, 2);
      skips.push_back(h);
    }
  }
  h = resnet(P, "mid_block.resnets.0", h, temb_s, 1280);
  h = transformer(P, "mid_block.attentions.0", h, cv, Sk, Cctx);
  h = resnet(P, "mid_block.resnets.1", h, temb_s, 1280);
  const int rch[4] = {1280, 1280, 640, 320};
  for (int i = 0; i < 4; ++i) {
    const std::string pre = "up_blocks." + std::to_string(i);
    for (int j = 0; j < 3; ++j) {
      Tensor4 s = skips.back();
      skips.pop_back();
      h = concat_c(h, s);
      h = resnet(P, pre + ".resnets." + std::to_string(j), h, temb_s, rch[i]);
      if (i > 0) h = transformer(P, pre + ".attentions." + std::to_string(j), h, cv, Sk, Cctx);
    }
    if (i < 3) h = conv_p(P, pre + ".upsamplers.0.conv", upsample2(h), rch[i], 3, 1);
  }
  h = gn_p(P, "conv_norm_out", h, 1e-5f, true);
  h = conv_p(P, "conv_out", h, 4, 3, 1);
  std::memcpy(out, h.d.data(), sizeof(float) * h.size());
}

// ---- SD VAE decoder (diffusers AutoencoderKL.decode; vae-wgsl.js:99-118 applies latent / 0.18215) ------
Tensor4 resnet_nt(Params& P, const std::string& pre, const Tensor4& x, int Co, float eps) {
  Tensor4 h = gn_p(P, pre + ".norm1", x, eps, true);
  h = conv_p(P, pre + ".conv1", h, Co, 3, 1);
  h = gn_p(P, pre + ".norm2", h, eps, true);
  h = conv_p(P, pre + ".conv2", h, Co, 3, 1);
  if (x.C != Co) {
    Tensor4 s = conv_p(P, pre + ".conv_shortcut", x, Co, 1, 1);
    for (size_t i = 0; i < h.size(); ++i) h.d[i] += s.d[i];
  } else {
    for (size_t i = 0; i < h.size(); ++i) h.d[i] += x.d[i];
  }
  return h;
}

// diffusers Attention in the VAE mid block: GroupNorm(32, 1e-6), one head of C channels (scale 1/sqrt(C)),
// biased q / k / v / out projections, residual.
Tensor4 vae_attn(Params& P, const std::string& pre, const Tensor4& x) {
  Tensor4 nx = gn_p(P, pre + ".group_norm", x, 1e-6f, false);
  const int N = x.N, C = x.C, HW = x.H * x.W;
  std::vector<float> tok((size_t)N * HW * C);
  for (int n = 0; n < N; ++n)
    for (int c = 0; c < C; ++c)
      for (int p = 0; p < HW; ++p) tok[((size_t)n * HW + p) * C + c] = nx.d[((size_t)n * C + c) * HW + p];
  auto q = linear_p(P, pre + ".to_q", tok, N * HW, C, C, true);
  auto k = linear_p(P, pre + ".to_k", tok, N * HW, C, C, true);
  auto v = linear_p(P, pre + ".to_v", tok, N * HW, C, C, true);
  std::vector<float> o((size_t)N * HW * C);
  const AttnStrides st{(long long)HW * C, C, 0};
  attention_rows(q.data(), k.data(), v.data(), o.data(), N, 1, HW, HW, C, st, st, st, nullptr, 0);
  auto y = linear_p(P, pre + ".to_out.0", o, N * HW, C, C, true);
  Tensor4 out = x;
  for (int n = 0; n < N; ++n)
    for (int c = 0; c < C; ++c)
      for (int p = 0; p < HW; ++p) out.d[((size_t)n * C + c) * HW + p] += y[((size_t)n * HW + p) * C + c];
  return out;
}

std::unordered_map<uint64_t, std::unordered_map<std::string, std::vector<float>>> g_vae_cache;

void o_vae_decode(const float* latent, int B, int h, int w, uint64_t seed, float* image) {
  Params P{seed, true, 0, {}, 0, &g_vae_cache[seed]};
  Tensor4 z = t4(B, 4, h, w);
  for (size_t i = 0; i < z.size(); ++i) z.d[i] = (float)((double)latent[i] / 0.18215);
  z = conv_p(P, "post_quant_conv", z, 4, 1, 1);
  Tensor4 x = conv_p(P, "decoder.conv_in", z, 512, 3, 1);
  x = resnet_nt(P, "decoder.mid_block.resnets.0", x, 512, 1e-6f);
  x = vae_attn(P, "decoder.mid_block.attentions.0", x);
  x = resnet_nt(P, "decoder.mid_block.resnets.1", x, 512, 1e-6f);
  const int ch[4] = {512, 512, 256, 128};
  for (int i = 0; i < 4; ++i) {
    const std::string pre = "decoder.up_blocks." + std::to_string(i);
    for (int j = 0; j < 3; ++j) x = resnet_nt(P, pre + ".resnets." + std::to_string(j), x, ch[i], 1e-6f);
    if (i < 3) x = conv_p(P, pre + ".upsamplers.0.conv", upsample2(x), ch[i], 3, 1);
  }
  x = gn_p(P, "decoder.conv_norm_out", x, 1e-6f, true);
  x = conv_p(P, "decoder.conv_out", x, 3, 3, 1);
  std::memcpy(image, x.d.data(), sizeof(float) * x.size());
}

// ---- OpenCLIP ViT-H text encoder (SD2.x / SD-Turbo; ONNX Runtime in the reference, text-encoder.js:
// 69-174).  HF CLIPTextModel: x = token_embedding[ids] + position_embedding; per layer
// x += out_proj(causal_attn(q/k/v_proj(LN1(x)))), x += fc2(gelu(fc1(LN2(x)))); final LayerNorm.
// GELU is the erf form of wgsl-ops.js:69 (the ONNX export's Erf op runs through the A&S erf there).
std::unordered_map<uint64_t, std::unordered_map<std::string, std::vector<float>>> g_text_cache;

void o_text_encode(const int32_t* ids, int B, int S, int layers, uint64_t seed, float* out) {
  Params P{seed, true, 0, {}, 0, &g_text_cache[seed]};
  const int D = 1024, F = 4096, V = 49408, H = 16, M = B * S;
  const float* tok = P.get("text_model.embeddings.token_embedding.weight", (size_t)V * D, 2, 1);
  const float* pos = P.get("text_model.embeddings.position_embedding.weight", (size_t)77 * D, 2, 1);
  std::vector<float> x((size_t)M * D);
  for (int t = 0; t < M; ++t)
    for (int c = 0; c < D; ++c) x[(size_t)t * D + c] = tok[(size_t)ids[t] * D + c] + pos[(size_t)(t % S) * D + c];
  for (int l = 0; l < layers; ++l) {
    const std::string pre = "text_model.encoder.layers." + std::to_string(l);
    auto n = ln_p(P, pre + ".layer_norm1", x, M, D);
    auto q = linear_p(P, pre + ".self_attn.q_proj", n, M, D, D, true);
    auto k = linear_p(P, pre + ".self_attn.k_proj", n, M, D, D, true);
    auto v = linear_p(P, pre + ".self_attn.v_proj", n, M, D, D, true);
    std::vector<float> o((size_t)M * D);
    const AttnStrides st{(long long)S * D, D, 64};
    attention_rows(q.data(), k.data(), v.data(), o.data(), B, H, S, S, 64, st, st, st, nullptr, 0, true);
    auto y = linear_p(P, pre + ".self_attn.out_proj", o, M, D, D, true);
    for (size_t i = 0; i < x.size(); ++i) x[i] += y[i];
    n = ln_p(P, pre + ".layer_norm2", x, M, D);
    auto h = linear_p(P, pre + ".mlp.fc1", n, M, D, F, true);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)h.size(); ++i) h[i] = gelu_erf(h[i]);
    y = linear_p(P, pre + ".mlp.fc2", h, M, F, D, true);
    for (size_t i = 0; i < x.size(); ++i) x[i] += y[i];
  }
  x = ln_p(P, "text_model.final_layer_norm", x, M, D);
  std::memcpy(out, x.data(), sizeof(float) * x.size());
}

double o_param_seconds() { return g_param_seconds; }
void o_clear_cache() {
  g_text_cache.clear();
  g_unet_cache.clear();
  g_vae_cache.clear();
}

void o_set_threads(int n) {  // torchrun sets OMP_NUM_THREADS=1 for multi-process jobs; the baseline uses all cores
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
int o_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
