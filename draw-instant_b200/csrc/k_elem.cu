// k_elem.cu — the reference's elementwise / layout op families (wgsl-ops.js:58-1168) plus the small
// GEMV-shaped kernels (timestep embedding, fused-tembed.js:73-130) and layout converters the fused
// blocks need.  All are HBM- or latency-bound: grid-stride loops sized to a multiple of the SM count,
// one warp per row for row reductions, index math in 32-bit like the reference's u32 cfg blocks.
#include <algorithm>

#include "di_common.cuh"

namespace di {

Ctx* ctx_of(di_ctx_t h);
void* workspace(Ctx* c, size_t bytes, int slot);

namespace {

inline int grid_for(Ctx* c, size_t n, int threads = 256) {
  return (int)std::max<size_t>(1, std::min<size_t>((n + threads - 1) / threads, (size_t)16 * c->num_sms));
}

__device__ __forceinline__ float unary_op(int op, float x) {
  switch (op) {
    case DI_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case DI_SQRT: return sqrtf(fmaxf(x, 0.0f));
    case DI_NEG: return -x;
    case DI_ABS: return fabsf(x);
    case DI_SIN: return sinf(x);
    case DI_COS: return cosf(x);
    case DI_EXP: return expf(x);
    case DI_LOG: return logf(fmaxf(x, 1e-12f));
    case DI_SILU: return x / (1.0f + expf(-x));
    case DI_GELU: return gelu_erf(x);
    default: return erf_as(x);  // DI_ERF
  }
}
__device__ __forceinline__ float binary_op(int op, float a, float b) {
  switch (op) {
    case DI_ADD: return a + b;
    case DI_SUB: return a - b;
    case DI_MUL: return a * b;
    case DI_DIV: return a / b;
    case DI_POW: {
      const float p = powf(fabsf(a), b);
      const bool neg = a < 0.0f && (b - floorf(b)) == 0.0f && ((int)b & 1) == 1;
      return neg ? -p : p;
    }
    case DI_MAX: return fmaxf(a, b);
    default: return fminf(a, b);
  }
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y, uint32_t n) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = unary_op(op, x[i]);
}
__global__ void binary_kernel(int op, const float* __restrict__ a, uint32_t na, const float* __restrict__ b,
                              uint32_t nb, float* __restrict__ y, uint32_t n) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = binary_op(op, a[i % na], b[i % nb]);
}

struct Cfg20 { uint32_t v[20]; };

__device__ __forceinline__ void decompose(const Cfg20& c, uint32_t i, uint32_t idx[4]) {
  uint32_t rem = i;
  idx[0] = idx[1] = idx[2] = idx[3] = 0;
  if (c.v[0] >= 4) { idx[3] = rem % c.v[7]; rem /= c.v[7]; }
  if (c.v[0] >= 3) { idx[2] = rem % c.v[6]; rem /= c.v[6]; }
  if (c.v[0] >= 2) { idx[1] = rem % c.v[5]; rem /= c.v[5]; }
  idx[0] = rem;
}

__global__ void binary_bcast_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                    float* __restrict__ y, Cfg20 c) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.v[16]; i += gridDim.x * blockDim.x) {
    uint32_t idx[4];
    decompose(c, i, idx);
    uint32_t ao = 0, bo = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) { ao += idx[d] * c.v[8 + d]; bo += idx[d] * c.v[12 + d]; }
    y[i] = binary_op(op, a[ao], b[bo]);
  }
}
__global__ void affine_bcast_kernel(const float* __restrict__ a, const float* __restrict__ g,
                                    const float* __restrict__ bt, float* __restrict__ y, Cfg20 c) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.v[16]; i += gridDim.x * blockDim.x) {
    uint32_t idx[4];
    decompose(c, i, idx);
    uint32_t ao = 0, bo = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) { ao += idx[d] * c.v[8 + d]; bo += idx[d] * c.v[12 + d]; }
    y[i] = a[ao] * g[bo] + bt[bo];
  }
}
__global__ void transpose_kernel(const float* __restrict__ x, float* __restrict__ y, Cfg20 c) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.v[16]; i += gridDim.x * blockDim.x) {
    uint32_t o[4];
    decompose(c, i, o);
    uint32_t in[4] = {0, 0, 0, 0};
    for (uint32_t k = 0; k < c.v[0] && k < 4; ++k) in[c.v[12 + k] & 3] = o[k];
    uint32_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) off += in[d] * c.v[8 + d];
    y[i] = x[off];
  }
}
__global__ void slice_kernel(const float* __restrict__ x, float* __restrict__ y, Cfg20 c) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < c.v[16]; i += gridDim.x * blockDim.x) {
    uint32_t o[4];
    decompose(c, i, o);
    uint32_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) off += (c.v[12 + d] + o[d]) * c.v[8 + d];
    y[i] = x[off];
  }
}

// Softmax / ReduceMean over the last dim: one warp per row.
__global__ void softmax_rows(const float* __restrict__ x, float* __restrict__ y, uint32_t inner, uint32_t rows) {
  pdl_begin();
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * inner;
  float m = -1e30f;
  for (uint32_t j = lane; j < inner; j += 32) m = fmaxf(m, xr[j]);
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(~0u, m, o));
  float s = 0.f;
  for (uint32_t j = lane; j < inner; j += 32) s += expf(xr[j] - m);
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(~0u, s, o);
  const float inv = 1.0f / s;
  for (uint32_t j = lane; j < inner; j += 32) y[(size_t)row * inner + j] = expf(xr[j] - m) * inv;
}
__global__ void reduce_mean_rows(const float* __restrict__ x, float* __restrict__ y, uint32_t inner, uint32_t rows) {
  pdl_begin();
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f;
  for (uint32_t j = lane; j < inner; j += 32) s += x[(size_t)row * inner + j];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(~0u, s, o);
  if (lane == 0) y[row] = s / (float)inner;
}

__global__ void resize_nearest_kernel(const float* __restrict__ x, float* __restrict__ y, uint32_t Hi, uint32_t Wi,
                                      uint32_t Ho, uint32_t Wo, uint32_t n) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t ox = i % Wo, t = i / Wo, oy = t % Ho, oc = t / Ho;
    y[i] = x[(oc * Hi + (oy * Hi) / Ho) * Wi + (ox * Wi) / Wo];
  }
}
__global__ void pow_scalar_kernel(const float* __restrict__ x, float* __restrict__ y, float e, uint32_t n) {
  pdl_begin();
  const float ei = floorf(e);
  const bool is_int = fabsf(e - ei) < 1e-6f;
  const bool odd = ((int)ei & 1) == 1;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = x[i];
    if (v < 0.0f && !is_int) { y[i] = 0.0f; continue; }
    const float s = (v < 0.0f && odd) ? -1.0f : 1.0f;
    y[i] = s * powf(fabsf(v), e);
  }
}
__global__ void concat_copy_kernel(const float* __restrict__ x, float* __restrict__ y, uint32_t stripe_in,
                                   uint32_t stripe_out, uint32_t off, uint32_t n) {
  pdl_begin();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[(i / stripe_in) * stripe_out + off + i % stripe_in] = x[i];
}

// Timestep embedding stage 1: h[b][o] = silu(W1[o] . [cos||sin](t_b f) + b1[o]); one warp per output o.
__global__ void tembed_stage1(const float* __restrict__ t, int B, const float* __restrict__ W1,
                              const float* __restrict__ b1, int Din, int Dh, float* __restrict__ h) {
  pdl_begin();
  extern __shared__ float emb[];  // [B][Din]
  const int half = Din / 2;
  const float LOG = 9.210340371976184f;  // ln(10000)
  for (int i = threadIdx.x; i < B * Din; i += blockDim.x) {
    const int b = i / Din, k = i % Din;
    const int fi = k < half ? k : k - half;
    const float freq = expf(-LOG * (float)fi / (float)half);
    const float arg = t[b] * freq;
    emb[i] = k < half ? cosf(arg) : sinf(arg);
  }
  __syncthreads();
  const int o = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (o >= Dh) return;
  for (int b = 0; b < B; ++b) {
    float s = 0.f;
    for (int k = lane; k < Din; k += 32) s += W1[(size_t)o * Din + k] * emb[b * Din + k];
    for (int q = 16; q; q >>= 1) s += __shfl_xor_sync(~0u, s, q);
    if (lane == 0) h[(size_t)b * Dh + o] = silu_f(s + b1[o]);
  }
}

}  // namespace

// y[b][n] = act_out(W[n] . act_in(x[b]) + bias[n]) for b < B; W [N,K] fp32 or fp16; one warp per n.
template <typename TW>
__global__ void gemv_rows(const float* __restrict__ x, int B, int K, const TW* __restrict__ W,
                          const float* __restrict__ bias, int N, int silu_in, float* __restrict__ y, int ldy) {
  pdl_begin();
  extern __shared__ float xs[];  // [B][K]
  for (int i = threadIdx.x; i < B * K; i += blockDim.x) {
    const float v = x[i];
    xs[i] = silu_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int n = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (n >= N) return;
  for (int b = 0; b < B; ++b) {
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += to_f<TW>(W[(size_t)n * K + k]) * xs[b * K + k];
    for (int q = 16; q; q >>= 1) s += __shfl_xor_sync(~0u, s, q);
    if (lane == 0) y[(size_t)b * ldy + n] = s + (bias ? bias[n] : 0.0f);
  }
}

int gemv(Ctx* c, const float* x, int B, int K, const void* W, int w_f16, const float* bias, int N, int silu_in,
         float* y, int ldy) {
  const size_t shm = sizeof(float) * (size_t)B * K;
  if (shm > 200 * 1024) return set_error(c, DI_EUNSUPPORTED, "gemv: input too large");
  if (shm > 48 * 1024) {
    cudaFuncSetAttribute(gemv_rows<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm);
    cudaFuncSetAttribute(gemv_rows<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm);
  }
  const int blocks = (N + 7) / 8;
  if (w_f16)
    launch_k(gemv_rows<__half>, blocks, 256, shm, c->stream, x, B, K, static_cast<const __half*>(W), bias, N, silu_in, y, ldy);
  else
    launch_k(gemv_rows<float>, blocks, 256, shm, c->stream, x, B, K, static_cast<const float*>(W), bias, N, silu_in, y, ldy);
  return check_launch(c, "gemv");
}

int tembed(Ctx* c, const float* t, int B, const float* W1, const float* b1, const float* W2, const float* b2, int Din,
           int Dh, float* hidden, float* y) {
  const size_t shm = sizeof(float) * (size_t)B * Din;
  if (shm > 48 * 1024 || Din % 2) return set_error(c, DI_EUNSUPPORTED, "tembed: sizes");
  launch_k(tembed_stage1, (Dh + 7) / 8, 256, shm, c->stream, t, B, W1, b1, Din, Dh, hidden);
  int r = check_launch(c, "tembed_stage1");
  if (r) return r;
  return gemv(c, hidden, B, Dh, W2, 0, b2, Dh, 0, y, Dh);
}

// Layout converters for the NCHW fp32 drop-ins: [N][C][HW] <-> [N][HW][C] through a 32x32 smem tile.
template <typename Tin, typename Tout>
__global__ void nchw_to_nhwc_kernel(const Tin* __restrict__ x, Tout* __restrict__ y, int C, int HW) {
  pdl_begin();
  __shared__ float tile[32][33];
  const int n = blockIdx.z, c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, p = p0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && p < HW) ? to_f<Tin>(x[((size_t)n * C + c) * HW + p]) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = p0 + i, c = c0 + threadIdx.x;
    if (c < C && p < HW) y[((size_t)n * HW + p) * C + c] = from_f<Tout>(tile[threadIdx.x][i]);
  }
}
template <typename Tin, typename Tout>
__global__ void nhwc_to_nchw_kernel(const Tin* __restrict__ x, Tout* __restrict__ y, int C, int HW) {
  pdl_begin();
  __shared__ float tile[32][33];
  const int n = blockIdx.z, c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = p0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && p < HW) ? to_f<Tin>(x[((size_t)n * HW + p) * C + c]) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, p = p0 + threadIdx.x;
    if (c < C && p < HW) y[((size_t)n * C + c) * HW + p] = from_f<Tout>(tile[threadIdx.x][i]);
  }
}

int nchw_to_nhwc(Ctx* c, int in_dt, int out_dt, const void* x, void* y, int N, int C, int HW) {
  dim3 grid((HW + 31) / 32, (C + 31) / 32, N), block(32, 8);
#define NC_CASE(TI, TO) \
  launch_k(nchw_to_nhwc_kernel<TI, TO>, grid, block, 0, c->stream, static_cast<const TI*>(x), static_cast<TO*>(y), C, HW)
  if (in_dt == DI_F32 && out_dt == DI_F32) NC_CASE(float, float);
  else if (in_dt == DI_F32 && out_dt == DI_F16) NC_CASE(float, __half);
  else if (in_dt == DI_F32 && out_dt == DI_BF16) NC_CASE(float, __nv_bfloat16);
  else if (in_dt == DI_F16 && out_dt == DI_F16) NC_CASE(__half, __half);
  else return set_error(c, DI_EINVAL, "nchw_to_nhwc dtype");
#undef NC_CASE
  return check_launch(c, "nchw_to_nhwc");
}
int nhwc_to_nchw(Ctx* c, int in_dt, int out_dt, const void* x, void* y, int N, int C, int HW) {
  dim3 grid((HW + 31) / 32, (C + 31) / 32, N), block(32, 8);
#define CN_CASE(TI, TO) \
  launch_k(nhwc_to_nchw_kernel<TI, TO>, grid, block, 0, c->stream, static_cast<const TI*>(x), static_cast<TO*>(y), C, HW)
  if (in_dt == DI_F32 && out_dt == DI_F32) CN_CASE(float, float);
  else if (in_dt == DI_F16 && out_dt == DI_F32) CN_CASE(__half, float);
  else if (in_dt == DI_BF16 && out_dt == DI_F32) CN_CASE(__nv_bfloat16, float);
  else if (in_dt == DI_F16 && out_dt == DI_F16) CN_CASE(__half, __half);
  else return set_error(c, DI_EINVAL, "nhwc_to_nchw dtype");
#undef CN_CASE
  return check_launch(c, "nhwc_to_nchw");
}

// fp32 -> fp16/bf16 cast with optional zero padding of each row to ld_out columns.
template <typename TO>
__global__ void cast_rows_kernel(const float* __restrict__ x, int rows, int cols, int ld_in, TO* __restrict__ y,
                                 int ld_out, int transpose) {
  pdl_begin();
  const size_t total = (size_t)rows * ld_out;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = i / ld_out, k = i % ld_out;
    float v = 0.f;
    if (k < cols) v = transpose ? x[(size_t)k * ld_in + r] : x[(size_t)r * ld_in + k];
    y[i] = from_f<TO>(v);
  }
}
// Writes y[rows][ld_out] (zero padded) from x either row-major [rows][cols] (transpose=0, row stride ld_in)
// or column-major x[cols][rows] (transpose=1, i.e. x[k][r] with row stride ld_in).
int cast_rows_f16(Ctx* c, const float* x, int rows, int cols, int ld_in, void* y, int ld_out, int transpose) {
  const size_t total = (size_t)rows * ld_out;
  launch_k(cast_rows_kernel<__half>, grid_for(c, total), 256, 0, c->stream, x, rows, cols, ld_in, static_cast<__half*>(y),
                                                                       ld_out, transpose);
  return check_launch(c, "cast_rows");
}

// fp16 bit patterns -> fp32 bit patterns with integer operations only, so every input maps exactly as
// the reference's host conversion does (wgsl-unet.js:23-47): subnormals renormalised, Inf kept, NaN
// payloads shifted into the fp32 mantissa unchanged.  Two halves per thread (one 32-bit load).
__global__ void f16_bits_to_f32_kernel(const uint16_t* __restrict__ h, uint32_t* __restrict__ f, size_t n) {
  pdl_begin();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t x = h[i];
    const uint32_t sign = (x & 0x8000u) << 16;
    int e = (x >> 10) & 0x1f;
    uint32_t m = x & 0x3ffu, bits;
    if (e == 0) {
      if (m == 0) {
        bits = sign;
      } else {
        const int lz = __clz(m) - 21;  // shifts that bring the leading one to bit 10
        m = (m << lz) & 0x3ffu;
        e = 1 - lz;
        bits = sign | ((uint32_t)(e + 112) << 23) | (m << 13);
      }
    } else if (e == 31) {
      bits = sign | 0x7f800000u | (m << 13);
    } else {
      bits = sign | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
    f[i] = bits;
  }
}

}  // namespace di

using namespace di;

extern "C" {

int di_f16_bytes_to_f32(di_ctx_t h, const void* src, float* dst, size_t n) {
  Ctx* c = ctx_of(h);
  if (!c || (n && (!src || !dst))) return DI_EINVAL;
  if (!n) return DI_OK;
  launch_k(f16_bits_to_f32_kernel, grid_for(c, n), 256, 0, c->stream, static_cast<const uint16_t*>(src),
           reinterpret_cast<uint32_t*>(dst), n);
  return check_launch(c, "f16_bytes_to_f32");
}

int di_unary(di_ctx_t h, int op, const float* X, float* Y, uint32_t n) {
  Ctx* c = ctx_of(h);
  if (!c || op < 0 || op > DI_ERF) return DI_EINVAL;
  if (!n) return DI_OK;
  launch_k(unary_kernel, grid_for(c, n), 256, 0, c->stream, op, X, Y, n);
  return check_launch(c, "unary");
}
int di_binary(di_ctx_t h, int op, const float* A, uint32_t nA, const float* B, uint32_t nB, float* Y, uint32_t n) {
  Ctx* c = ctx_of(h);
  if (!c || op < 0 || op > DI_MIN || !nA || !nB) return DI_EINVAL;
  if (!n) return DI_OK;
  launch_k(binary_kernel, grid_for(c, n), 256, 0, c->stream, op, A, nA, B, nB, Y, n);
  return check_launch(c, "binary");
}
int di_binary_bcast(di_ctx_t h, int op, const float* A, const float* B, float* Y, const uint32_t cfg[20]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || op < 0 || op > DI_MIN || cfg[0] < 1 || cfg[0] > 4) return DI_EINVAL;
  Cfg20 k;
  memcpy(k.v, cfg, sizeof k.v);
  if (!k.v[16]) return DI_OK;
  launch_k(binary_bcast_kernel, grid_for(c, k.v[16]), 256, 0, c->stream, op, A, B, Y, k);
  return check_launch(c, "binary_bcast");
}
int di_affine_bcast(di_ctx_t h, const float* A, const float* G, const float* Bt, float* Y, const uint32_t cfg[20]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || cfg[0] < 1 || cfg[0] > 4) return DI_EINVAL;
  Cfg20 k;
  memcpy(k.v, cfg, sizeof k.v);
  if (!k.v[16]) return DI_OK;
  launch_k(affine_bcast_kernel, grid_for(c, k.v[16]), 256, 0, c->stream, A, G, Bt, Y, k);
  return check_launch(c, "affine_bcast");
}
int di_softmax(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[2]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !cfg[0]) return DI_EINVAL;
  if (!cfg[1]) return DI_OK;
  launch_k(softmax_rows, (cfg[1] + 7) / 8, 256, 0, c->stream, X, Y, cfg[0], cfg[1]);
  return check_launch(c, "softmax");
}
int di_reduce_mean(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[2]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !cfg[0]) return DI_EINVAL;
  if (!cfg[1]) return DI_OK;
  launch_k(reduce_mean_rows, (cfg[1] + 7) / 8, 256, 0, c->stream, X, Y, cfg[0], cfg[1]);
  return check_launch(c, "reduce_mean");
}
int di_resize_nearest(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[8]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !cfg[3] || !cfg[4]) return DI_EINVAL;
  if (!cfg[5]) return DI_OK;
  launch_k(resize_nearest_kernel, grid_for(c, cfg[5]), 256, 0, c->stream, X, Y, cfg[1], cfg[2], cfg[3], cfg[4], cfg[5]);
  return check_launch(c, "resize_nearest");
}
int di_transpose(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[20]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || cfg[0] < 1 || cfg[0] > 4) return DI_EINVAL;
  Cfg20 k;
  memcpy(k.v, cfg, sizeof k.v);
  if (!k.v[16]) return DI_OK;
  launch_k(transpose_kernel, grid_for(c, k.v[16]), 256, 0, c->stream, X, Y, k);
  return check_launch(c, "transpose");
}
int di_pow_scalar(di_ctx_t h, const float* X, float* Y, float e, uint32_t n) {
  Ctx* c = ctx_of(h);
  if (!c) return DI_EINVAL;
  if (!n) return DI_OK;
  launch_k(pow_scalar_kernel, grid_for(c, n), 256, 0, c->stream, X, Y, e, n);
  return check_launch(c, "pow_scalar");
}
int di_slice(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[20]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || cfg[0] < 1 || cfg[0] > 4) return DI_EINVAL;
  Cfg20 k;
  memcpy(k.v, cfg, sizeof k.v);
  if (!k.v[16]) return DI_OK;
  launch_k(slice_kernel, grid_for(c, k.v[16]), 256, 0, c->stream, X, Y, k);
  return check_launch(c, "slice");
}
int di_concat_copy(di_ctx_t h, const float* X, float* Y, const uint32_t cfg[4]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !cfg[0]) return DI_EINVAL;
  if (!cfg[3]) return DI_OK;
  launch_k(concat_copy_kernel, grid_for(c, cfg[3]), 256, 0, c->stream, X, Y, cfg[0], cfg[1], cfg[2], cfg[3]);
  return check_launch(c, "concat_copy");
}
int di_tembed(di_ctx_t h, const float* t, int B, const float* W1, const float* b1, const float* W2, const float* b2,
              int Din, int Dh, float* y) {
  Ctx* c = ctx_of(h);
  if (!c || B <= 0 || Din <= 0 || Dh <= 0) return DI_EINVAL;
  float* hidden = static_cast<float*>(workspace(c, sizeof(float) * (size_t)B * Dh, 1));
  if (!hidden) return set_error(c, DI_ENOMEM, "tembed workspace");
  return tembed(c, t, B, W1, b1, W2, b2, Din, Dh, hidden, y);
}

}  // extern "C"
