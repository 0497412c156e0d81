// k_ops32.cu — the reference's fp32 MatMul / Gemm / Conv op entry points (wgsl-ops.js:477-711, :821-910)
// on the tcgen05 GEMM at fp32-level accuracy.  Every fp32 operand x is split into two bf16 terms,
// x = hi + lo with hi = bf16(x), lo = bf16(x - hi) (bf16 keeps the fp32 exponent range), and a row of
// K values is packed as three K-segments (each padded to a multiple of 64) so that ONE bf16 GEMM of
// depth 3K sums  a_hi.b_hi + a_hi.b_lo + a_lo.b_hi  in fp32: A rows are [hi | hi | lo], B rows are
// [hi | lo | hi].  The dropped a_lo.b_lo term and the rounding of lo leave about 2^-16 relative error
// per product, well inside the reference's 1e-3 gates (the plain bf16/fp16 product would not be).
// The output is written in fp32 in the reference's layout.  Conv uses an explicit im2col here (the
// generic, any-shape NCHW op); the fast NHWC path (di_conv3x3_nhwc) is implicit-GEMM via TMA.
#include <algorithm>

#include "di_common.cuh"

namespace di {

int gemm_linear(Ctx* c, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
                const float* bias, const void* R, int res_f32, void* Y, int out_f32, int geglu, const float* rowvec,
                int rowvec_div, void* splitk_ws = nullptr, const GnFuse* gnf = nullptr, int gnf_hw = 0, int act = 0);

namespace {

inline int pad64(int k) { return (k + 63) / 64 * 64; }

struct Split2 {
  __nv_bfloat16 hi, lo;
};
__device__ __forceinline__ Split2 split_bf16(float v) {
  Split2 r;
  r.hi = __float2bfloat16_rn(v);
  r.lo = __float2bfloat16_rn(v - __bfloat162float(r.hi));
  return r;
}
// Writes the 3-segment row (segment length seg): role 0 (A) = [hi | hi | lo], role 1 (B) = [hi | lo | hi].
__device__ __forceinline__ void put3(__nv_bfloat16* row, int seg, int k, float v, int role) {
  const Split2 s = split_bf16(v);
  row[k] = s.hi;
  row[seg + k] = role ? s.lo : s.hi;
  row[2 * seg + k] = role ? s.hi : s.lo;
}

// y[rows][3*seg] from x row-major [rows][cols] (transpose=0, row stride ld_in) or column-major
// x[cols][rows] (transpose=1, x[k][r] with row stride ld_in); columns >= cols are zero.
__global__ void split3_rows_kernel(const float* __restrict__ x, int rows, int cols, int ld_in, int seg, int transpose,
                                   int role, __nv_bfloat16* __restrict__ y) {
  pdl_begin();
  const size_t total = (size_t)rows * seg;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = i / seg, k = i % seg;
    float v = 0.f;
    if (k < cols) v = transpose ? x[(size_t)k * ld_in + r] : x[(size_t)r * ld_in + k];
    put3(y + (size_t)r * 3 * seg, seg, k, v, role);
  }
}

int split3(Ctx* c, const float* x, int rows, int cols, int ld_in, int seg, int transpose, int role, void* y) {
  const size_t total = (size_t)rows * seg;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)8 * c->num_sms);
  launch_k(split3_rows_kernel, std::max(blocks, 1), 256, 0, c->stream, x, rows, cols, ld_in, seg, transpose, role,
           static_cast<__nv_bfloat16*>(y));
  return check_launch(c, "split3_rows");
}

// im2col for one image: col[p] = 3-segment split row (role A) of the patch, K order ci*K*K + ky*K + kx,
// each segment padded to ldk.
__global__ void im2col_kernel(const float* __restrict__ x, int Ci, int H, int W, int K, int S, int PAD, int Ho,
                              int Wo, int ldk, __nv_bfloat16* __restrict__ col) {
  pdl_begin();
  const int KD = Ci * K * K;
  const size_t total = (size_t)Ho * Wo * ldk;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int kd = i % ldk;
    const int p = i / ldk;
    float v = 0.f;
    if (kd < KD) {
      const int ci = kd / (K * K), kk = kd % (K * K), ky = kk / K, kx = kk % K;
      const int oy = p / Wo, ox = p % Wo;
      const int iy = oy * S + ky - PAD, ix = ox * S + kx - PAD;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = x[((size_t)ci * H + iy) * W + ix];
    }
    put3(col + (size_t)p * 3 * ldk, ldk, kd, v, 0);
  }
}

// y[co][p] = t[p][co] (pixel-major GEMM output -> NCHW)
__global__ void pm_to_cm_kernel(const float* __restrict__ t, int P, int Co, float* __restrict__ y) {
  pdl_begin();
  const size_t total = (size_t)P * Co;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = i % P, co = i / P;
    y[i] = t[(size_t)p * Co + co];
  }
}

}  // namespace

}  // namespace di

using namespace di;

extern "C" {

int di_matmul(di_ctx_t h, const float* A, const float* B, float* Y, const uint32_t cfg[4], uint32_t batch) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !batch) return DI_EINVAL;
  const int M = cfg[0], N = cfg[1], K = cfg[2], bb = cfg[3];
  if (M <= 0 || N <= 0 || K <= 0) return DI_EINVAL;
  const int Kp = pad64(K);
  const int rowsA = bb ? M : M * (int)batch;  // shared B: the whole batch is one tall GEMM
  const int K3 = 3 * Kp;
  __nv_bfloat16* a = static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)M * batch * K3, 2));
  __nv_bfloat16* b =
      static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)N * K3 * (bb ? batch : 1), 3));
  if (!a || !b) return set_error(c, DI_ENOMEM, "matmul workspace");
  int r = split3(c, A, M * batch, K, K, Kp, 0, 0, a);
  if (r) return r;
  const int nb = bb ? (int)batch : 1;
  for (int z = 0; z < nb; ++z) {
    r = split3(c, B + (size_t)z * K * N, N, K, N, Kp, 1, 1, b + (size_t)z * N * K3);  // B^T, K-major
    if (r) return r;
  }
  if (!bb) return gemm_linear(c, DI_BF16, a, K3, nullptr, rowsA, K3, b, N, nullptr, nullptr, 0, Y, 1, 0, nullptr, 1);
  for (int z = 0; z < (int)batch; ++z) {
    r = gemm_linear(c, DI_BF16, a + (size_t)z * M * K3, K3, nullptr, M, K3, b + (size_t)z * N * K3, N, nullptr,
                    nullptr, 0, Y + (size_t)z * M * N, 1, 0, nullptr, 1);
    if (r) return r;
  }
  return DI_OK;
}

int di_gemm(di_ctx_t h, const float* A, const float* B, const float* C, float* Y, const uint32_t cfg[4]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg) return DI_EINVAL;
  const int M = cfg[0], N = cfg[1], K = cfg[2], transB = cfg[3];
  if (M <= 0 || N <= 0 || K <= 0) return DI_EINVAL;
  const int Kp = pad64(K);
  const int K3 = 3 * Kp;
  __nv_bfloat16* a = static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)M * K3, 2));
  __nv_bfloat16* b = static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)N * K3, 3));
  if (!a || !b) return set_error(c, DI_ENOMEM, "gemm workspace");
  int r = split3(c, A, M, K, K, Kp, 0, 0, a);
  if (r) return r;
  r = transB ? split3(c, B, N, K, K, Kp, 0, 1, b) : split3(c, B, N, K, N, Kp, 1, 1, b);
  if (r) return r;
  return gemm_linear(c, DI_BF16, a, K3, nullptr, M, K3, b, N, C, nullptr, 0, Y, 1, 0, nullptr, 1);
}

int di_conv(di_ctx_t h, const float* X, const float* W, const float* bias, float* Y, const uint32_t cfg[12],
            uint32_t n_batch) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg || !n_batch) return DI_EINVAL;
  const int Ci = cfg[0], Co = cfg[1], K = cfg[2], H = cfg[4], Wd = cfg[5], PAD = cfg[6], S = cfg[7], Ho = cfg[8],
            Wo = cfg[9];
  if (Ci <= 0 || Co <= 0 || K <= 0 || S <= 0 || Ho <= 0 || Wo <= 0 || (int)cfg[3] != K * K)
    return set_error(c, DI_EINVAL, "conv: bad cfg");
  const int KD = Ci * K * K, Kp = pad64(KD), P = Ho * Wo;
  const int K3 = 3 * Kp;
  __nv_bfloat16* col = static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)P * K3, 2));
  __nv_bfloat16* w = static_cast<__nv_bfloat16*>(workspace(c, sizeof(__nv_bfloat16) * (size_t)Co * K3, 3));
  float* t = static_cast<float*>(workspace(c, sizeof(float) * (size_t)P * Co, 1));
  if (!col || !w || !t) return set_error(c, DI_ENOMEM, "conv workspace");
  int r = split3(c, W, Co, KD, KD, Kp, 0, 1, w);  // [Co][Ci*K*K] is already K-major
  if (r) return r;
  const int blocks = 8 * c->num_sms;
  for (uint32_t n = 0; n < n_batch; ++n) {
    launch_k(im2col_kernel, blocks, 256, 0, c->stream, X + (size_t)n * Ci * H * Wd, Ci, H, Wd, K, S, PAD, Ho, Wo, Kp, col);
    r = check_launch(c, "im2col");
    if (r) return r;
    r = gemm_linear(c, DI_BF16, col, K3, nullptr, P, K3, w, Co, bias, nullptr, 0, t, 1, 0, nullptr, 1);
    if (r) return r;
    launch_k(pm_to_cm_kernel, blocks, 256, 0, c->stream, t, P, Co, Y + (size_t)n * Co * P);
    r = check_launch(c, "conv_out_layout");
    if (r) return r;
  }
  return DI_OK;
}

}  // extern "C"
