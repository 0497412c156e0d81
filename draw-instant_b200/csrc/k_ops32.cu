// k_ops32.cu — the reference's fp32 MatMul / Gemm / Conv op entry points (wgsl-ops.js:477-711, :821-910)
// on the tcgen05 GEMM.  Operands are packed once per call into library-owned scratch as fp16 with K
// padded to a multiple of 64 (fp16 carries the same 10-bit mantissa as tf32; accumulation is fp32),
// the output is written in fp32 in the reference's layout.  Conv uses an explicit im2col here (the
// generic, any-shape NCHW op); the fast NHWC path (di_conv3x3_nhwc) is implicit-GEMM via TMA.
#include <algorithm>

#include "di_common.cuh"

namespace di {

int gemm_linear(Ctx* c, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
                const float* bias, const void* R, int res_f32, void* Y, int out_f32, int geglu, const float* rowvec,
                int rowvec_div, void* splitk_ws = nullptr);
int cast_rows_f16(Ctx* c, const float* x, int rows, int cols, int ld_in, void* y, int ld_out, int transpose);

namespace {

inline int pad64(int k) { return (k + 63) / 64 * 64; }

// im2col for one image: col[p][kd] (fp16, row = output pixel, K = ci*K*K + ky*K + kx padded to ldk).
__global__ void im2col_kernel(const float* __restrict__ x, int Ci, int H, int W, int K, int S, int PAD, int Ho,
                              int Wo, int ldk, __half* __restrict__ col) {
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
    col[i] = __float2half_rn(v);
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
  __half* a = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)M * batch * Kp, 2));
  __half* b = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)N * Kp * (bb ? batch : 1), 3));
  if (!a || !b) return set_error(c, DI_ENOMEM, "matmul workspace");
  int r = cast_rows_f16(c, A, M * batch, K, K, a, Kp, 0);
  if (r) return r;
  const int nb = bb ? (int)batch : 1;
  for (int z = 0; z < nb; ++z) {
    r = cast_rows_f16(c, B + (size_t)z * K * N, N, K, N, b + (size_t)z * N * Kp, Kp, 1);  // B^T, K-major
    if (r) return r;
  }
  if (!bb) return gemm_linear(c, DI_F16, a, Kp, nullptr, rowsA, Kp, b, N, nullptr, nullptr, 0, Y, 1, 0, nullptr, 1);
  for (int z = 0; z < (int)batch; ++z) {
    r = gemm_linear(c, DI_F16, a + (size_t)z * M * Kp, Kp, nullptr, M, Kp, b + (size_t)z * N * Kp, N, nullptr,
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
  __half* a = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)M * Kp, 2));
  __half* b = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)N * Kp, 3));
  if (!a || !b) return set_error(c, DI_ENOMEM, "gemm workspace");
  int r = cast_rows_f16(c, A, M, K, K, a, Kp, 0);
  if (r) return r;
  r = transB ? cast_rows_f16(c, B, N, K, K, b, Kp, 0) : cast_rows_f16(c, B, N, K, N, b, Kp, 1);
  if (r) return r;
  return gemm_linear(c, DI_F16, a, Kp, nullptr, M, Kp, b, N, C, nullptr, 0, Y, 1, 0, nullptr, 1);
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
  __half* col = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)P * Kp, 2));
  __half* w = static_cast<__half*>(workspace(c, sizeof(__half) * (size_t)Co * Kp, 3));
  float* t = static_cast<float*>(workspace(c, sizeof(float) * (size_t)P * Co, 1));
  if (!col || !w || !t) return set_error(c, DI_ENOMEM, "conv workspace");
  int r = cast_rows_f16(c, W, Co, KD, KD, w, Kp, 0);  // [Co][Ci*K*K] is already K-major
  if (r) return r;
  const int blocks = 8 * c->num_sms;
  for (uint32_t n = 0; n < n_batch; ++n) {
    launch_k(im2col_kernel, blocks, 256, 0, c->stream, X + (size_t)n * Ci * H * Wd, Ci, H, Wd, K, S, PAD, Ho, Wo, Kp, col);
    r = check_launch(c, "im2col");
    if (r) return r;
    r = gemm_linear(c, DI_F16, col, Kp, nullptr, P, Kp, w, Co, bias, nullptr, 0, t, 1, 0, nullptr, 1);
    if (r) return r;
    launch_k(pm_to_cm_kernel, blocks, 256, 0, c->stream, t, P, Co, Y + (size_t)n * Co * P);
    r = check_launch(c, "conv_out_layout");
    if (r) return r;
  }
  return DI_OK;
}

}  // extern "C"
