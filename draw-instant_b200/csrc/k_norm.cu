// k_norm.cu — GroupNorm / InstanceNorm / LayerNorm (+SiLU) for sm_100a.
//
// Bandwidth-bound: each kernel is measured by achieved HBM GB/s.  The reference runs one 256-thread
// workgroup per (n, group) with a shared-memory tree (wgsl-ops.js:390-458, fused-groupnorm.js:145-227),
// i.e. 32 workgroups for a whole feature map.  Here statistics are split over many CTAs (per-chunk
// partial sum / sum-of-squares written to a small scratch buffer, reduced in a fixed order so results
// are run-to-run deterministic), and the normalise pass is a separate fully parallel, vectorised
// elementwise kernel that re-derives mean / rstd per CTA from the partials.
//
// Numerics follow the reference: mean = sum/n, var = sumsq/n - mean^2 clamped at 0,
// y = (x - mean) * (1/sqrt(var + eps)) * gamma + beta, optional SiLU x/(1+exp(-x)).
#include <algorithm>
#include <cstdlib>

#include "di_common.cuh"

namespace di {

Ctx* ctx_of(di_ctx_t h);
void* workspace(Ctx* c, size_t bytes, int slot);

namespace {

template <typename T> struct Vec8 { T v[8]; };

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      T two[2];
      memcpy(two, &w[q], 4);
      f[2 * q] = to_f<T>(two[0]);
      f[2 * q + 1] = to_f<T>(two[1]);
    }
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      T two[2] = {from_f<T>(f[2 * q]), from_f<T>(f[2 * q + 1])};
      memcpy(&w[q], two, 4);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---------------------------------------------------------------------------------------------
// NHWC GroupNorm.  x = concat(x1[P, C1], x2[P, C2]) per pixel.
//
// Statistics pass: the pixels of image n are cut into `chunks` chunks of ~32 pixels; CTA (chunk, n) is a
// (V vectors of 8 channels) x (R pixel rows) block that sums its chunk per channel, then per group.
// CTAs form clusters of `cl` consecutive chunks: after a cluster barrier the rank-0 CTA adds the
// cluster's group sums from the other CTAs' shared memory (distributed shared memory, fixed rank
// order) and writes one (sum, sum-of-squares) per group: partial[n][cluster][g].  So the normalise
// pass folds only chunks / cl partials per group, and everything is run-to-run deterministic.
// ---------------------------------------------------------------------------------------------
constexpr int kGnRows = 8;  // pixels per thread per round in the statistics pass

__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

template <typename T>
__global__ void gn_nhwc_partial(const T* __restrict__ x1, int C1, const T* __restrict__ x2, int C2, int HW,
                                int chunk_pixels, int G, float2* __restrict__ partial) {
  pdl_begin();
  extern __shared__ float sh[];
  __shared__ float s_grp[2 * 128];  // this CTA's (sum, sumsq) per group
  const int C = C1 + C2, V = blockDim.x, R = blockDim.y;
  const int n = blockIdx.y, chunk = blockIdx.x;
  const int v = threadIdx.x, r = threadIdx.y, tid = r * V + v, nthr = V * R;
  float* ssum = sh;            // [R][C]
  float* ssq = sh + R * C;     // [R][C]
  {
    float s[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { s[j] = 0.f; q[j] = 0.f; }
    const int c = v * 8;
    const int p0 = chunk * chunk_pixels, p1 = min(HW, p0 + chunk_pixels);
    const T* base = c < C1 ? x1 + (size_t)n * HW * C1 + c : x2 + (size_t)n * HW * C2 + (c - C1);
    const size_t ld = c < C1 ? C1 : C2;
    // rounds of kGnRows pixels per thread, every load of a round issued before any use
    for (int pr = p0 + r; pr < p1; pr += kGnRows * R) {
      uint4 raw[kGnRows];  // 16-bit inputs: eight channels per 16-byte load
#pragma unroll
      for (int u = 0; u < kGnRows; ++u) {
        const int p = pr + u * R;
        if constexpr (sizeof(T) == 2)
          if (p < p1) raw[u] = __ldg(reinterpret_cast<const uint4*>(base + (size_t)p * ld));
      }
#pragma unroll
      for (int u = 0; u < kGnRows; ++u) {
        const int p = pr + u * R;
        if (p < p1) {
          float f[8];
          if constexpr (sizeof(T) == 4) load8<T>(base + (size_t)p * ld, f);  // fp32: loaded at use
          else load8<T>(reinterpret_cast<const T*>(&raw[u]), f);
#pragma unroll
          for (int j = 0; j < 8; ++j) { s[j] += f[j]; q[j] += f[j] * f[j]; }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { ssum[r * C + c + j] = s[j]; ssq[r * C + c + j] = q[j]; }
  }
  __syncthreads();
  for (int cc = tid; cc < C; cc += nthr) {  // fold the R rows per channel (fixed order)
    float s = 0.f, q = 0.f;
    for (int rr = 0; rr < R; ++rr) { s += ssum[rr * C + cc]; q += ssq[rr * C + cc]; }
    ssum[cc] = s;
    ssq[cc] = q;
  }
  __syncthreads();
  const int cpg = C / G;
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int cc = g * cpg; cc < (g + 1) * cpg; ++cc) { s += ssum[cc]; q += ssq[cc]; }
    s_grp[2 * g] = s;
    s_grp[2 * g + 1] = q;
  }
  cluster_sync();  // every CTA of the cluster has its group sums in shared memory
  const uint32_t rank = cluster_ctarank();
  uint32_t csize;
  asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  if (rank == 0) {
    const uint32_t base_addr = smem_u32(s_grp);
    for (int g = tid; g < G; g += nthr) {
      float s = 0.f, q = 0.f;
      for (uint32_t k = 0; k < csize; ++k) {
        const uint32_t a = mapa_shared(base_addr, k) + 8u * g;
        s += ld_dsmem_f32(a);
        q += ld_dsmem_f32(a + 4);
      }
      const int cluster = chunk / (int)csize, ncl = gridDim.x / (int)csize;
      partial[((size_t)n * ncl + cluster) * G + g] = make_float2(s, q);
    }
  }
  cluster_sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
}

// GroupNorm folded into a consumer's operand load: one cluster of kTabCluster CTAs per image computes
// the group statistics (each CTA a slice of the pixels, folded by the rank-0 CTA through distributed
// shared memory in fixed rank order) and writes the per-channel affine of the normalisation,
// table[n][c] = (scale, shift) with scale = gamma[c] * rstd[g], shift = beta[c] - mean[g] * scale,
// so the consumer applies y = x * scale + shift (then SiLU) to the raw activations as it loads them.
constexpr int kTabCluster = 16;

template <typename T>
__global__ void gn_table_kernel(const T* __restrict__ x1, int C1, const T* __restrict__ x2, int C2, int HW, int G,
                                float eps, const float* __restrict__ gamma, const float* __restrict__ beta,
                                float2* __restrict__ table) {
  pdl_begin();
  extern __shared__ float sh[];
  __shared__ float s_grp[2 * 128];
  __shared__ float s_mean[128], s_rstd[128];
  const int C = C1 + C2, V = blockDim.x, R = blockDim.y;
  const int n = blockIdx.y, rank = (int)cluster_ctarank();
  const int v = threadIdx.x, r = threadIdx.y, tid = r * V + v, nthr = V * R;
  const int per = (HW + kTabCluster - 1) / kTabCluster;
  float* ssum = sh;         // [R][C]
  float* ssq = sh + R * C;  // [R][C]
  {
    float s[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { s[j] = 0.f; q[j] = 0.f; }
    const int c = v * 8;
    const int p0 = rank * per, p1 = min(HW, p0 + per);
    const T* base = c < C1 ? x1 + (size_t)n * HW * C1 + c : x2 + (size_t)n * HW * C2 + (c - C1);
    const size_t ld = c < C1 ? C1 : C2;
    for (int pr = p0 + r; pr < p1; pr += kGnRows * R) {
      uint4 raw[kGnRows];
#pragma unroll
      for (int u = 0; u < kGnRows; ++u) {
        const int p = pr + u * R;
        if constexpr (sizeof(T) == 2)
          if (p < p1) raw[u] = __ldg(reinterpret_cast<const uint4*>(base + (size_t)p * ld));
      }
#pragma unroll
      for (int u = 0; u < kGnRows; ++u) {
        const int p = pr + u * R;
        if (p < p1) {
          float f[8];
          if constexpr (sizeof(T) == 4) load8<T>(base + (size_t)p * ld, f);
          else load8<T>(reinterpret_cast<const T*>(&raw[u]), f);
#pragma unroll
          for (int j = 0; j < 8; ++j) { s[j] += f[j]; q[j] += f[j] * f[j]; }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { ssum[r * C + c + j] = s[j]; ssq[r * C + c + j] = q[j]; }
  }
  __syncthreads();
  for (int cc = tid; cc < C; cc += nthr) {
    float s = 0.f, q = 0.f;
    for (int rr = 0; rr < R; ++rr) { s += ssum[rr * C + cc]; q += ssq[rr * C + cc]; }
    ssum[cc] = s;
    ssq[cc] = q;
  }
  __syncthreads();
  const int cpg = C / G;
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int cc = g * cpg; cc < (g + 1) * cpg; ++cc) { s += ssum[cc]; q += ssq[cc]; }
    s_grp[2 * g] = s;
    s_grp[2 * g + 1] = q;
  }
  cluster_sync();
  if (rank == 0) {
    const uint32_t base_addr = smem_u32(s_grp);
    for (int g = tid; g < G; g += nthr) {
      float s = 0.f, q = 0.f;
      for (int k = 0; k < kTabCluster; ++k) {
        const uint32_t a = mapa_shared(base_addr, (uint32_t)k) + 8u * g;
        s += ld_dsmem_f32(a);
        q += ld_dsmem_f32(a + 4);
      }
      const float cnt = (float)cpg * (float)HW;
      const float mean = s / cnt;
      const float var = fmaxf(q / cnt - mean * mean, 0.0f);
      s_mean[g] = mean;
      s_rstd[g] = 1.0f / sqrtf(var + eps);
    }
    __syncthreads();
    for (int cc = tid; cc < C; cc += nthr) {
      const int g = cc / cpg;
      const float sc = s_rstd[g] * gamma[cc];
      table[(size_t)n * C + cc] = make_float2(sc, beta[cc] - s_mean[g] * sc);
    }
  }
  cluster_sync();
}

// GroupNorm(32) from statistics a producer GEMM accumulated in exact fixed point (gn_fixed):
// stats[n][g] = {S, HI, LO} with sum = S / 2^24 and sum of squares = HI / 2^8 + LO / 2^48.  Grid
// (blocks, N): each block builds image n's per-channel (scale, shift) table in shared memory (double
// arithmetic, the variance clamped at 0 as in wgsl-ops.js:390-458), then normalises 8 channels per thread.
template <typename T>
__global__ void gn_apply_stats(const T* __restrict__ x, int C, int HW, const long long* __restrict__ stats,
                               float eps, const float* __restrict__ gamma, const float* __restrict__ beta, int silu,
                               T* __restrict__ y) {
  pdl_begin();
  extern __shared__ float2 gtab[];
  __shared__ float2 gmr[32];  // per group (mean, rstd)
  const int n = blockIdx.y, cpg = C / 32;
  if (threadIdx.x < 32) {
    const long long* st = stats + ((size_t)n * 32 + threadIdx.x) * 3;
    const double cnt = (double)cpg * (double)HW;
    const double sum = (double)st[0] * 0x1p-24;
    const double sq = (double)st[1] * 0x1p-8 + (double)st[2] * 0x1p-48;
    const double mean = sum / cnt;
    const double var = fmax(sq / cnt - mean * mean, 0.0);
    gmr[threadIdx.x] = make_float2((float)mean, (float)(1.0 / sqrt(var + (double)eps)));
  }
  __syncthreads();
  for (int cc = threadIdx.x; cc < C; cc += blockDim.x) {
    const float2 mr = gmr[cc / cpg];
    const float sc = mr.y * gamma[cc];
    gtab[cc] = make_float2(sc, beta[cc] - mr.x * sc);
  }
  __syncthreads();
  const int V = C / 8;
  const size_t per_img = (size_t)HW * V;
  const T* xi = x + (size_t)n * HW * C;
  T* yi = y + (size_t)n * HW * C;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < per_img; e += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % V) * 8;
    const size_t off = (e / V) * C + c;
    float f[8];
    load8<T>(xi + off, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 t = gtab[c + j];
      const float z = fmaf(f[j], t.x, t.y);
      f[j] = silu ? silu_f(z) : z;
    }
    store8<T>(yi + off, f);
  }
}

// Normalise with a precomputed (scale, shift) table (gn_table_nhwc): one 8-channel vector per thread,
// y = silu?(x * scale + shift); table rows are read through L1 (they are tiny and shared by all pixels).
template <typename Tin, typename Tout>
__global__ void gn_apply_table(const Tin* __restrict__ x1, int C1, const Tin* __restrict__ x2, int C2, int HW,
                               const float2* __restrict__ table, int silu, size_t total, Tout* __restrict__ y) {
  pdl_begin();
  const int C = C1 + C2, V = C / 8;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int v = (int)(e % V);
    const size_t pix = e / V;  // n * HW + p
    const int n = (int)(pix / HW), c = v * 8;
    float f[8];
    if (c < C1) load8<Tin>(x1 + pix * C1 + c, f);
    else load8<Tin>(x2 + pix * C2 + (c - C1), f);
    const float4* t = reinterpret_cast<const float4*>(table + (size_t)n * C + c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 q = __ldg(t + j);
      float a = fmaf(f[2 * j], q.x, q.y), b = fmaf(f[2 * j + 1], q.z, q.w);
      if (silu) {
        a = __fdividef(a, 1.0f + __expf(-a));
        b = __fdividef(b, 1.0f + __expf(-b));
      }
      f[2 * j] = a;
      f[2 * j + 1] = b;
    }
    store8<Tout>(y + pix * C + c, f);
  }
}

// Single-launch GroupNorm(+SiLU) of concat(x1, x2) for maps that fit in the shared memory of at most one
// CTA per SM.  Grid (cpi, N): CTA (k, n) owns pixels [k * per, min(HW, (k + 1) * per)) of image n.
//   1. one bulk copy per input brings the CTA's slice (contiguous in NHWC) into shared memory;
//   2. per-channel sums and sums of squares (fp32, one 8-channel vector per thread) fold to per-group
//      sums, written to partial[n][k][g];
//   3. a grid barrier (every CTA is resident: the grid is at most one CTA per SM), then every CTA folds
//      its image's cpi partials in a fixed order (deterministic, identical in every CTA) to mean / rstd;
//   4. the slice is normalised from shared memory and written once.
// Global traffic is the minimum, one read and one write of the map, in one launch instead of the
// statistics + normalise pair.  The barrier is a {arrivals, generation} word pair: the last CTA to arrive
// resets the arrivals and bumps the generation; the others wait for the bump, bounded by kWaitTimeoutNs
// (then DEVERR_GRID_BARRIER is recorded and the kernel still finishes).  The next kernel is released
// (pdl_trigger) at once: a dependent grid launches only after every CTA of this one has executed the
// trigger, i.e. once the whole grid is resident, so its CTAs can never hold an SM this grid still needs.
constexpr int kGridSub = 8;  // fixed partition of the partial fold (deterministic order)

template <typename T>
__global__ void __launch_bounds__(512) gn_nhwc_grid(const T* __restrict__ x1, int C1, const T* __restrict__ x2, int C2, int HW, int per,
                             int G, float eps, const float* __restrict__ gamma, const float* __restrict__ beta,
                             int silu, T* __restrict__ y, float2* __restrict__ partial, unsigned* bar, int* err) {
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ float s_fold[2 * kGridSub * 128];
  __shared__ float s_mean[128], s_rstd[128];
  const int C = C1 + C2, V = blockDim.x, R = blockDim.y;
  const int n = blockIdx.y, k = blockIdx.x, cpi = gridDim.x;
  const int v = threadIdx.x, r = threadIdx.y, tid = r * V + v, nthr = V * R;
  const int p0 = k * per, cnt = max(0, min(HW, p0 + per) - p0);
  uint8_t* s1 = gsm;                                   // [cnt][C1]
  uint8_t* s2 = gsm + (size_t)per * C1 * sizeof(T);    // [cnt][C2]
  float* ssum = reinterpret_cast<float*>(gsm + (size_t)per * C * sizeof(T));  // [R][C]
  float* ssq = ssum + R * C;                                                  // [R][C]
  if (tid == 0) {
    mbar_init(&mbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // x1 / x2 are written by the previous kernel
  if (tid == 0) {
    const uint32_t b1 = (uint32_t)((size_t)cnt * C1 * sizeof(T)), b2 = (uint32_t)((size_t)cnt * C2 * sizeof(T));
    mbar_arrive_expect_tx(&mbar, b1 + b2);
    if (b1) bulk_load(s1, x1 + ((size_t)n * HW + p0) * C1, b1, &mbar);
    if (b2) bulk_load(s2, x2 + ((size_t)n * HW + p0) * C2, b2, &mbar);
  }
  mbar_wait(&mbar, 0, err, DEVERR_WAIT_EPI);
  const int c = v * 8;
  const uint8_t* src = c < C1 ? s1 + (size_t)c * sizeof(T) : s2 + (size_t)(c - C1) * sizeof(T);
  const size_t row_bytes = (c < C1 ? C1 : C2) * sizeof(T);
  {
    float s[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { s[j] = 0.f; q[j] = 0.f; }
    for (int p = r; p < cnt; p += R) {
      float f[8];
      load8<T>(reinterpret_cast<const T*>(src + p * row_bytes), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) { s[j] += f[j]; q[j] += f[j] * f[j]; }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { ssum[r * C + c + j] = s[j]; ssq[r * C + c + j] = q[j]; }
  }
  __syncthreads();
  for (int cc = tid; cc < C; cc += nthr) {
    float s = 0.f, q = 0.f;
    for (int rr = 0; rr < R; ++rr) { s += ssum[rr * C + cc]; q += ssq[rr * C + cc]; }
    ssum[cc] = s;
    ssq[cc] = q;
  }
  __syncthreads();
  const int cpg = C / G;
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int cc = g * cpg; cc < (g + 1) * cpg; ++cc) { s += ssum[cc]; q += ssq[cc]; }
    partial[((size_t)n * cpi + k) * G + g] = make_float2(s, q);
  }
  __syncthreads();
  if (tid == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    const unsigned gen = ld_acquire_gpu(bar + 1);  // cannot move before every CTA of this launch arrives
    __threadfence();                               // this CTA's partials before its arrival
    const unsigned old = atomicAdd(bar, 1u);
    if (old == total - 1) {
      atomicExch(bar, 0u);  // arrivals reset for the next launch, before anyone is released
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_gpu(bar + 1) == gen) {
        if (globaltimer() - t0 > kWaitTimeoutNs) {
          atomicOr(err, DEVERR_GRID_BARRIER);
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  // fold the image's cpi partials: (group g, subset u) sums partials u, u + kGridSub, ... in order, then
  // the kGridSub subset sums are added in order (the same arithmetic in every CTA of the image)
  for (int idx = tid; idx < G * kGridSub; idx += nthr) {
    const int g = idx % G, u = idx / G;
    float s = 0.f, q = 0.f;
    const float2* pp = partial + (size_t)n * cpi * G + g;
    int kk = u;
    for (; kk + 7 * kGridSub < cpi; kk += 8 * kGridSub) {  // eight loads in flight, added in order
      float2 t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = __ldcg(pp + (size_t)(kk + i * kGridSub) * G);
#pragma unroll
      for (int i = 0; i < 8; ++i) { s += t[i].x; q += t[i].y; }
    }
    for (; kk < cpi; kk += kGridSub) {
      const float2 t = __ldcg(pp + (size_t)kk * G);
      s += t.x;
      q += t.y;
    }
    s_fold[2 * (u * G + g)] = s;
    s_fold[2 * (u * G + g) + 1] = q;
  }
  __syncthreads();
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int u = 0; u < kGridSub; ++u) { s += s_fold[2 * (u * G + g)]; q += s_fold[2 * (u * G + g) + 1]; }
    const float cntf = (float)cpg * (float)HW;
    const float mean = s / cntf;
    const float var = fmaxf(q / cntf - mean * mean, 0.0f);
    s_mean[g] = mean;
    s_rstd[g] = 1.0f / sqrtf(var + eps);
  }
  __syncthreads();
  float sc[8], sh[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int g = (c + j) / cpg;
    sc[j] = s_rstd[g] * __ldg(gamma + c + j);
    sh[j] = __ldg(beta + c + j) - s_mean[g] * sc[j];
  }
  T* yo = y + ((size_t)n * HW + p0) * C + c;
  for (int p = r; p < cnt; p += R) {
    float f[8];
    load8<T>(reinterpret_cast<const T*>(src + p * row_bytes), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = fmaf(f[j], sc[j], sh[j]);
      f[j] = silu ? __fdividef(a, 1.0f + __expf(-a)) : a;
    }
    store8<T>(yo + (size_t)p * C, f);
  }
}

// Single-launch GroupNorm(+SiLU) of concat(x1, x2) for maps whose per-image slice fits one cluster:
// grid (kGnCluster, N), clusters of kGnCluster CTAs, one cluster per image.  CTA rank k owns pixels
// [k * per, min(HW, (k + 1) * per)):
//   1. one bulk copy per input brings the slice (contiguous in NHWC) into shared memory;
//   2. per-channel sums and sums of squares (fp32, one 8-channel vector per thread) fold to per-group
//      sums in this CTA's shared memory;
//   3. after a cluster barrier every CTA reads all ranks' group sums through distributed shared memory,
//      in rank order (the same arithmetic in every CTA: deterministic), to mean / rstd; a second cluster
//      barrier lets the ranks' shared memory go;
//   4. the slice is normalised from shared memory and written once.
// One read and one write of the map in one launch, with no grid-wide barrier and no global scratch; only
// kGnCluster SMs per image are held, so the consumer's CTAs start on the others.
constexpr int kGnCluster = 16;

template <typename T>
__global__ void __launch_bounds__(1024) gn_nhwc_cluster(const T* __restrict__ x1, int C1, const T* __restrict__ x2,
                                                        int C2, int HW, int per, int G, float eps,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, int silu, T* __restrict__ y,
                                                        int* err) {
  extern __shared__ __align__(16) uint8_t csm[];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ float s_grp[2 * 128];
  __shared__ float s_mean[128], s_rstd[128];
  const int C = C1 + C2, V = blockDim.x, R = blockDim.y;
  const int n = blockIdx.y, k = (int)cluster_ctarank();
  const int v = threadIdx.x, r = threadIdx.y, tid = r * V + v, nthr = V * R;
  const int p0 = k * per, cnt = max(0, min(HW, p0 + per) - p0);
  uint8_t* s1 = csm;                                                         // [cnt][C1]
  uint8_t* s2 = csm + (size_t)per * C1 * sizeof(T);                          // [cnt][C2]
  float* ssum = reinterpret_cast<float*>(csm + (size_t)per * C * sizeof(T));  // [R][C]
  float* ssq = ssum + R * C;                                                  // [R][C]
  if (tid == 0) {
    mbar_init(&mbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // x1 / x2 are written by the previous kernel
  if (tid == 0) {
    const uint32_t b1 = (uint32_t)((size_t)cnt * C1 * sizeof(T)), b2 = (uint32_t)((size_t)cnt * C2 * sizeof(T));
    mbar_arrive_expect_tx(&mbar, b1 + b2);
    if (b1) bulk_load(s1, x1 + ((size_t)n * HW + p0) * C1, b1, &mbar);
    if (b2) bulk_load(s2, x2 + ((size_t)n * HW + p0) * C2, b2, &mbar);
  }
  const bool landed = mbar_wait(&mbar, 0, err, DEVERR_WAIT_EPI);
  const int c = v * 8;
  const uint8_t* src = c < C1 ? s1 + (size_t)c * sizeof(T) : s2 + (size_t)(c - C1) * sizeof(T);
  const size_t row_bytes = (c < C1 ? C1 : C2) * sizeof(T);
  {
    float s[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { s[j] = 0.f; q[j] = 0.f; }
    for (int p = r; landed && p < cnt; p += R) {
      float f[8];
      load8<T>(reinterpret_cast<const T*>(src + p * row_bytes), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) { s[j] += f[j]; q[j] += f[j] * f[j]; }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { ssum[r * C + c + j] = s[j]; ssq[r * C + c + j] = q[j]; }
  }
  __syncthreads();
  for (int cc = tid; cc < C; cc += nthr) {  // fold the R rows per channel (fixed order)
    float s = 0.f, q = 0.f;
    for (int rr = 0; rr < R; ++rr) { s += ssum[rr * C + cc]; q += ssq[rr * C + cc]; }
    ssum[cc] = s;
    ssq[cc] = q;
  }
  __syncthreads();
  const int cpg = C / G;
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int cc = g * cpg; cc < (g + 1) * cpg; ++cc) { s += ssum[cc]; q += ssq[cc]; }
    s_grp[2 * g] = s;
    s_grp[2 * g + 1] = q;
  }
  cluster_sync();  // every rank's group sums are in its shared memory
  const uint32_t base_addr = smem_u32(s_grp);
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int kk = 0; kk < kGnCluster; ++kk) {
      const uint32_t a = mapa_shared(base_addr, (uint32_t)kk) + 8u * g;
      s += ld_dsmem_f32(a);
      q += ld_dsmem_f32(a + 4);
    }
    const float cntf = (float)cpg * (float)HW;
    const float mean = s / cntf;
    const float var = fmaxf(q / cntf - mean * mean, 0.0f);
    s_mean[g] = mean;
    s_rstd[g] = 1.0f / sqrtf(var + eps);
  }
  cluster_sync();  // all ranks have read every rank's sums (and s_mean / s_rstd are visible in the CTA)
  float sc[8], sh[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int g = (c + j) / cpg;
    sc[j] = s_rstd[g] * __ldg(gamma + c + j);
    sh[j] = __ldg(beta + c + j) - s_mean[g] * sc[j];
  }
  T* yo = y + ((size_t)n * HW + p0) * C + c;
  for (int p = r; landed && p < cnt; p += R) {
    float f[8];
    load8<T>(reinterpret_cast<const T*>(src + p * row_bytes), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = fmaf(f[j], sc[j], sh[j]);
      f[j] = silu ? __fdividef(a, 1.0f + __expf(-a)) : a;
    }
    store8<T>(yo + (size_t)p * C, f);
  }
}

// Normalise pass.  Block = V threads (one 8-channel vector each) x R pixel rows, so every thread keeps
// the same 8 channels for the whole grid and applies them as one FMA per element with per-thread
// scale / shift (gamma * rstd, beta - mean * gamma * rstd); two pixels per thread per round.
template <typename Tin, typename Tout>
__global__ void gn_nhwc_apply(const Tin* __restrict__ x1, int C1, const Tin* __restrict__ x2, int C2, int HW, int G,
                              const float2* __restrict__ partial, int ncl, const float* __restrict__ gamma,
                              const float* __restrict__ beta, float eps, int silu, Tout* __restrict__ y) {
  pdl_begin();
  extern __shared__ float2 s_part[];  // [ncl][G]
  __shared__ float s_mean[128], s_rstd[128];
  const int C = C1 + C2, V = C / 8, cpg = C / G;
  const int n = blockIdx.y;
  const int nthr = blockDim.x * blockDim.y, tid = threadIdx.y * blockDim.x + threadIdx.x;
  const float2* src = partial + (size_t)n * ncl * G;
  for (int k = tid; k < ncl * G; k += nthr) s_part[k] = src[k];
  __syncthreads();
  for (int g = tid; g < G; g += nthr) {
    float s = 0.f, q = 0.f;
    for (int k = 0; k < ncl; ++k) {
      const float2 pq = s_part[k * G + g];
      s += pq.x;
      q += pq.y;
    }
    const float cnt = (float)cpg * (float)HW;
    const float mean = s / cnt;
    const float var = fmaxf(q / cnt - mean * mean, 0.0f);
    s_mean[g] = mean;
    s_rstd[g] = 1.0f / sqrtf(var + eps);
  }
  __syncthreads();
  const int v = threadIdx.x, c = v * 8;
  if (v >= V) return;
  float sc[8], sf[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int g = (c + j) / cpg;
    sc[j] = s_rstd[g] * __ldg(gamma + c + j);
    sf[j] = __ldg(beta + c + j) - s_mean[g] * sc[j];
  }
  const Tin* base = c < C1 ? x1 + (size_t)n * HW * C1 + c : x2 + (size_t)n * HW * C2 + (c - C1);
  const size_t ld = c < C1 ? C1 : C2;
  Tout* out = y + (size_t)n * HW * C + c;
  const int R = blockDim.y, stride = gridDim.x * R;
  for (int p0 = blockIdx.x * R + threadIdx.y; p0 < HW; p0 += 2 * stride) {
    float f[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int p = p0 + u * stride;
      if (p < HW) load8<Tin>(base + (size_t)p * ld, f[u]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int p = p0 + u * stride;
      if (p < HW) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float o = fmaf(f[u][j], sc[j], sf[j]);
          f[u][j] = silu ? __fdividef(o, 1.0f + __expf(-o)) : o;
        }
        store8<Tout>(out + (size_t)p * C, f[u]);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// NCHW fp32 GroupNorm (op family).  Group (n, g) is the contiguous span [(n*C + g*cpg)*HW, +cpg*HW).
// ---------------------------------------------------------------------------------------------
__global__ void gn_nchw_partial(const float* __restrict__ x, int G, size_t gsize, int nchunks,
                                float2* __restrict__ partial) {
  pdl_begin();
  const int chunk = blockIdx.x, g = blockIdx.y, n = blockIdx.z;
  const size_t base = ((size_t)n * G + g) * gsize;
  const size_t per = (gsize + nchunks - 1) / nchunks;
  const size_t b0 = chunk * per, b1 = min(gsize, b0 + per);
  float s = 0.f, q = 0.f;
  for (size_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
    const float v = x[base + i];
    s += v; q += v * v;
  }
  __shared__ float ws[32], wq[32];
  for (int o = 16; o; o >>= 1) { s += __shfl_xor_sync(~0u, s, o); q += __shfl_xor_sync(~0u, q, o); }
  if ((threadIdx.x & 31) == 0) { ws[threadIdx.x / 32] = s; wq[threadIdx.x / 32] = q; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float S = 0.f, Q = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) { S += ws[w]; Q += wq[w]; }
    partial[((size_t)n * G + g) * nchunks + chunk] = make_float2(S, Q);
  }
}

__global__ void gn_nchw_apply(const float* __restrict__ x, int C, int G, int HW, int nchunks,
                              const float2* __restrict__ partial, const float* __restrict__ gamma,
                              const float* __restrict__ beta, float eps, int silu, int clamp, size_t total,
                              float* __restrict__ y) {
  pdl_begin();
  const int cpg = C / G;
  const float cnt = (float)cpg * (float)HW;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t nc = i / HW;
    const int c = nc % C;
    const size_t n = nc / C;
    const int g = c / cpg;
    float s = 0.f, q = 0.f;
    const float2* pp = partial + ((size_t)n * G + g) * nchunks;
    for (int k = 0; k < nchunks; ++k) { s += pp[k].x; q += pp[k].y; }
    const float mean = s / cnt;
    float var = q / cnt - mean * mean;
    if (clamp) var = fmaxf(var, 0.0f);
    const float o = (x[i] - mean) * (1.0f / sqrtf(var + eps)) * gamma[c] + beta[c];
    y[i] = silu ? silu_f(o) : o;
  }
}

// ---------------------------------------------------------------------------------------------
// LayerNorm: one warp per row.  Token-major [rows, D]; T in/out, gamma/beta fp32.
// ---------------------------------------------------------------------------------------------
template <typename Tin, typename Tout>
__global__ void layer_norm_rows(const Tin* __restrict__ x, const float* __restrict__ g, const float* __restrict__ b,
                                Tout* __restrict__ y, int rows, int D, float eps) {
  pdl_begin();
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const Tin* xr = x + (size_t)row * D;
  float s = 0.f, q = 0.f;
  for (int i = lane; i < D; i += 32) { const float v = to_f<Tin>(xr[i]); s += v; q += v * v; }
  for (int o = 16; o; o >>= 1) { s += __shfl_xor_sync(~0u, s, o); q += __shfl_xor_sync(~0u, q, o); }
  const float mean = s / (float)D;
  const float var = fmaxf(q / (float)D - mean * mean, 0.0f);
  const float inv = 1.0f / sqrtf(var + eps);
  for (int i = lane; i < D; i += 32) y[(size_t)row * D + i] = from_f<Tout>((to_f<Tin>(xr[i]) - mean) * inv * g[i] + b[i]);
}

// LayerNorm with the row held in registers: one warp per row, lane l owns the 8-element chunks
// l, l + 32, ... (NV chunks at most, D <= 256 NV), read once with 16/32-byte loads; the same
// E[x^2] - mean^2 statistics as layer_norm_rows.  Needs D % 8 == 0 and 16-byte aligned rows.
template <typename Tin, typename Tout, int NV>
__global__ void layer_norm_rows_vec(const Tin* __restrict__ x, const float* __restrict__ g,
                                    const float* __restrict__ b, Tout* __restrict__ y, int rows, int D, float eps) {
  pdl_begin();
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nch = D / 8;
  const Tin* xr = x + (size_t)row * D;
  float v[NV][8];
  float s = 0.f, q = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int ch = lane + 32 * k;
    if (ch < nch) {
      load8<Tin>(xr + ch * 8, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) { s += v[k][i]; q += v[k][i] * v[k][i]; }
    }
  }
  for (int o = 16; o; o >>= 1) { s += __shfl_xor_sync(~0u, s, o); q += __shfl_xor_sync(~0u, q, o); }
  const float mean = s / (float)D;
  const float var = fmaxf(q / (float)D - mean * mean, 0.0f);
  const float inv = 1.0f / sqrtf(var + eps);
  Tout* yr = y + (size_t)row * D;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int ch = lane + 32 * k;
    if (ch < nch) {
      float gg[8], bb[8], o8[8];
      load8<float>(g + ch * 8, gg);
      load8<float>(b + ch * 8, bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = (v[k][i] - mean) * inv * gg[i] + bb[i];
      store8<Tout>(yr + ch * 8, o8);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// Host entry points (also used by the fused blocks / U-Net plan).
// ---------------------------------------------------------------------------------------------
// Statistics-pass geometry: chunks of ~32 pixels (at most 128 per image), in clusters of up to 8 CTAs
// (cl divides chunks); the partial buffer holds chunks / cl = max(1, min(16, HW / 256)) entries per
// (image, group).
static void gn_geometry(int HW, int* chunks, int* cl) {
  int ch = std::max(1, std::min(128, HW / 32));
  const int k = std::min(8, ch);
  *chunks = (ch / k) * k;
  *cl = k;
}

template <typename Tin, typename Tout>
static int gn_nhwc_impl(Ctx* c, const Tin* x1, int C1, const Tin* x2, int C2, int N, int HW, int G, float eps,
                        const float* gamma, const float* beta, int silu, Tout* y, float2* partial) {
  const int C = C1 + C2;
  if (C % 8 || C1 % 8 || G <= 0 || G > 128 || C % G) return set_error(c, DI_EINVAL, "group_norm_nhwc: bad channels");
  const int V = C / 8;
  if (V > 1024) return set_error(c, DI_EUNSUPPORTED, "group_norm_nhwc: too many channels");
  int chunks, cl;
  gn_geometry(HW, &chunks, &cl);
  const int ncl = chunks / cl;
  const int chunk_pixels = (HW + chunks - 1) / chunks;
  if (!partial) {
    partial = static_cast<float2*>(workspace(c, sizeof(float2) * (size_t)N * ncl * G, 0));
    if (!partial) return set_error(c, DI_ENOMEM, "group_norm_nhwc: workspace");
  }
  const int R = std::max(1, 256 / V);
  const size_t shm = sizeof(float) * 2 * R * C;
  launch_k_cluster(gn_nhwc_partial<Tin>, dim3(chunks, N), dim3(V, R), shm, c->stream, cl, x1, C1, x2, C2, HW,
                   chunk_pixels, G, partial);
  // normalise: V x Ra threads per block, two pixels per thread
  const int Ra = std::max(1, 256 / V);
  const int ablocks = std::max(1, (HW + 2 * Ra - 1) / (2 * Ra));
  launch_k(gn_nhwc_apply<Tin, Tout>, dim3(ablocks, N), dim3(V, Ra), sizeof(float2) * ncl * G, c->stream, x1, C1, x2,
           C2, HW, G, partial, ncl, gamma, beta, eps, silu, y);
  return check_launch(c, "group_norm_nhwc");
}

int group_norm_nhwc(Ctx* c, int in_dtype, int out_dtype, const void* x1, int C1, const void* x2, int C2, int N,
                    int HW, int G, float eps, const float* gamma, const float* beta, int silu, void* y,
                    void* partial_ws) {
  float2* pw = static_cast<float2*>(partial_ws);
#define GN_CASE(TI, TO)                                                                                        \
  return gn_nhwc_impl<TI, TO>(c, static_cast<const TI*>(x1), C1, static_cast<const TI*>(x2), C2, N, HW, G, eps, \
                              gamma, beta, silu, static_cast<TO*>(y), pw)
  if (in_dtype == DI_F16 && out_dtype == DI_F16) GN_CASE(__half, __half);
  if (in_dtype == DI_BF16 && out_dtype == DI_BF16) GN_CASE(__nv_bfloat16, __nv_bfloat16);
  if (in_dtype == DI_F32 && out_dtype == DI_F16) GN_CASE(float, __half);
  if (in_dtype == DI_F32 && out_dtype == DI_BF16) GN_CASE(float, __nv_bfloat16);
  if (in_dtype == DI_F32 && out_dtype == DI_F32) GN_CASE(float, float);
#undef GN_CASE
  return set_error(c, DI_EINVAL, "group_norm_nhwc: dtype combination");
}

// Loads the device code of the kernels group_norm_nhwc runs for fp16 and bf16 (under CUDA's lazy module
// loading a kernel is otherwise loaded, and its memory allocated, at its first launch).
int gn_nhwc_preload(Ctx* c) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, gn_nhwc_partial<__half>) != cudaSuccess ||
      cudaFuncGetAttributes(&a, gn_nhwc_partial<__nv_bfloat16>) != cudaSuccess ||
      cudaFuncGetAttributes(&a, gn_nhwc_apply<__half, __half>) != cudaSuccess ||
      cudaFuncGetAttributes(&a, gn_nhwc_apply<__nv_bfloat16, __nv_bfloat16>) != cudaSuccess)
    return set_error(c, DI_ECUDA, "group_norm_nhwc: loading the kernels failed");
  return DI_OK;
}

// Statistics of concat(x1, x2) -> table[N][C] of (scale, shift) for an operand-fused GroupNorm.
int gn_table_nhwc(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G, float eps,
                  const float* gamma, const float* beta, float2* table) {
  const int C = C1 + C2;
  if (C % 8 || C1 % 8 || G <= 0 || G > 128 || C % G || N <= 0 || HW <= 0)
    return set_error(c, DI_EINVAL, "gn_table_nhwc: bad shape");
  const int V = C / 8;
  if (V > 1024) return set_error(c, DI_EUNSUPPORTED, "gn_table_nhwc: too many channels");
  const int R = std::max(1, 256 / V);
  const size_t shm = sizeof(float) * 2 * R * C;
  static unsigned attr_done = 0;  // per-device bit: clusters of 16 need the non-portable size opt-in
  if (!(attr_done & (1u << (c->device & 31)))) {
    if (cudaFuncSetAttribute(gn_table_kernel<__half>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess ||
        cudaFuncSetAttribute(gn_table_kernel<__nv_bfloat16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess)
      return set_error(c, DI_ECUDA, "gn_table_nhwc: cluster attribute");
    attr_done |= 1u << (c->device & 31);
  }
  if (dtype == DI_BF16)
    launch_k_cluster(gn_table_kernel<__nv_bfloat16>, dim3(kTabCluster, N), dim3(V, R), shm, c->stream, kTabCluster,
                     static_cast<const __nv_bfloat16*>(x1), C1, static_cast<const __nv_bfloat16*>(x2), C2, HW, G, eps,
                     gamma, beta, table);
  else
    launch_k_cluster(gn_table_kernel<__half>, dim3(kTabCluster, N), dim3(V, R), shm, c->stream, kTabCluster,
                     static_cast<const __half*>(x1), C1, static_cast<const __half*>(x2), C2, HW, G, eps, gamma, beta,
                     table);
  return check_launch(c, "gn_table_nhwc");
}

// GroupNorm(+SiLU) of concat(x1, x2) through the statistics table: two launches (cluster statistics,
// then a fully parallel elementwise normalise).  `table` holds N * C (scale, shift) pairs.
int gn_nhwc_via_table(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                      float eps, const float* gamma, const float* beta, int silu, void* y, float2* table) {
  int r = gn_table_nhwc(c, dtype, x1, C1, x2, C2, N, HW, G, eps, gamma, beta, table);
  if (r) return r;
  const int C = C1 + C2;
  const size_t total = (size_t)N * HW * (C / 8);
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((total + 255) / 256, (size_t)16 * c->num_sms));
  if (dtype == DI_BF16)
    launch_k(gn_apply_table<__nv_bfloat16, __nv_bfloat16>, blocks, 256, 0, c->stream,
             static_cast<const __nv_bfloat16*>(x1), C1, static_cast<const __nv_bfloat16*>(x2), C2, HW, table, silu,
             total, static_cast<__nv_bfloat16*>(y));
  else
    launch_k(gn_apply_table<__half, __half>, blocks, 256, 0, c->stream, static_cast<const __half*>(x1), C1,
             static_cast<const __half*>(x2), C2, HW, table, silu, total, static_cast<__half*>(y));
  return check_launch(c, "gn_apply_table");
}

// ---- single-launch GroupNorm (gn_nhwc_grid) ----
// Largest per-CTA slice of the map kept in shared memory; larger maps use the two-launch paths.
constexpr size_t kGridSliceMax = 160u << 10;

// Geometry of gn_nhwc_grid: cpi CTAs per image (cpi * N <= SMs, so the whole grid is resident at once),
// `per` pixels each (at least 4 where the map allows), a V x R thread block.  False when the map does not
// fit (slice beyond kGridSliceMax, too many images for one CTA each, channel count unsupported).
bool gn_grid_geometry(int num_sms, int N, int HW, int C, int G, int* cpi, int* per, int* R, size_t* smem) {
  if (N <= 0 || HW <= 0 || C % 8 || G <= 0 || G > 128 || C % G) return false;
  const int V = C / 8;
  if (V > 512) return false;
  int k = std::min(num_sms / N, (HW + 3) / 4);
  if (k < 1) return false;
  const int pp = (HW + k - 1) / k;
  k = (HW + pp - 1) / pp;  // no empty CTAs
  const size_t slice = (size_t)pp * C * 2;
  if (slice > kGridSliceMax) return false;
  const int r = std::max(1, (256 + V - 1) / V);
  *cpi = k;
  *per = pp;
  *R = r;
  *smem = slice + sizeof(float) * 2 * (size_t)r * C;
  return true;
}

// DI_GN_GRID=1 turns the single-launch path on (read once per process).  Off by default: inside the
// U-Net step on B200 it measured slower than the statistics-table + normalise pair (225.5 vs 232.7
// steps/s at batch 1).  The grid barrier across ~148 SMs (fence, same-address atomics, polling) and the
// fold of every CTA's partials cost about as much as the kernel boundary they replace, and the
// statistics pass gains little from more CTAs on maps of a few MB.
bool gn_grid_enabled() {
  static const bool on = [] {
    const char* e = getenv("DI_GN_GRID");
    return e && e[0] == '1';
  }();
  return on;
}

size_t gn_grid_ws_bytes(Ctx* c, int N, int HW, int C, int G) {
  int cpi, per, R;
  size_t smem;
  if (!gn_grid_geometry(c->num_sms, N, HW, C, G, &cpi, &per, &R, &smem)) return 0;
  return sizeof(float2) * (size_t)N * cpi * G;
}

// GroupNorm(+SiLU) of concat(x1, x2) (16-bit in and out) in one launch.  Returns 1 when the map does not
// fit this path or a pointer is not 16-byte aligned (nothing launched; the caller takes a two-launch
// path), 0 when launched, a negative DI_E* code on error.  `partial` holds gn_grid_ws_bytes bytes; `bar`
// is a zero-initialised {arrivals, generation} pair not used by any concurrently running launch.
// Whether gn_nhwc_grid takes this shape on this device: geometry accepted and at least one CTA per SM
// resident for every CTA of the grid (the barrier needs the whole grid at once).
bool gn_grid_usable(Ctx* c, int dtype, int N, int HW, int C1, int C2, int G) {
  const int C = C1 + C2;
  int cpi, per, R;
  size_t smem;
  if (!gn_grid_enabled() || (dtype != DI_F16 && dtype != DI_BF16) || C1 % 8 || C2 % 8 ||
      !gn_grid_geometry(c->num_sms, N, HW, C, G, &cpi, &per, &R, &smem))
    return false;
  static unsigned attr_done = 0;  // per-device bit
  if (!(attr_done & (1u << (c->device & 31)))) {
    // R * C <= 4096 for every geometry gn_grid_geometry accepts (R = ceil(256 / V), C = 8 V, V <= 512)
    const int maxdyn = (int)(kGridSliceMax + sizeof(float) * 2 * 4096);
    if (cudaFuncSetAttribute(gn_nhwc_grid<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxdyn) !=
            cudaSuccess ||
        cudaFuncSetAttribute(gn_nhwc_grid<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxdyn) !=
            cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    attr_done |= 1u << (c->device & 31);
  }
  int occ = 0;
  const cudaError_t e =
      dtype == DI_BF16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gn_nhwc_grid<__nv_bfloat16>, (C / 8) * R, smem)
                       : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gn_nhwc_grid<__half>, (C / 8) * R, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return occ >= 1 && (long long)cpi * N <= (long long)occ * c->num_sms;
}

int gn_nhwc_grid_launch(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                        float eps, const float* gamma, const float* beta, int silu, void* y, float2* partial,
                        unsigned* bar) {
  const int C = C1 + C2;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(x1) || (C2 && !al(x2)) || !al(y) || !partial || !bar) return 1;
  if (!gn_grid_usable(c, dtype, N, HW, C1, C2, G)) return 1;
  int cpi, per, R;
  size_t smem;
  gn_grid_geometry(c->num_sms, N, HW, C, G, &cpi, &per, &R, &smem);
  const dim3 grid(cpi, N), block(C / 8, R);
  if (dtype == DI_BF16)
    launch_k(gn_nhwc_grid<__nv_bfloat16>, grid, block, smem, c->stream, static_cast<const __nv_bfloat16*>(x1), C1,
             static_cast<const __nv_bfloat16*>(x2), C2, HW, per, G, eps, gamma, beta, silu,
             static_cast<__nv_bfloat16*>(y), partial, bar, c->d_err);
  else
    launch_k(gn_nhwc_grid<__half>, grid, block, smem, c->stream, static_cast<const __half*>(x1), C1,
             static_cast<const __half*>(x2), C2, HW, per, G, eps, gamma, beta, silu, static_cast<__half*>(y),
             partial, bar, c->d_err);
  const int rc = check_launch(c, "gn_nhwc_grid");
  return rc ? rc : 0;
}

// The cluster GroupNorm's geometry: pixels per CTA, pixel rows per block and dynamic shared memory.
static bool gn_cluster_geometry(int HW, int C1, int C2, int G, int* per, int* R, size_t* smem) {
  const int C = C1 + C2;
  if (HW <= 0 || C % 8 || C1 % 8 || C2 % 8 || G <= 0 || G > 128 || C % G || C / 8 > 1024) return false;
  *per = (HW + kGnCluster - 1) / kGnCluster;
  *R = std::max(1, 256 / (C / 8));
  *smem = (size_t)*per * C * 2 + 2 * sizeof(float) * (size_t)*R * C;
  // every per-CTA bulk copy starts on a 16-byte boundary: per * C1 * 2 and per * C2 * 2 are multiples of 16
  return *smem <= (200u << 10);
}

bool gn_cluster_usable(int dtype, int HW, int C1, int C2, int G) {
  if (dtype != DI_F16 && dtype != DI_BF16) return false;
  // Opt-in (DI_GN_CLUSTER=1): measured slower than the two-launch path inside the U-Net step (235.8 vs
  // 239.7 steps/s), so the statistics-table + normalise pair stays the default.
  static const bool off = [] {
    const char* e = getenv("DI_GN_CLUSTER");
    return !(e && e[0] == '1');
  }();
  int per, R;
  size_t smem;
  return !off && gn_cluster_geometry(HW, C1, C2, G, &per, &R, &smem);
}

// Returns 1 (nothing launched) when the shape does not fit the cluster path.
int gn_nhwc_cluster_launch(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                           float eps, const float* gamma, const float* beta, int silu, void* y) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (N <= 0 || !al(x1) || (C2 && !al(x2)) || !al(y) || !gn_cluster_usable(dtype, HW, C1, C2, G)) return 1;
  int per, R;
  size_t smem;
  gn_cluster_geometry(HW, C1, C2, G, &per, &R, &smem);
  static unsigned attr_done[2] = {0, 0};  // per dtype, per-device bit
  const int di = dtype == DI_BF16 ? 1 : 0;
  if (!(attr_done[di] & (1u << (c->device & 31)))) {
    const void* kern = dtype == DI_BF16 ? (const void*)gn_nhwc_cluster<__nv_bfloat16> : (const void*)gn_nhwc_cluster<__half>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 << 10) != cudaSuccess)
      return set_error(c, DI_ECUDA, "gn_nhwc_cluster: kernel attributes");
    attr_done[di] |= 1u << (c->device & 31);
  }
  const dim3 grid(kGnCluster, N), block((C1 + C2) / 8, R);
  if (dtype == DI_BF16)
    launch_k_cluster(gn_nhwc_cluster<__nv_bfloat16>, grid, block, smem, c->stream, kGnCluster,
                     static_cast<const __nv_bfloat16*>(x1), C1, static_cast<const __nv_bfloat16*>(x2), C2, HW, per, G,
                     eps, gamma, beta, silu, static_cast<__nv_bfloat16*>(y), c->d_err);
  else
    launch_k_cluster(gn_nhwc_cluster<__half>, grid, block, smem, c->stream, kGnCluster, static_cast<const __half*>(x1),
                     C1, static_cast<const __half*>(x2), C2, HW, per, G, eps, gamma, beta, silu,
                     static_cast<__half*>(y), c->d_err);
  return check_launch(c, "gn_nhwc_cluster");
}

size_t gn_nhwc_ws_bytes(int N, int HW, int G) {
  int chunks, cl;
  gn_geometry(HW, &chunks, &cl);
  return sizeof(float2) * (size_t)N * (chunks / cl) * G;
}

int group_norm_nchw(Ctx* c, const float* x, const float* g, const float* b, float* y, int N, int C, int HW, int G,
                    float eps, int silu, int clamp) {
  if (N <= 0 || C <= 0 || HW <= 0 || G <= 0 || C % G) return set_error(c, DI_EINVAL, "group_norm: bad cfg");
  const size_t gsize = (size_t)(C / G) * HW;
  const int target = 4 * c->num_sms;
  int chunks = (int)std::max<size_t>(1, std::min<size_t>((gsize + 2047) / 2048, (size_t)std::max(1, target / (N * G))));
  float2* partial = static_cast<float2*>(workspace(c, sizeof(float2) * (size_t)N * G * chunks, 0));
  if (!partial) return set_error(c, DI_ENOMEM, "group_norm: workspace");
  launch_k(gn_nchw_partial, dim3(chunks, G, N), 256, 0, c->stream, x, G, gsize, chunks, partial);
  const size_t total = (size_t)N * C * HW;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)8 * c->num_sms);
  launch_k(gn_nchw_apply, blocks, 256, 0, c->stream, x, C, G, HW, chunks, partial, g, b, eps, silu, clamp, total, y);
  return check_launch(c, "group_norm_nchw");
}

// GroupNorm(32)(+SiLU) of x [N, HW, C] (fp16) from producer statistics (Ctx::gn_stats): one pass.
int gn_apply_with_stats(Ctx* c, const void* x, int C, int N, int HW, const long long* stats, float eps,
                        const float* gamma, const float* beta, int silu, void* y) {
  if (C % 32 || C % 8 || N <= 0 || HW <= 0) return set_error(c, DI_EINVAL, "gn_apply_with_stats: shape");
  const size_t per_img = (size_t)HW * (C / 8);
  const int bx = (int)std::max<size_t>(1, std::min<size_t>((per_img + 255) / 256, (size_t)(8 * c->num_sms + N - 1) / N));
  launch_k(gn_apply_stats<__half>, dim3(bx, N), 256, sizeof(float2) * C, c->stream, static_cast<const __half*>(x), C,
           HW, stats, eps, gamma, beta, silu, static_cast<__half*>(y));
  return check_launch(c, "gn_apply_stats");
}

int layer_norm(Ctx* c, int in_dtype, int out_dtype, const void* x, const float* g, const float* b, void* y, int rows,
               int D, float eps) {
  const int blocks = (rows + 7) / 8;
  // vector path: rows of whole 8-element chunks, 16-byte aligned base pointers (fp32 gamma / beta too)
  const bool vec = D % 8 == 0 && D <= 2048 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                    reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
  const int nv = (D + 255) / 256;
#define LN_VEC(TI, TO, NV)                                                                                     \
  if (nv <= NV) {                                                                                             \
    launch_k(layer_norm_rows_vec<TI, TO, NV>, blocks, 256, 0, c->stream, static_cast<const TI*>(x), g, b,     \
             static_cast<TO*>(y), rows, D, eps);                                                              \
    return check_launch(c, "layer_norm");                                                                     \
  }
#define LN_CASE(TI, TO)                                                                                         \
  if (vec) { LN_VEC(TI, TO, 1) LN_VEC(TI, TO, 2) LN_VEC(TI, TO, 4) LN_VEC(TI, TO, 8) }                        \
  launch_k(layer_norm_rows<TI, TO>, blocks, 256, 0, c->stream, static_cast<const TI*>(x), g, b, static_cast<TO*>(y), \
                                                         rows, D, eps);                                         \
  return check_launch(c, "layer_norm")
  if (in_dtype == DI_F32 && out_dtype == DI_F32) { LN_CASE(float, float); }
  if (in_dtype == DI_F32 && out_dtype == DI_F16) { LN_CASE(float, __half); }
  if (in_dtype == DI_F16 && out_dtype == DI_F16) { LN_CASE(__half, __half); }
  if (in_dtype == DI_BF16 && out_dtype == DI_BF16) { LN_CASE(__nv_bfloat16, __nv_bfloat16); }
#undef LN_CASE
#undef LN_VEC
  return set_error(c, DI_EINVAL, "layer_norm: dtype combination");
}

}  // namespace di

using namespace di;

extern "C" {

int di_group_norm_nhwc(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                       float eps, const float* gamma, const float* beta, int fuse_silu, void* y) {
  Ctx* c = ctx_of(h);
  if (!c) return DI_EINVAL;
  if (!x2) C2 = 0;
  // With DI_GN_GRID=1, maps small enough for one CTA per SM take the single-launch kernel (16-bit data).
  const size_t ws = (dtype == DI_F16 || dtype == DI_BF16) && gn_grid_enabled() ? gn_grid_ws_bytes(c, N, HW, C1 + C2, G)
                                                                             : 0;
  if (ws) {
    if (!c->gn_bar) {
      if (cudaMalloc(&c->gn_bar, 2 * sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        c->gn_bar = nullptr;
        return set_error(c, DI_ENOMEM, "group_norm_nhwc: barrier word");
      }
      cudaMemset(c->gn_bar, 0, 2 * sizeof(unsigned));
    }
    float2* part = static_cast<float2*>(workspace(c, ws, 0));
    if (!part) return set_error(c, DI_ENOMEM, "group_norm_nhwc: workspace");
    const int r = gn_nhwc_grid_launch(c, dtype, x1, C1, x2, C2, N, HW, G, eps, gamma, beta, fuse_silu, y, part,
                                      c->gn_bar);
    if (r <= 0) return r;  // launched (0) or failed; 1: not applicable, two-launch path below
  }
  // Maps whose per-image slice fits one 16-CTA cluster's shared memory: one launch, one read, one write.
  {
    const int r = gn_nhwc_cluster_launch(c, dtype, x1, C1, x2, C2, N, HW, G, eps, gamma, beta, fuse_silu, y);
    if (r <= 0) return r;
  }
  return group_norm_nhwc(c, dtype, dtype, x1, C1, x2, C2, N, HW, G, eps, gamma, beta, fuse_silu, y, nullptr);
}

int di_gn_table_nhwc(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW, int G,
                     float eps, const float* gamma, const float* beta, float* table) {
  Ctx* c = ctx_of(h);
  if (!c || !table || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  return gn_table_nhwc(c, dtype, x1, C1, x2, x2 ? C2 : 0, N, HW, G, eps, gamma, beta, reinterpret_cast<float2*>(table));
}

int di_group_norm(di_ctx_t h, const float* X, const float* gamma, const float* beta, float* Y, const void* cfg32,
                  int fuse_silu) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg32) return DI_EINVAL;
  const uint32_t* u = static_cast<const uint32_t*>(cfg32);
  float eps;
  memcpy(&eps, u + 4, 4);
  const int N = u[0], G = u[1], cpg = u[2], HW = u[3];
  return group_norm_nchw(c, X, gamma, beta, Y, N, G * cpg, HW, G, eps, fuse_silu, 1);
}

int di_instance_norm(di_ctx_t h, const float* X, const float* gamma, const float* beta, float* Y,
                     const uint32_t cfg[4]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg) return DI_EINVAL;
  // cfg = {C, HW, N, _}; eps hard-coded 1e-5 as in wgsl-ops.js:313-317.
  return group_norm_nchw(c, X, gamma, beta, Y, (int)cfg[2], (int)cfg[0], (int)cfg[1], (int)cfg[0], 1e-5f, 0, 1);
}

int di_layer_norm(di_ctx_t h, const float* X, const float* gamma, const float* beta, float* Y, const uint32_t cfg[2]) {
  Ctx* c = ctx_of(h);
  if (!c || !cfg) return DI_EINVAL;
  // cfg = {innerLen, rows}; eps 1e-5 (wgsl-ops.js:780).
  return layer_norm(c, DI_F32, DI_F32, X, gamma, beta, Y, (int)cfg[1], (int)cfg[0], 1e-5f);
}

}  // extern "C"
