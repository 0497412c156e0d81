// k_gemm.cu — tcgen05 / TMEM / TMA GEMM and implicit-GEMM 3x3 convolution (sm_100a).
//
// Replaces the reference's 64x64 fp32 FMA tiles (WGSL_MATMUL wgsl-ops.js:477-556, WGSL_GEMM :821-897,
// WGSL_CONV_MM :584-698, the fused-block matmuls fused-block-full.js:128-186, and the direct convs
// fused-resnet.js:173-208 / fused-conv.js:50-100) with one warp-specialised tensor-core kernel:
//
//   warp 0      TMA producer: A tile (128 rows x 64 K, 128B-swizzled) + B tile (BN rows x 64 K) per stage
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per stage, accumulator in TMEM,
//               tcgen05.commit releases the stage back to the producer
//   warps 2..5  epilogue: tcgen05.ld of the 128 x BN fp32 accumulator (one TMEM lane = one output row),
//               + bias + per-image row vector (timestep embedding) + residual, or the GEGLU gate,
//               converted and stored.
//
// A-operand modes (the "implicit im2col" is done by the TMA unit, no im2col buffer exists):
//   0  linear: A = X[M,K] row-major, optionally concat(X1[:, :K1], X2[:, K1:]) along K (two maps)
//   1  conv 3x3 stride 1 pad 1, NHWC: one 4-D box {64 ch, Wo, rows, images} per (tap, 64-channel block),
//      shifted by (ky-1, kx-1); out-of-range rows/columns are zero-filled by TMA = the conv padding.
//      Two input tensors (skip concat) are two maps split on the channel block.
//   2  conv 3x3 stride 2 pad 1: four parity maps (even/odd row x even/odd column) so every tap is a
//      unit-stride box of the half-resolution grid.
// B = weights [N rows, K] K-major; conv weights packed [Co][ky][kx][Ci] so K order = (tap, channel).
//
// Every mbarrier wait is time-bounded (di_common.cuh): on timeout the kernel records an error code,
// skips the remaining work, frees its TMEM and returns.
#include <algorithm>
#include <mutex>

#include "di_common.cuh"

namespace di {

Ctx* ctx_of(di_ctx_t h);

struct GemmParams {
  CUtensorMap tmA[4];
  CUtensorMap tmB;
  int staged;       // epilogue stores through the shared-memory staging slab (16-byte aligned rows)
  int mode;        // 0 linear, 1 conv s1, 2 conv s2
  int M, N;        // output rows, accumulator columns (geglu: 2F packed columns)
  int num_k;       // K blocks of 64
  int k_split;     // K (or channel) blocks served by source 0
  int cin_blocks;  // conv: channel blocks per tap
  int HWo, Wo;     // conv: output pixels per image, output width
  const float* bias;
  const float* rowvec;  // adds rowvec[(m / rowvec_div) * rowvec_ld + n]
  int rowvec_div, rowvec_ld;
  const void* residual;  // [M, ldr] (out dtype, or fp32 when res_f32)
  int ldr, res_f32;
  void* out;
  int ldo, out_f32;
  int geglu;
  int act;  // after bias / row vector, before the residual: 0 none, 1 SiLU (y = silu(acc + b) + r), 2 GELU (erf)
  int vec_ok;  // 16-byte aligned rows for out / residual: vectorised epilogue
  int b_early;     // weights are constant data: fetch the first B stages before the dependency wait
  int splits;      // K splits; > 1 writes raw fp32 partials, the reduce kernel applies the epilogue
  // Cluster split-K (splits > 1, launched as clusters of `splits` CTAs): CTA rank r of a cluster takes K
  // split r of the cluster's tiles, and the cluster sums its partials through distributed shared memory in
  // the epilogue (fixed rank order), so no fp32 partials reach global memory and no reduce kernel runs.
  int cs;
  // 16-bit output stored by TMA from the 64-byte-swizzled staging slab (box 32 x 32): set by launch_gemm
  CUtensorMap tmO;
  int tma_out;
  // LayerNorm of the A rows folded in (plain and GEGLU instantiations, no split, single CTAs): the B rows
  // hold W[n][k] * gamma[k], ln_c1[n] = sum_k of those, and the bias holds b[n] + sum_k W[n][k] * beta[k];
  // the epilogue warps take each row's mean / rstd from the A tiles in shared memory during the main loop
  // and the epilogue computes rstd * (acc - mean * ln_c1[n]) + bias[n].
  int ln;
  float ln_eps;
  const float* ln_c1;
  int dbg;  // diagnostics (DI_GEMM_DEBUG): 1 skip output / partial stores, 2 skip the bias/residual epilogue
  int m_tiles, n_tiles;  // 128-row M tiles and BN-column N tiles (set by launch_gemm)
  float* partial;  // [splits][M][N] fp32 when splits > 1
  long long* gstats;  // GroupNorm(32) statistics of the fp16 output (Ctx::gn_stats), or null
  int g_cpg, g_hw;    // channels per group (N / 32), output rows per image
  int* err;
  unsigned long long* trace;  // diagnostics: kTracePoints %globaltimer stamps per CTA, or null
  // GroupNorm(+SiLU) of the A operand (GnFuse): applied in shared memory by the epilogue warps between
  // the TMA load and the MMA; gn_C = input channels, gn_HW = pixels per image, conv_bh = image rows
  // per 128-row conv tile.
  const float2* gn_tab;
  int gn_silu, gn_C, gn_HW, conv_bh;
};

// Diagnostics: per-CTA timeline points of the first work unit (di_debug_gemm_trace).
constexpr int kTracePoints = 16;
static unsigned long long* g_trace = nullptr;
static int g_trace_ctas = 0;
static const bool g_gemm_generic = [] {  // diagnostics: DI_GEMM_GENERIC=1 never uses the plain epilogue
  const char* e = getenv("DI_GEMM_GENERIC");
  return e && e[0] == '1';
}();

namespace {

constexpr int BM = 128, BK = 64;
// Warps: 0 = TMA producer, 1 = MMA issuer, 2 .. 2 + kEpiWarps - 1 = epilogue.  Two epilogue warps share
// each TMEM lane quarter (a warp may only read lanes 32 * (warp % 4) ..), splitting the column chunks.
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;

template <int BN, int STAGES, bool PAIR = false>
struct GemmSmem {
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // a pair splits B's rows
  static constexpr uint32_t EPI_BYTES = kEpiWarps * 4096;  // one 32 x 128 B staging slab per epilogue warp
  static constexpr uint32_t TOTAL = 1024 + STAGES * (A_BYTES + B_BYTES) + EPI_BYTES + 512;  // + align + barriers
};

__device__ __forceinline__ void store_row32(void* out, size_t off, const float* v, int out_f32, bool bf16) {
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + off);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (bf16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + off);
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  }
}

__device__ __forceinline__ void load_row32(const void* src, size_t off, float* v, int is_f32, bool bf16) {
  if (is_f32) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(src) + off);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 t = s[j];
      v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
  } else {
    const uint4* s = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + off);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 t = s[j];
      uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f;
        if (bf16) f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[q]));
        else f = __half22float2(*reinterpret_cast<__half2*>(&w[q]));
        v[8 * j + 2 * q] = f.x; v[8 * j + 2 * q + 1] = f.y;
      }
    }
  }
}

__device__ __forceinline__ float load_one(const void* src, size_t off, int is_f32, bool bf16) {
  if (is_f32) return static_cast<const float*>(src)[off];
  if (bf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[off]);
  return __half2float(static_cast<const __half*>(src)[off]);
}
__device__ __forceinline__ void store_one(void* dst, size_t off, float v, int is_f32, bool bf16) {
  if (is_f32) static_cast<float*>(dst)[off] = v;
  else if (bf16) static_cast<__nv_bfloat16*>(dst)[off] = __float2bfloat16_rn(v);
  else static_cast<__half*>(dst)[off] = __float2half_rn(v);
}

// Persistent tile-scheduled kernel: grid = min(units, SMs), one CTA per SM.  A unit is one
// (K split, 128-row M tile, BN-column N tile); CTA b processes units b, b + grid, ...  The smem ring
// runs continuously across units, and the accumulator is double-buffered in TMEM (2 x BN columns)
// so the epilogue of one unit overlaps the main loop of the next.
//
// PAIR: clusters of two CTAs on two SMs run one 256-row tile with cta_group::2 MMAs.  Each CTA loads its
// own 128 A rows and half of B's BN rows, so a K block moves (128 + BN/2) rows per SM instead of
// (128 + BN): the main loop is bound by each SM's L2 -> shared-memory rate, so this halves the B
// traffic per FLOP.  The leader (rank 0) issues the MMAs; the peer's TMA loads count their bytes on the
// leader's `full` barrier; MMA commits arrive on `empty` / `tfull` in both CTAs; both CTAs' epilogue
// warps release the accumulator on the leader's `tempty`.  Units then index 256-row M tiles.
// GroupNorm(32) statistics of one warp's 32 x 32 output chunk (rows r0 .., lane = row, columns nb ..):
// the values as stored (rounded to fp16), reduced over the warp per group, three int64 atomics per
// group touched.  The chunk's rows belong to one image (rows per image are a multiple of 32).
template <typename P>
__device__ __forceinline__ void gn_stats_chunk(const float (&v)[32], int nb, int r0, int m, int lane, const P& p) {
  // a 32-column chunk meets at most 5 groups for cpg >= 8 (the GroupNorm(32) consumers here have C >= 256)
  const int cpg = p.g_cpg;
  const int g0 = nb / cpg;
  const int n = r0 / p.g_hw;
  long long s[5] = {0, 0, 0, 0, 0}, hi[5] = {0, 0, 0, 0, 0}, lo[5] = {0, 0, 0, 0, 0};
  if (m < p.M) {
    int k = 0, next = (g0 + 1) * cpg - nb;  // chunk column where group g0 + k + 1 starts
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j == next) { ++k; next += cpg; }
      if (nb + j < p.N) {
        long long a, b, c;
        gn_fixed(__half2float(__float2half_rn(v[j])), a, b, c);
#pragma unroll
        for (int t = 0; t < 5; ++t)
          if (t == k) { s[t] += a; hi[t] += b; lo[t] += c; }
      }
    }
  }
  const int ng = min(5, min(31, (min(nb + 31, p.N - 1)) / cpg) - g0 + 1);
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    if (t >= ng) break;
    long long a = s[t], b = hi[t], c = lo[t];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
      c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    if (lane == 0) {
      unsigned long long* d = reinterpret_cast<unsigned long long*>(p.gstats + ((size_t)n * 32 + g0 + t) * 3);
      atomicAdd(d, (unsigned long long)a);
      atomicAdd(d + 1, (unsigned long long)b);
      atomicAdd(d + 2, (unsigned long long)c);
    }
  }
}

// MODE: 0 generic epilogue (every runtime variant), 1 operand-fused GroupNorm (XF), 2 plain epilogue: 16-bit
// output through the staging slab, no split-K, GEGLU, statistics or fp32 operands (compiled without them);
// 3 split-K partials: raw fp32 partial stores only (no epilogue arithmetic, no GEGLU / statistics / cluster);
// 4 GEGLU without split: value * GELU(gate) to a 16-bit output.
template <int BN, int STAGES, bool BF16, bool PAIR = false, int MODE = 0>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  using S = GemmSmem<BN, STAGES, PAIR>;
  constexpr uint32_t STAGE_TX = S::A_BYTES + S::B_BYTES;
  constexpr uint32_t TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint8_t* sEpi = sB + STAGES * S::B_BYTES;  // 1024-aligned: A and B stage sizes are multiples of 1 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + S::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained by the epilogue
  uint64_t* afull = tempty + 2;       // [STAGES] this CTA's A tile landed (operand-fused GroupNorm only)
  uint64_t* aready = afull + STAGES;  // [STAGES] A tiles transformed (on the pair leader: both CTAs')
  uint64_t* xfull = aready + STAGES;   // [kEpiWarps] cluster split-K: every rank's slab of this warp written
  uint64_t* xempty = xfull + kEpiWarps;  // [kEpiWarps] cluster split-K: every rank done reading this warp's slab
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xempty + kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;  // 0 = leader
  // Cluster split-K: rank csr runs split csr of tiles cluster, cluster + clusters, ... (units
  // csr * per_split + tile), so every CTA of a cluster walks the same tiles in the same order.
  const int CS = (PAIR || MODE >= 2) ? 0 : p.cs;  // cluster size of the split-K cluster, 0 = off
  const int csr = CS ? (int)cluster_ctarank() : 0;
  const int cta0 = PAIR ? blockIdx.x >> 1 : (CS ? csr * p.m_tiles * p.n_tiles + (int)blockIdx.x / CS : blockIdx.x);
  const int cstride = PAIR ? gridDim.x >> 1 : (CS ? (int)gridDim.x / CS : gridDim.x);
  unsigned long long* tr = p.trace ? p.trace + (size_t)blockIdx.x * kTracePoints : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  const int nt = p.n_tiles, per_split = p.m_tiles * p.n_tiles;
  const int units = CS ? (csr + 1) * per_split : per_split * p.splits;  // loop bound of this CTA's units
  const int kper = (p.num_k + p.splits - 1) / p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (!PAIR && p.ln) ? 1 + kEpiWarps : 1);  // + the LayerNorm statistics readers
      mbar_init(&afull[s], 1);
      mbar_init(&aready[s], (PAIR ? 2 : 1) * kEpiWarps);  // one arrival per transforming warp
    }
    // tempty: one arrival per epilogue warp (of both CTAs of a pair, on the leader's barrier)
    for (int s = 0; s < 2; ++s) { mbar_init(&tfull[s], 1); mbar_init(&tempty[s], (PAIR ? 2 : 1) * kEpiWarps); }
    for (int w = 0; w < kEpiWarps; ++w) { mbar_init(&xfull[w], CS ? CS : 1); mbar_init(&xempty[w], CS ? CS : 1); }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (PAIR) { tmem_alloc_pair(tmem_slot, TMEM_COLS); tmem_relinquish_pair(); }
    else { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
  }
  tc_fence_before();
  if (PAIR || CS) cluster_sync();  // every CTA's barriers initialised before any cross-CTA signal
  else __syncthreads();
  tc_fence_after();
  const uint32_t full0_leader = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
  const uint32_t tempty_leader = PAIR ? mapa_shared(smem_u32(tempty), 0) : smem_u32(tempty);
  const uint32_t aready_leader = PAIR ? mapa_shared(smem_u32(aready), 0) : smem_u32(aready);
  constexpr bool xform = MODE == 1;  // operand-fused GroupNorm (p.gn_tab): a separate instantiation
  constexpr bool PLAIN = MODE == 2, PARTIAL = MODE == 3, GEGLU = MODE == 4;
  const int out_f32 = (PLAIN || GEGLU) ? 0 : p.out_f32, res_f32 = PLAIN ? 0 : p.res_f32, vec_ok = PLAIN ? 1 : p.vec_ok;
  const int staged = PLAIN ? 1 : p.staged;
  const uint32_t tmem = *tmem_slot;
  if (tr && threadIdx.x == 0) tr[1] = globaltimer();
  // Programmatic dependent launch: let the next kernel be scheduled right away.  Everything before
  // pdl_wait() below reads only constant data (tensor maps, weights), so it overlaps the previous
  // kernel's tail; activations are read only after the wait.
  pdl_trigger();

  // m0: this CTA's first output row (a pair's tile is 256 rows, the peer takes the second 128)
  auto decode = [&](int u, int& m0, int& n0, int& sp, int& kb0, int& kb1) {
    sp = u / per_split;
    const int r = u - sp * per_split;
    m0 = (r / nt) * (PAIR ? 2 * BM : BM) + (int)rank * BM;
    n0 = (r % nt) * BN;
    kb0 = sp * kper;
    kb1 = min(p.num_k, kb0 + kper);
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      for (int i = 0; i < 4; ++i) tma_prefetch_desc(&p.tmA[i]);
      tma_prefetch_desc(&p.tmB);
      // Weight tiles of the first ring stages are requested before the dependency wait (constant data).
      // In a pair, rank r loads B rows n0 + r * BN/2 .. and only the leader arms `full` (both CTAs' bytes).
      const int brow = PAIR ? (int)rank * (BN / 2) : 0;
      // `full` counts the bytes the MMA needs; with the fused GroupNorm the A tile instead lands on this
      // CTA's own `afull` (for the transforming warps) and `full` only counts B.
      auto armB = [&](int s) {
        const uint32_t tx = xform ? S::B_BYTES : STAGE_TX;
        if (!PAIR) mbar_arrive_expect_tx(&full[s], tx);
        else if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * tx);
      };
      auto armA = [&](int s) {
        if (xform) mbar_arrive_expect_tx(&afull[s], S::A_BYTES);
      };
      auto load2 = [&](void* dst, const CUtensorMap* m, int s, int c0, int c1) {
        if (PAIR) tma_load_2d_pair(dst, m, full0_leader + s * 8, c0, c1);
        else tma_load_2d(dst, m, &full[s], c0, c1);
      };
      auto loadA2 = [&](void* dst, const CUtensorMap* m, int s, int c0, int c1) {
        if (xform) tma_load_2d(dst, m, &afull[s], c0, c1);
        else load2(dst, m, s, c0, c1);
      };
      auto loadA4 = [&](void* dst, const CUtensorMap* m, int s, int c0, int c1, int c2, int c3) {
        if (xform) tma_load_4d(dst, m, &afull[s], c0, c1, c2, c3);
        else if (PAIR) tma_load_4d_pair(dst, m, full0_leader + s * 8, c0, c1, c2, c3);
        else tma_load_4d(dst, m, &full[s], c0, c1, c2, c3);
      };
      int npre = 0;
      {
        int m0, n0, sp, kb0, kb1;
        decode(cta0, m0, n0, sp, kb0, kb1);
        npre = p.b_early ? min(STAGES, kb1 - kb0) : 0;
        for (int i = 0; i < npre; ++i) {
          armB(i);
          load2(sB + i * S::B_BYTES, &p.tmB, i, (kb0 + i) * BK, n0 + brow);
        }
      }
      pdl_wait();
      if (tr) tr[2] = globaltimer();
      int it = 0;
      for (int u = cta0; u < units && !*abort_flag; u += cstride) {
        int m0, n0, sp, kb0, kb1;
        decode(u, m0, n0, sp, kb0, kb1);
        int img = 0, y0 = 0, x0 = 0;  // tile origin; x0 > 0 only for rows wider than a tile
        if (p.mode != 0) {
          img = m0 / p.HWo;
          y0 = (m0 % p.HWo) / p.Wo;
          x0 = (m0 % p.HWo) % p.Wo;
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const bool pre = it < npre;  // B already requested, barrier already armed
          if (!pre) {
            if (*abort_flag || !mbar_wait<PAIR>(&empty[s], ph ^ 1, p.err, DEVERR_WAIT_TMA)) { *abort_flag = 1; break; }
            armB(s);
          }
          armA(s);
          uint8_t* dA = sA + s * S::A_BYTES;
          if (p.mode == 0) {
            if (kb < p.k_split) loadA2(dA, &p.tmA[0], s, kb * BK, m0);
            else loadA2(dA, &p.tmA[1], s, (kb - p.k_split) * BK, m0);
          } else {
            const int tap = kb / p.cin_blocks, cb = kb % p.cin_blocks;
            const int ky = tap / 3, kx = tap % 3;
            if (p.mode == 1) {
              const bool first = cb < p.k_split;
              loadA4(dA, &p.tmA[first ? 0 : 1], s, (first ? cb : cb - p.k_split) * BK, x0 + kx - 1, y0 + ky - 1,
                     img);
            } else {
              const int py = ky == 1 ? 0 : 1, px = kx == 1 ? 0 : 1;
              loadA4(dA, &p.tmA[py * 2 + px], s, cb * BK, x0 + (kx == 0 ? -1 : 0), y0 + (ky == 0 ? -1 : 0), img);
            }
          }
          if (!pre) load2(sB + s * S::B_BYTES, &p.tmB, s, kb * BK, n0 + brow);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the pair leader only) ----------------
    if (rank == 0 && elect_one()) {
      constexpr uint32_t idesc = idesc_f16(PAIR ? 2 * BM : BM, BN, BF16);
      auto commit = [&](uint64_t* bar) {
        if (PAIR) umma_commit_pair(bar, 0x3);
        else umma_commit(bar);
      };
      int it = 0, lt = 0;
      for (int u = cta0; u < units; u += cstride, ++lt) {
        int m0, n0, sp, kb0, kb1;
        decode(u, m0, n0, sp, kb0, kb1);
        const int ab = lt & 1;
        if (*abort_flag || !mbar_wait<PAIR>(&tempty[ab], ((lt >> 1) & 1) ^ 1, p.err, DEVERR_WAIT_MMA)) {
          *abort_flag = 1;
          commit(&tfull[ab]);
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + ab * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (*abort_flag || !mbar_wait<PAIR>(&full[s], ph, p.err, DEVERR_WAIT_MMA) ||
              (xform && !mbar_wait<PAIR>(&aready[s], ph, p.err, DEVERR_WAIT_MMA))) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          if (tr && lt == 0 && kb == kb0) tr[3] = globaltimer();
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * S::A_BYTES), b0 = smem_u32(sB + s * S::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + k * 32, 16, 1024);
            if (PAIR) umma_f16_pair(dt, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else umma_f16(dt, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          commit(&empty[s]);
        }
        commit(&tfull[ab]);
        if (tr && lt == 0) tr[4] = globaltimer();
        if (!ok) break;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    // Per 32-column chunk: tcgen05.ld of this warp's 32 accumulator rows, bias / row vector / residual /
    // GEGLU in registers, then (staged) the 32x32 tile goes through a swizzled shared-memory slab and is
    // written back with whole-row-segment (coalesced) stores, or else it is stored row by row.
    pdl_wait();  // residual reads / output writes follow the previous kernel
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int half = (warp - 2) / 4;  // which alternate column chunks this warp handles
    uint8_t* stg = sEpi + (warp - 2) * 4096;
    const bool LN = (PLAIN || GEGLU) && !PAIR && p.ln;
    float ln_rs = 1.f, ln_rm = 0.f;  // this row's rstd and rstd * mean (LayerNorm fold)
    int lit = 0;                     // ring position of the statistics readers (same sequence as the producer)
    // Epilogue on one row's 32 columns: bias, per-image row vector, activation, residual (not GEGLU).
    auto epi = [&](float (&v)[32], int nb, int m) {
      const int n_out = p.N;
      const bool full = nb + 32 <= n_out;
      if (LN) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (nb + j < n_out) v[j] = fmaf(ln_rs, v[j], -ln_rm * p.ln_c1[nb + j]);
      }
      if (p.bias) {
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += __ldg(p.bias + nb + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < n_out) v[j] += p.bias[nb + j];
        }
      }
      if (p.rowvec) {
        const float* rv = p.rowvec + (size_t)(m / p.rowvec_div) * p.rowvec_ld + nb;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += __ldg(rv + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < n_out) v[j] += rv[j];
        }
      }
      if (p.act == 1) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
      } else if (p.act == 2) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
      }
      if (p.residual) {
        if (full && vec_ok) {
          float rr[32];
          load_row32(p.residual, (size_t)m * p.ldr + nb, rr, res_f32, BF16);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += rr[j];
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < n_out) v[j] += load_one(p.residual, (size_t)m * p.ldr + nb + j, res_f32, BF16);
        }
      }
    };
    // Stores one warp's 32 x 32 chunk (rows m0 + 32q .., columns nb ..): to the fp32 split-K partials
    // (to_partial) or to the output, through the staging slab (staged) or row by row.
    auto store_chunk = [&](const float (&v)[32], int nb, int m0, int m, int sp, bool to_partial, bool staged) {
      const int n_out = to_partial ? p.N : (p.geglu ? p.N / 2 : p.N);
      if (staged) {
        // The warp's 32 x 32 tile goes through a swizzled staging slab (conflict-free writes of one row
        // per lane), then is read back so that each store instruction writes whole 64/128-byte row
        // segments of 8 or 4 rows (coalesced), instead of 32 rows 16 bytes at a time.
        if (p.tma_out && lane == 0) bulk_wait_read0();  // the previous chunk's TMA store has read the slab
        __syncwarp();  // the previous chunk's read-back is done
        if (to_partial || out_f32) {
          // 32 fp32 per row = 128 B; 16-byte chunk j of row r at j ^ (r & 7)
          float4* rp = reinterpret_cast<float4*>(stg + lane * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            rp[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
          // 32 x 16-bit per row = 64 B; 16-byte chunk j of row r at j ^ ((r >> 1) & 3)
          uint4* rp = reinterpret_cast<uint4*>(stg + lane * 64);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float x0 = v[8 * j + 2 * k], x1 = v[8 * j + 2 * k + 1];
              if (BF16) {
                __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
                w[k] = *reinterpret_cast<uint32_t*>(&h2);
              } else {
                __half2 h2 = __floats2half2_rn(x0, x1);
                w[k] = *reinterpret_cast<uint32_t*>(&h2);
              }
            }
            rp[j ^ ((lane >> 1) & 3)] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        __syncwarp();
        const int mrow0 = m0 + q * 32;
        if (to_partial || out_f32) {
          float* base = to_partial ? p.partial + (size_t)sp * p.M * p.N : static_cast<float*>(p.out);
          const int ld = to_partial ? p.N : p.ldo;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3), ch = lane & 7;
            const float4 val = reinterpret_cast<const float4*>(stg + r * 128)[ch ^ (r & 7)];
            const int mm = mrow0 + r, col = nb + ch * 4;
            if (mm < p.M && col < n_out) {
              float* d = base + (size_t)mm * ld + col;
              if (col + 4 <= n_out) {
                *reinterpret_cast<float4*>(d) = val;
              } else {
                const float t[4] = {val.x, val.y, val.z, val.w};
                for (int k = 0; k < 4 && col + k < n_out; ++k) d[k] = t[k];
              }
            }
          }
        } else if (p.tma_out) {
          // the slab's 16-byte chunk j of row r sits at j ^ ((r >> 1) & 3): the TMA 64-byte swizzle
          fence_async_smem();  // this lane's slab writes, visible to the TMA unit
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&p.tmO, stg, nb, mrow0);
            bulk_commit();
          }
        } else {
          uint16_t* base = static_cast<uint16_t*>(p.out);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i * 8 + (lane >> 2), ch = lane & 3;
            const uint4 val = reinterpret_cast<const uint4*>(stg + r * 64)[ch ^ ((r >> 1) & 3)];
            const int mm = mrow0 + r, col = nb + ch * 8;
            if (mm < p.M && col < n_out) {
              uint16_t* d = base + (size_t)mm * p.ldo + col;
              if (col + 8 <= n_out) {
                *reinterpret_cast<uint4*>(d) = val;
              } else {
                const uint32_t t[4] = {val.x, val.y, val.z, val.w};
                for (int k = 0; k < 8 && col + k < n_out; ++k) d[k] = static_cast<uint16_t>(t[k >> 1] >> (16 * (k & 1)));
              }
            }
          }
        }
      } else if (m < p.M) {
        if (to_partial) {
          float* dst = p.partial + ((size_t)sp * p.M + m) * p.N + nb;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < p.N) dst[j] = v[j];
        } else if (vec_ok && nb + 32 <= n_out) {
          store_row32(p.out, (size_t)m * p.ldo + nb, v, out_f32, BF16);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (nb + j < n_out) store_one(p.out, (size_t)m * p.ldo + nb + j, v[j], out_f32, BF16);
        }
      }
    };
    // Cluster split-K epilogue of one 32 x 32 chunk (this warp's rows m0 + 32q .., columns nb ..): the raw
    // partial goes to this warp's slab; once every rank's slab of this warp holds the same chunk, rank r
    // sums rows r, r + CS, ... over the ranks' slabs in rank order (distributed shared memory reads),
    // applies the epilogue and stores them.  Rounds alternate on xfull / xempty (one arrival per rank).
    int xr = 0;
    const int ew = warp - 2;
    auto cs_reduce = [&](const float (&v)[32], int nb, int m0, int n_out) -> bool {
      if (xr > 0 && !mbar_wait<true>(&xempty[ew], (xr - 1) & 1, p.err, DEVERR_WAIT_EPI)) return false;
      float4* rp = reinterpret_cast<float4*>(stg + lane * 128);
#pragma unroll
      for (int j = 0; j < 8; ++j) rp[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      __syncwarp();
      if (lane < CS) mbar_arrive_cluster(mapa_shared(smem_u32(&xfull[ew]), lane));
      if (!mbar_wait<true>(&xfull[ew], xr & 1, p.err, DEVERR_WAIT_EPI)) return false;
      const int sub = lane >> 3, quad = lane & 7;
      const uint32_t sl = smem_u32(stg);
      const int nown = (32 - csr + CS - 1) / CS;  // rows csr, csr + CS, ... below 32
      for (int k0 = 0; k0 < nown; k0 += 4) {
        const int k = k0 + sub, r = csr + CS * k;
        if (k < nown) {
          const uint32_t off = sl + r * 128 + ((quad ^ (r & 7)) << 4);
          float4 a = ld_cluster_f4(mapa_shared(off, 0));
          for (int pr = 1; pr < CS; ++pr) {
            const float4 b = ld_cluster_f4(mapa_shared(off, pr));
            a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
          }
          const int mm = m0 + q * 32 + r, col = nb + quad * 4;
          if (mm < p.M && col < n_out) {
            float f[4] = {a.x, a.y, a.z, a.w};
            const int nc = min(4, n_out - col);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (j < nc) {
                if (p.bias) f[j] += __ldg(p.bias + col + j);
                if (p.rowvec) f[j] += __ldg(p.rowvec + (size_t)(mm / p.rowvec_div) * p.rowvec_ld + col + j);
                if (p.act == 1) f[j] = silu_f(f[j]);
                else if (p.act == 2) f[j] = gelu_erf(f[j]);
                if (p.residual) f[j] += load_one(p.residual, (size_t)mm * p.ldr + col + j, p.res_f32, BF16);
              }
            }
            const size_t o = (size_t)mm * p.ldo + col;
            if (nc == 4 && p.vec_ok) {
              if (p.out_f32) {
                *reinterpret_cast<float4*>(static_cast<float*>(p.out) + o) = make_float4(f[0], f[1], f[2], f[3]);
              } else {
                uint32_t w0, w1;
                if (BF16) {
                  __nv_bfloat162 h0 = __floats2bfloat162_rn(f[0], f[1]), h1 = __floats2bfloat162_rn(f[2], f[3]);
                  w0 = *reinterpret_cast<uint32_t*>(&h0); w1 = *reinterpret_cast<uint32_t*>(&h1);
                } else {
                  __half2 h0 = __floats2half2_rn(f[0], f[1]), h1 = __floats2half2_rn(f[2], f[3]);
                  w0 = *reinterpret_cast<uint32_t*>(&h0); w1 = *reinterpret_cast<uint32_t*>(&h1);
                }
                *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + o) = make_uint2(w0, w1);
              }
            } else {
              for (int j = 0; j < nc; ++j) store_one(p.out, o + j, f[j], p.out_f32, BF16);
            }
          }
        }
      }
      __syncwarp();
      if (lane < CS) mbar_arrive_cluster(mapa_shared(smem_u32(&xempty[ew]), lane));
      ++xr;
      return true;
    };
    int lt = 0, xit = 0;
    for (int u = cta0; u < units; u += cstride, ++lt) {
      int m0, n0, sp, kb0, kb1;
      decode(u, m0, n0, sp, kb0, kb1);
      const int ab = lt & 1;
      const int m = m0 + row;
      if (xform) {
        // ---- operand-fused GroupNorm: normalise (+SiLU) this unit's A tiles in shared memory ----
        // Thread tt handles the 16-byte chunks tt + 256 i (i < 4) of the 128 x 8-chunk tile: a warp
        // instruction covers four whole 128-byte rows (bank-conflict free).  Rows outside the image
        // (conv padding, zero-filled by TMA) and rows past M are left as loaded (zero).
        const int tt = (warp - 2) * 32 + lane, pc = tt & 7;
        int r_img[4], r_y[4], r_x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rw = (tt >> 3) + 32 * i, mr = m0 + rw;
          r_y[i] = 0;
          r_x[i] = 0;
          if (p.mode == 0) {
            r_img[i] = mr < p.M ? mr / p.gn_HW : -1;
          } else {  // output pixel of tile row rw (any tile geometry)
            const int pix = mr % p.HWo;
            r_img[i] = mr < p.M ? mr / p.HWo : -1;
            r_y[i] = pix / p.Wo;
            r_x[i] = pix % p.Wo;
          }
        }
        const int Ho = p.mode == 0 ? 0 : p.HWo / p.Wo;
        // The unit's (scale, shift) rows are staged in the epilogue slabs (free until this unit's
        // epilogue; the barrier keeps the previous unit's epilogue stores out of the way) when they fit,
        // so the per-K-block lookups are shared-memory reads instead of global-memory round trips.
        const int img_lo = m0 / p.gn_HW, img_hi = (min(m0 + BM, p.M) - 1) / p.gn_HW;
        const int tab_n = (img_hi - img_lo + 1) * p.gn_C;  // (scale, shift) pairs
        const bool tab_smem = tab_n * 8 <= (int)S::EPI_BYTES;
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kEpiWarps) : "memory");
        if (tab_smem) {
          const float4* src = reinterpret_cast<const float4*>(p.gn_tab + (size_t)img_lo * p.gn_C);
          float4* dst = reinterpret_cast<float4*>(sEpi);
          for (int i = tt; i < tab_n / 2; i += 32 * kEpiWarps) dst[i] = __ldg(src + i);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kEpiWarps) : "memory");
        const float4* tab_base = tab_smem ? reinterpret_cast<const float4*>(sEpi) - (size_t)img_lo * p.gn_C / 2
                                          : reinterpret_cast<const float4*>(p.gn_tab);
        for (int kb = kb0; kb < kb1; ++kb, ++xit) {
          const int s = xit % STAGES;
          const uint32_t ph = (xit / STAGES) & 1;
          if (tr && lt == 0 && threadIdx.x == 64 && kb == kb0) tr[8] = globaltimer();
          const bool okx = mbar_wait(&afull[s], ph, p.err, DEVERR_WAIT_EPI) && !*abort_flag;
          if (tr && lt == 0 && threadIdx.x == 64 && kb == kb0) tr[9] = globaltimer();
          if (tr && lt == 0 && threadIdx.x == 64 && kb == kb0 + 1) tr[12] = globaltimer();
          int gch, dy = 0, dx = 0;
          if (p.mode == 0) {
            gch = kb * BK;
          } else {
            const int tap = kb / p.cin_blocks;
            gch = (kb % p.cin_blocks) * BK;
            dy = tap / 3 - 1;
            dx = tap % 3 - 1;
          }
          uint8_t* tile = sA + s * S::A_BYTES;
          // all loads of the four chunks first (independent), then the arithmetic, then the stores
          uint4 raw[4];
          float4 tv[4][4];
          bool vld[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rw = (tt >> 3) + 32 * i;
            bool valid = okx && r_img[i] >= 0;
            if (p.mode != 0)
              valid = valid && (unsigned)(r_y[i] + dy) < (unsigned)Ho && (unsigned)(r_x[i] + dx) < (unsigned)p.Wo;
            vld[i] = valid;
            const int lc = pc ^ (rw & 7);  // 128B swizzle: physical chunk pc of row rw holds logical chunk lc
            const float4* tb = tab_base + ((size_t)(valid ? r_img[i] : img_lo) * p.gn_C + gch + lc * 8) / 2;
            raw[i] = *reinterpret_cast<const uint4*>(tile + rw * 128 + pc * 16);
#pragma unroll
            for (int e = 0; e < 4; ++e) tv[i][e] = tb[e];  // (scale, shift) of channels 2e, 2e + 1
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float4 t = tv[i][e];
              float2 f;
              if (BF16) f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[e]));
              else f = __half22float2(*reinterpret_cast<__half2*>(&w[e]));
              const float y0 = fmaf(f.x, t.x, t.y), y1 = fmaf(f.y, t.z, t.w);
              if (BF16) {
                __nv_bfloat162 h = __floats2bfloat162_rn(y0, y1);
                if (p.gn_silu) {  // silu(y) = y * (0.5 + 0.5 tanh(y / 2))
                  __nv_bfloat162 hh = __hmul2(h, __floats2bfloat162_rn(0.5f, 0.5f));
                  uint32_t th, hv = *reinterpret_cast<uint32_t*>(&hh);
                  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(th) : "r"(hv));
                  const __nv_bfloat162 sg = __hfma2(*reinterpret_cast<__nv_bfloat162*>(&th),
                                                    __floats2bfloat162_rn(0.5f, 0.5f), __floats2bfloat162_rn(0.5f, 0.5f));
                  h = __hmul2(h, sg);
                }
                w[e] = *reinterpret_cast<uint32_t*>(&h);
              } else {
                __half2 h = __floats2half2_rn(y0, y1);
                if (p.gn_silu) {
                  __half2 hh = __hmul2(h, __float2half2_rn(0.5f));
                  uint32_t th, hv = *reinterpret_cast<uint32_t*>(&hh);
                  asm("tanh.approx.f16x2 %0, %1;" : "=r"(th) : "r"(hv));
                  const __half2 sg = __hfma2(*reinterpret_cast<__half2*>(&th), __float2half2_rn(0.5f), __float2half2_rn(0.5f));
                  h = __hmul2(h, sg);
                }
                w[e] = *reinterpret_cast<uint32_t*>(&h);
              }
            }
            // padding rows (TMA zero fill) and rows past M keep their loaded zeros
            if (vld[i])
              *reinterpret_cast<uint4*>(tile + ((tt >> 3) + 32 * i) * 128 + pc * 16) = make_uint4(w[0], w[1], w[2], w[3]);
          }
#ifndef DI_XF_NOFENCE
          fence_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
#endif
          __syncwarp();
#ifdef DI_XF_CTA_ARRIVE
          if (lane == 0) mbar_arrive(&aready[s]);
#else
          if (lane == 0) mbar_arrive_cluster(aready_leader + s * 8);
#endif
          if (tr && lt == 0 && threadIdx.x == 64 && kb == kb0) tr[10] = globaltimer();
          if (tr && lt == 0 && threadIdx.x == 64 && kb == kb1 - 1) tr[11] = globaltimer();
        }
      }
      // Plain epilogue: the operands that do not depend on the accumulator are fetched one chunk ahead on all
      // 32 lanes (the first chunk's before the accumulator wait, i.e. during the main loop): lane j holds
      // column j's bias and row-vector values (broadcast later by full-warp shuffles), each lane its own
      // row's 32 residual values.  A chunk takes this path when it is whole and its 32 rows share one image.
      if (LN) {
        // LayerNorm statistics of this warp's 32 rows (one row per lane, all 64 columns of every K block)
        float sum = 0.f, sq = 0.f;
        for (int kb = kb0; kb < kb1; ++kb, ++lit) {
          const int s = lit % STAGES;
          const bool okl = mbar_wait(&full[s], (lit / STAGES) & 1, p.err, DEVERR_WAIT_EPI) && !*abort_flag;
          if (okl) {
            const uint4* rowp = reinterpret_cast<const uint4*>(sA + s * S::A_BYTES + row * 128);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 u = rowp[j];
              const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uint32_t we = w[e];
                float2 f;
                if (BF16) f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&we));
                else f = __half22float2(*reinterpret_cast<__half2*>(&we));
                sum += f.x + f.y;
                sq = fmaf(f.x, f.x, fmaf(f.y, f.y, sq));
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
        const float kk = (float)(p.num_k * BK);
        const float mean = sum / kk;
        const float var = fmaxf(sq / kk - mean * mean, 0.0f);
        ln_rs = 1.0f / sqrtf(var + p.ln_eps);
        ln_rm = ln_rs * mean;
      }
      float pf_b = 0.f, pf_r = 0.f, pf_c = 0.f;
      uint4 pf_res[4] = {};
      auto pf_fast = [&](int c) {
        return PLAIN && n0 + c * 32 + 32 <= p.N && (!p.rowvec || p.rowvec_div % 32 == 0);
      };
      auto pf_fetch = [&](int c) {
        const int nbc = n0 + c * 32;
        if (p.bias) pf_b = __ldg(p.bias + nbc + lane);
        if (LN) pf_c = __ldg(p.ln_c1 + nbc + lane);
        if (p.rowvec && m0 + q * 32 < p.M)
          pf_r = __ldg(p.rowvec + (size_t)((m0 + q * 32) / p.rowvec_div) * p.rowvec_ld + nbc + lane);
        if (p.residual && m < p.M) {
          const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.residual) + (size_t)m * p.ldr + nbc);
#pragma unroll
          for (int j = 0; j < 4; ++j) pf_res[j] = __ldg(src + j);
        }
      };
      if (PLAIN && pf_fast(half)) pf_fetch(half);
      const bool okw = mbar_wait<PAIR>(&tfull[ab], (lt >> 1) & 1, p.err, DEVERR_WAIT_EPI) && !*abort_flag;
      const bool ok = __all_sync(0xffffffffu, okw);
      if (tr && lt == 0 && threadIdx.x == 64) tr[5] = globaltimer();
      tc_fence_after();
      const uint32_t trow = tmem + ab * BN + (static_cast<uint32_t>(q * 32) << 16);
      const bool split = PARTIAL || (!PLAIN && !GEGLU && p.splits > 1);
      const bool gg = GEGLU || (!PLAIN && !PARTIAL && p.geglu && !split);  // split-K stores raw packed partials; the reduce applies GEGLU
      bool xok = true;  // cluster split-K exchange still in step with the peers
      const int nchunks = gg ? BN / 64 : BN / 32;
      const int n_out = gg ? p.N / 2 : p.N;
#pragma unroll 1
      for (int c = half; c < nchunks; c += kEpiWarps / 4) {
        float v[32];
        int nb;  // first output column of the chunk
        {
          uint32_t r[32];
          if (gg) {
            // each 128 accumulator columns hold 64 value rows then the matching 64 gate rows
            const int g = c >> 1, h = c & 1;
            uint32_t rg[32];
            tmem_ld32(trow + g * 128 + h * 32, r);
            tmem_ld32(trow + g * 128 + 64 + h * 32, rg);
            tmem_wait_ld();
            const int nv = n0 + g * 128 + h * 32;  // packed value column
            nb = (n0 + g * 128) / 2 + h * 32;
            if (nb < n_out) {
              // bias of value column nv + lane and gate column nv + 64 + lane, broadcast by full-warp shuffles
              // (nb is warp-uniform and no lane skips this block)
              const float bvl = p.bias ? __ldg(p.bias + nv + lane) : 0.f;
              const float bgl = p.bias ? __ldg(p.bias + nv + 64 + lane) : 0.f;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float a = __uint_as_float(r[j]), gt = __uint_as_float(rg[j]);
                if (LN) {
                  a = fmaf(ln_rs, a, -ln_rm * __ldg(p.ln_c1 + nv + j));
                  gt = fmaf(ln_rs, gt, -ln_rm * __ldg(p.ln_c1 + nv + 64 + j));
                }
                a += __shfl_sync(0xffffffffu, bvl, j);
                gt += __shfl_sync(0xffffffffu, bgl, j);
                v[j] = a * gelu_erf(gt);
              }
            }
          } else {
            if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[8] = globaltimer();
            const bool fastc = pf_fast(c);
            const float cb = pf_b, cr = pf_r, cc1 = pf_c;
            uint4 cres[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) cres[j] = pf_res[j];
            if (PLAIN && c + kEpiWarps / 4 < nchunks && pf_fast(c + kEpiWarps / 4)) pf_fetch(c + kEpiWarps / 4);
            tmem_ld32(trow + c * 32, r);
            tmem_wait_ld();
            if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[9] = globaltimer();
            nb = n0 + c * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (PLAIN && fastc) {  // warp-uniform: the shuffles run on all 32 lanes
              if (LN) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = fmaf(ln_rs, v[j], -ln_rm * __shfl_sync(0xffffffffu, cc1, j));
              }
              if (p.bias) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, cb, j);
              }
              if (p.rowvec) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, cr, j);
              }
              if (p.act == 1) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
              } else if (p.act == 2) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
              }
              if (p.residual) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t w[4] = {cres[j].x, cres[j].y, cres[j].z, cres[j].w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    uint32_t we = w[e];
                    float2 f;
                    if (BF16) f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&we));
                    else f = __half22float2(*reinterpret_cast<__half2*>(&we));
                    v[8 * j + 2 * e] += f.x;
                    v[8 * j + 2 * e + 1] += f.y;
                  }
                }
              }
            } else if (!split && nb < n_out && m < p.M && (PLAIN || !(p.dbg & 2))) {
              epi(v, nb, m);
            }
            if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[10] = globaltimer();
          }
        }
        if (MODE == 0 && p.gstats && !split && ok && nb < n_out) gn_stats_chunk(v, nb, m0 + q * 32, m, lane, p);
        if (!ok || nb >= n_out) continue;  // warp-uniform
        if (!split) {
          if (PLAIN || !(p.dbg & 1)) store_chunk(v, nb, m0, m, sp, false, staged);
          if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[11] = globaltimer();
          if (tr && lt == 0 && threadIdx.x == 64 && c == half + 2) tr[12] = globaltimer();
          continue;
        }
        if (CS) {
          if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[13] = globaltimer();
          if (xok) xok = cs_reduce(v, nb, m0, n_out);
          if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[14] = globaltimer();
          continue;
        }
        if (PARTIAL || !(p.dbg & 1)) store_chunk(v, nb, m0, m, sp, true, staged);  // fp32 partials: the reduce kernel finishes them
        if (tr && lt == 0 && threadIdx.x == 64 && c == half) tr[11] = globaltimer();
        if (tr && lt == 0 && threadIdx.x == 64 && c == half + 2) tr[12] = globaltimer();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // CTA-scope arrive unless the pair leader's barrier is remote
        if (PAIR) mbar_arrive_cluster(tempty_leader + ab * 8);
        else mbar_arrive(&tempty[ab]);
      }
      if (tr && lt == 0 && threadIdx.x == 64) tr[6] = globaltimer();
      if (!ok || !xok) break;
    }
    if (p.tma_out && lane == 0) bulk_wait0();  // every output store of this warp has completed
  }
  tc_fence_before();
  if (PAIR || CS) cluster_sync();  // no CTA leaves while a cluster peer may still read its slabs or signal it
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem, TMEM_COLS);
    else tmem_dealloc(tmem, TMEM_COLS);
  }
  if (tr && threadIdx.x == 0) tr[7] = globaltimer();
}

// Pairs of CTAs that can be resident at once (clusters of 2 need both SMs in one GPC), per device.
static int g_max_pairs[32] = {0};
// Cluster split-K: clusters of n = 2 .. kMaxClusterSplit CTAs that can be resident at once, per device.
constexpr int kMaxClusterSplit = 8;
static int g_max_clusters[32][kMaxClusterSplit + 1] = {};

static int max_clusters(Ctx* c, int n) {
  int& mc = g_max_clusters[c->device & 31][n];
  if (mc) return mc;
  using S = GemmSmem<128, 6, false>;
  auto kern = gemm_tc_kernel<128, 6, false, false, 0>;
  mc = std::max(1, c->num_sms / (2 * n));  // conservative if the query fails
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n * (c->num_sms / n));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = S::TOTAL;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int k = 0;
    if (cudaOccupancyMaxActiveClusters(&k, kern, &cfg) == cudaSuccess && k > 0) mc = std::min(k, c->num_sms / n);
  }
  cudaGetLastError();
  return mc;
}

template <int BN, int STAGES, bool BF16, bool PAIR, int XF>
int launch_variant(Ctx* c, const GemmParams& p) {
  using S = GemmSmem<BN, STAGES, PAIR>;
  auto kern = gemm_tc_kernel<BN, STAGES, BF16, PAIR, XF>;
  static unsigned attr_done = 0;  // per-device bit: dynamic smem opt-in is a per-device attribute
  if (!(attr_done & (1u << (c->device & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) != cudaSuccess)
      return set_error(c, DI_ECUDA, "gemm: cudaFuncSetAttribute failed");
    attr_done |= 1u << (c->device & 31);
  }
  const int units = p.m_tiles * p.n_tiles * p.splits;
  int grid;
  if (PAIR) {
    const int pairs = g_max_pairs[c->device & 31] > 0 ? g_max_pairs[c->device & 31] : c->num_sms / 2;
    grid = 2 * std::min(units, pairs);
  } else {
    grid = std::min(units, c->num_sms);
  }
  if (!PAIR && p.cs) {  // clusters of p.cs CTAs, one cluster per tile at a time
    const int per_split = p.m_tiles * p.n_tiles;
    grid = p.cs * std::min(per_split, max_clusters(c, p.cs));
  }
  GemmParams q = p;
  q.trace = (g_trace && grid <= g_trace_ctas) ? g_trace : nullptr;
  if (PAIR) launch_k_cluster(kern, grid, kGemmThreads, S::TOTAL, c->stream, 2, q);
  else if (p.cs) launch_k_cluster(kern, grid, kGemmThreads, S::TOTAL, c->stream, p.cs, q);
  else launch_k(kern, grid, kGemmThreads, S::TOTAL, c->stream, q);
  return check_launch(c, "gemm_tc_kernel");
}

// Queries (once per device) how many 2-CTA clusters of the paired kernel fit on the GPU at once.
static int max_pairs(Ctx* c) {
  int& mp = g_max_pairs[c->device & 31];
  if (mp) return mp;
  using S = GemmSmem<256, 6, true>;
  auto kern = gemm_tc_kernel<256, 6, false, true, 0>;
  mp = c->num_sms / 2;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * mp);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = S::TOTAL;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) mp = std::min(mp, n);
  }
  cudaGetLastError();
  return mp;
}

// Sums the split-K partials and applies the epilogue (bias, per-image row vector, residual or GEGLU).
__global__ void splitk_reduce(const float* __restrict__ part, int splits, int M, int N, const float* __restrict__ bias,
                              const float* __restrict__ rowvec, int rowvec_div, int rowvec_ld, const void* residual,
                              int ldr, int res_f32, void* out, int ldo, int out_f32, int geglu, int bf16, int act) {
  pdl_begin();

  const size_t slice = (size_t)M * N;
  const int NO = geglu ? N / 2 : N;
  if (!geglu && (N & 3) == 0 && (ldo & 3) == 0 && (!residual || (ldr & 3) == 0)) {
    // four columns per thread: float4 partial loads
    const size_t total4 = (size_t)M * N / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4; i += (size_t)gridDim.x * blockDim.x) {
      const int m = (int)((i * 4) / N), o = (int)((i * 4) % N);
      float4 v = reinterpret_cast<const float4*>(part)[i];
      for (int z = 1; z < splits; ++z) {
        const float4 w = reinterpret_cast<const float4*>(part + z * slice)[i];
        v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
      }
      float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (bias) f[j] += bias[o + j];
        if (rowvec) f[j] += rowvec[(size_t)(m / rowvec_div) * rowvec_ld + o + j];
        if (act) f[j] = act == 1 ? silu_f(f[j]) : gelu_erf(f[j]);
        if (residual) f[j] += load_one(residual, (size_t)m * ldr + o + j, res_f32, bf16);
        store_one(out, (size_t)m * ldo + o + j, f[j], out_f32, bf16);
      }
    }
    return;
  }
  const size_t total = (size_t)M * NO;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = i / NO, o = i % NO;
    if (!geglu) {
      float v = 0.f;
      for (int z = 0; z < splits; ++z) v += part[z * slice + (size_t)m * N + o];
      if (bias) v += bias[o];
      if (rowvec) v += rowvec[(size_t)(m / rowvec_div) * rowvec_ld + o];
      if (act) v = act == 1 ? silu_f(v) : gelu_erf(v);
      if (residual) v += load_one(residual, (size_t)m * ldr + o, res_f32, bf16);
      store_one(out, (size_t)m * ldo + o, v, out_f32, bf16);
    } else {
      const int nv = (o / 64) * 128 + (o % 64), ng = nv + 64;
      float a = 0.f, g = 0.f;
      for (int z = 0; z < splits; ++z) {
        a += part[z * slice + (size_t)m * N + nv];
        g += part[z * slice + (size_t)m * N + ng];
      }
      if (bias) { a += bias[nv]; g += bias[ng]; }
      store_one(out, (size_t)m * ldo + o, a * gelu_erf(g), out_f32, bf16);
    }
  }
}

// Split-K reduce of an fp16 output whose GroupNorm(32) statistics are wanted: grid (row blocks, images),
// N / 4 threads per block, thread t owns columns 4t .. 4t + 3 for every row of its block (coalesced float4
// partial loads), keeps its groups' fixed-point sums (gn_fixed) in registers, folds them through shared
// memory, and the block adds 32 x 3 int64 per image to the statistics.
__global__ void splitk_reduce_gn(const float* __restrict__ part, int splits, int M, int N, const float* __restrict__ bias,
                                 const float* __restrict__ rowvec, int rowvec_div, int rowvec_ld,
                                 const __half* __restrict__ residual, int ldr, __half* __restrict__ out, int ldo, int act,
                                 long long* __restrict__ gstats, int cpg, int hw) {
  pdl_begin();
  __shared__ long long acc[32 * 3];
  for (int i = threadIdx.x; i < 96; i += blockDim.x) acc[i] = 0;
  __syncthreads();
  const int n = blockIdx.y, rb = gridDim.x;
  const int rows = (hw + rb - 1) / rb;
  const int r0 = n * hw + blockIdx.x * rows, r1 = min(n * hw + hw, r0 + rows);
  const int o = threadIdx.x * 4;
  const size_t slice = (size_t)M * N;
  const int ga = o / cpg, gb = (o + 3) / cpg;
  long long s[2] = {0, 0}, hi[2] = {0, 0}, lo[2] = {0, 0};
#pragma unroll 4
  for (int m = r0; m < r1; ++m) {
    float4 v = reinterpret_cast<const float4*>(part + (size_t)m * N + o)[0];
    for (int z = 1; z < splits; ++z) {
      const float4 w = reinterpret_cast<const float4*>(part + z * slice + (size_t)m * N + o)[0];
      v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
    }
    float f[4] = {v.x, v.y, v.z, v.w};
    __half h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (bias) f[j] += bias[o + j];
      if (rowvec) f[j] += rowvec[(size_t)(m / rowvec_div) * rowvec_ld + o + j];
      if (act) f[j] = act == 1 ? silu_f(f[j]) : gelu_erf(f[j]);
      if (residual) f[j] += __half2float(residual[(size_t)m * ldr + o + j]);
      h[j] = __float2half_rn(f[j]);
      long long a, b, c;
      gn_fixed(__half2float(h[j]), a, b, c);
      const int k = (o + j) / cpg - ga;
      s[k] += a; hi[k] += b; lo[k] += c;
    }
    __half2* dst = reinterpret_cast<__half2*>(out + (size_t)m * ldo + o);
    dst[0] = __halves2half2(h[0], h[1]);
    dst[1] = __halves2half2(h[2], h[3]);
  }
  unsigned long long* sa = reinterpret_cast<unsigned long long*>(acc);
  atomicAdd(sa + ga * 3, (unsigned long long)s[0]);
  atomicAdd(sa + ga * 3 + 1, (unsigned long long)hi[0]);
  atomicAdd(sa + ga * 3 + 2, (unsigned long long)lo[0]);
  if (gb != ga) {
    atomicAdd(sa + gb * 3, (unsigned long long)s[1]);
    atomicAdd(sa + gb * 3 + 1, (unsigned long long)hi[1]);
    atomicAdd(sa + gb * 3 + 2, (unsigned long long)lo[1]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 96; i += blockDim.x)
    if (acc[i]) atomicAdd(reinterpret_cast<unsigned long long*>(gstats + (size_t)n * 96 + i), (unsigned long long)acc[i]);
}

}  // namespace

// Tiling: N tile width (128 / 160 / 192 / 256) and K splits from a cost model in units of one 128-wide
// K block of MMA work per SM: units = M tiles x N tiles x splits run on min(units, SMs) persistent CTAs;
// cost = rounds x (K blocks per unit x (128 + BN)/256 + per-unit overhead) + split-K reduce (partial-sum
// traffic and one launch).  GEGLU needs BN in {128, 256} (value/gate rows packed per 128 columns).
void choose_tiling(Ctx* c, int M, int N, int num_k, int geglu, int* bn, int* splits, int* pair, int* cs) {
  static const int cands[4] = {128, 160, 192, 256};
  const int mt = (M + BM - 1) / BM;
  *pair = 0;
  *cs = 0;
  // Cluster split-K (partials summed through distributed shared memory, no reduce launch): not for GEGLU
  // (value and gate columns sit in different chunks) nor with epilogue GroupNorm statistics.
  // Opt-in (DI_CLUSTER_SPLIT=1): measured slower than the reduce kernel in the U-Net step so far.
  static const int cs_ok = [] {
    const char* e = getenv("DI_CLUSTER_SPLIT");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  static const double cs_cost = [] {  // exchange cost per 32-column chunk round, in K-block units
    const char* e = getenv("DI_CLUSTER_SPLIT_COST");
    return e ? atof(e) : 1.0;
  }();
  const bool allow_cs = cs_ok && !geglu && !c->gn_stats;
  // Tuning / diagnostics override: DI_GEMM_TILING="bn,splits[,pair]" forces the tiling of every GEMM.
  static int forced_bn = -1, forced_s = 1, forced_pair = 0;
  if (forced_bn < 0) {
    forced_bn = 0;
    if (const char* e = getenv("DI_GEMM_TILING")) {
      int b = 0, s = 1, pr = 0;
      if (sscanf(e, "%d,%d,%d", &b, &s, &pr) >= 1 && (b == 128 || b == 160 || b == 192 || b == 256)) {
        forced_bn = b;
        forced_s = std::max(1, s);
        forced_pair = pr == 2 ? 2 : (pr ? 1 : 0);
      }
    }
  }
  if (forced_bn && !c->ln_c1 && (!geglu || forced_bn % 128 == 0)) {
    *bn = forced_bn;
    int fs = forced_s;
    // forced pair value 2 = cluster split-K instead of paired tiles
    const bool fcs = forced_pair == 2 && allow_cs;
    if (fcs) fs = std::min(fs, kMaxClusterSplit);
    while (!fcs && fs > 1 && (size_t)M * N * fs * 4 > kSplitKWsBytes) --fs;
    const int per = (num_k + fs - 1) / fs;
    *splits = (num_k + per - 1) / per;
    *pair = forced_pair == 1 && M > BM;
    *cs = (fcs && *splits > 1) ? *splits : 0;
    return;
  }
  // Model in units of one BN=128 K block on one CTA (~0.3 us, measured with the per-CTA trace).  A K
  // block of the main loop costs nearly the same for any tile width: 1.0 at BN=128, +20% at BN=256 for
  // one CTA and +5% for a pair, whose tile has twice the rows; so wide and paired tiles do more work
  // per unit of time, narrow and split tiles fill more SMs.  A tile adds ~8 for its first load and the
  // epilogue; split-K adds the reduce launch and the fp32 partial traffic; a wave holds min(SMs,
  // resident pairs) units.
  const int pairs = max_pairs(c);
  static const int pair_ok = [] {  // diagnostics: DI_GEMM_PAIR=0 disables paired-CTA tiles
    const char* e = getenv("DI_GEMM_PAIR");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  static const double split_cost = [] {  // the reduce launch, in K-block units; DI_SPLIT_COST overrides
    const char* e = getenv("DI_SPLIT_COST");
    return e ? atof(e) : 9.0;
  }();
  double best = 1e30;
  *bn = 128;
  *splits = 1;
  const bool single = c->ln_c1 != nullptr;  // folded LayerNorm: whole K per CTA, no CTA pairs
  for (int pr = 0; pr < 2; ++pr) {
    if (pr && (M <= BM || !pair_ok || single)) continue;
    const int mtiles = pr ? (M + 2 * BM - 1) / (2 * BM) : mt;
    const int slots = pr ? pairs : c->num_sms;  // concurrently running units
    for (int bc : cands) {
      if (geglu && (bc % 128 || N % bc)) continue;
      const int nt = geglu ? N / bc : (N + bc - 1) / bc;
      const int smax = single ? 1 : std::max(1, std::min(16, num_k / 4));
      const double kb_cost = 1.0 + (pr ? 0.05 : 0.2) * (bc - 128) / 128.0;
      for (int s = 1; s <= smax; ++s) {
        const int per = (num_k + s - 1) / s;
        const int seff = (num_k + per - 1) / per;
        if (seff != s) continue;
        // global partials must fit the buffer (a cluster split needs none)
        const bool fits = s == 1 || (size_t)M * N * s * 4 <= kSplitKWsBytes;
        if (!fits && !(allow_cs && !pr && s <= kMaxClusterSplit)) break;
        // a folded LayerNorm keeps one tile per CTA (its statistics readers would hold the ring otherwise)
        if (single && (long long)mtiles * (geglu ? N / bc : (N + bc - 1) / bc) > slots) continue;
        const long long units = (long long)mtiles * nt * s;
        const long long rounds = (units + slots - 1) / slots;
        double cost = (double)rounds * (per * kb_cost + 8.0) + 4.0;
        if (s > 1) cost += split_cost + (double)M * N * s * 8.0 / 6.4e12 / 290e-9;
        if (!fits) cost = 1e30;
        if (cost < best - 1e-9 || (cost < best + 1e-9 && bc > *bn)) {
          best = cost;
          *bn = bc;
          *splits = s;
          *pair = pr;
          *cs = 0;
        }
        // the same split as a cluster split-K: one tile per cluster at a time, partials exchanged on chip
        if (!pr && s > 1 && s <= kMaxClusterSplit && allow_cs) {
          const int ncl = max_clusters(c, s);
          const long long tiles = (long long)mtiles * nt;
          const long long crounds = (tiles + ncl - 1) / ncl;
          const double ccost = (double)crounds * (per * kb_cost + 8.0 + cs_cost * (bc / 64.0)) + 4.0;
          if (ccost < best - 1e-9 || (ccost < best + 1e-9 && bc > *bn)) {
            best = ccost;
            *bn = bc;
            *splits = s;
            *pair = 0;
            *cs = s;
          }
        }
      }
    }
  }
}

int gemm_kernel_count(Ctx* c, int M, int N, int K, int geglu) {
  int bn, s, pr, cs;
  choose_tiling(c, M, N, K / 64, geglu, &bn, &s, &pr, &cs);
  return (s > 1 && !cs) ? 2 : 1;
}

template <int XF>
static int dispatch_xf(Ctx* c, const GemmParams& p, int bn, bool bf16, bool pair) {
  if (pair) {
    switch (bn) {
      case 256: return bf16 ? launch_variant<256, 6, true, true, XF>(c, p) : launch_variant<256, 6, false, true, XF>(c, p);
      case 192: return bf16 ? launch_variant<192, 6, true, true, XF>(c, p) : launch_variant<192, 6, false, true, XF>(c, p);
      case 160: return bf16 ? launch_variant<160, 7, true, true, XF>(c, p) : launch_variant<160, 7, false, true, XF>(c, p);
      default: return bf16 ? launch_variant<128, 8, true, true, XF>(c, p) : launch_variant<128, 8, false, true, XF>(c, p);
    }
  }
  switch (bn) {
    case 256: return bf16 ? launch_variant<256, 4, true, false, XF>(c, p) : launch_variant<256, 4, false, false, XF>(c, p);
    case 192: return bf16 ? launch_variant<192, 4, true, false, XF>(c, p) : launch_variant<192, 4, false, false, XF>(c, p);
    case 160: return bf16 ? launch_variant<160, 5, true, false, XF>(c, p) : launch_variant<160, 5, false, false, XF>(c, p);
    default: return bf16 ? launch_variant<128, 6, true, false, XF>(c, p) : launch_variant<128, 6, false, false, XF>(c, p);
  }
}

static int dispatch_variant(Ctx* c, const GemmParams& p, int bn, bool bf16, bool pair) {
  if (p.gn_tab) return dispatch_xf<1>(c, p, bn, bf16, pair);
  const bool plain = !p.geglu && p.splits <= 1 && !p.gstats && !p.out_f32 && !p.res_f32 && p.staged && !p.cs &&
                     !p.dbg && !g_gemm_generic;
  const bool partial = p.splits > 1 && !p.cs && !p.gstats && !p.dbg && !g_gemm_generic;  // GEGLU packs raw partials too
  if (partial) return dispatch_xf<3>(c, p, bn, bf16, pair);
  if (p.geglu && p.splits <= 1 && !p.out_f32 && !p.dbg && !g_gemm_generic) return dispatch_xf<4>(c, p, bn, bf16, pair);
  if (p.ln && !plain) return set_error(c, DI_EINVAL, "gemm: a folded LayerNorm needs the plain or GEGLU epilogue");
  return plain ? dispatch_xf<2>(c, p, bn, bf16, pair) : dispatch_xf<0>(c, p, bn, bf16, pair);
}

int launch_gemm(Ctx* c, GemmParams& p, bool bf16, int bn, int splits, int pair, int cs, void* splitk_ws) {
  p.err = c->d_err;
  p.gstats = nullptr;
  if (c->gn_stats) {
    if (bf16 || p.out_f32 || p.geglu || p.N % 32 || p.N < 256 || p.N > 4096 || c->gn_stats_hw <= 0 || c->gn_stats_hw % 32 ||
        p.M % c->gn_stats_hw || (p.residual && p.res_f32))
      return set_error(c, DI_EINVAL, "gemm: GroupNorm statistics need fp16 output, N % 32 == 0, whole images");
    p.gstats = c->gn_stats;
    p.g_cpg = p.N / 32;
    p.g_hw = c->gn_stats_hw;
  }
  p.staged = (p.vec_ok && splits <= 1) ? 1 : 0;
  p.ln = 0;
  if (c->ln_c1) {
    if (splits > 1 || pair || p.out_f32 || !p.staged || p.gn_tab || p.gstats || !p.bias)
      return set_error(c, DI_EINVAL, "gemm: a folded LayerNorm needs one unsplit single-CTA tile, 16-bit aligned output");
    p.ln = 1;
    p.ln_c1 = c->ln_c1;
    p.ln_eps = c->ln_eps;
  }
  p.b_early = c->weights_const ? 1 : 0;
  static const int dbg = [] {
    const char* e = getenv("DI_GEMM_DEBUG");
    return e ? atoi(e) : 0;
  }();
  p.dbg = dbg;
  if (dbg & 4) p.staged = 0;
  p.splits = std::max(1, splits);
  p.m_tiles = pair ? (p.M + 2 * BM - 1) / (2 * BM) : (p.M + BM - 1) / BM;
  p.n_tiles = p.geglu ? p.N / bn : (p.N + bn - 1) / bn;
  p.cs = 0;
  if (p.splits > 1 && cs && !pair && !p.geglu && !p.gstats && !p.gn_tab && p.splits <= kMaxClusterSplit) {
    p.cs = p.splits;  // partials summed on chip by the cluster, epilogue in the same kernel
    p.staged = 0;
    return dispatch_variant(c, p, bn, bf16, false);
  }
  if (p.splits > 1) {
    const size_t need = sizeof(float) * (size_t)p.splits * p.M * p.N;
    if (need > kSplitKWsBytes) return set_error(c, DI_EINVAL, "gemm: split-K partials exceed the workspace");
    p.partial = static_cast<float*>(splitk_ws ? splitk_ws : workspace(c, need, 4));
    if (!p.partial) return set_error(c, DI_ENOMEM, "gemm: split-K workspace");
    p.staged = (p.N % 4 == 0 && reinterpret_cast<uintptr_t>(p.partial) % 16 == 0) ? 1 : 0;
    int r = dispatch_variant(c, p, bn, bf16, pair);
    if (r) return r;
    if (p.gstats) {
      // N / 4 <= 1024 threads; row blocks so that the grid covers the SMs about twice
      const int imgs = p.M / p.g_hw;
      const int rb = std::max(1, std::min(p.g_hw, (2 * c->num_sms + imgs - 1) / imgs));
      launch_k(splitk_reduce_gn, dim3(rb, imgs), p.N / 4, 0, c->stream, p.partial, p.splits, p.M, p.N, p.bias,
               p.rowvec, p.rowvec_div, p.rowvec_ld, static_cast<const __half*>(p.residual), p.ldr,
               static_cast<__half*>(p.out), p.ldo, p.act, p.gstats, p.g_cpg, p.g_hw);
      return check_launch(c, "splitk_reduce_gn");
    }
    const size_t total = (size_t)p.M * (p.geglu ? p.N / 2 : p.N);
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)8 * c->num_sms);
    launch_k(splitk_reduce, blocks, 256, 0, c->stream, p.partial, p.splits, p.M, p.N, p.bias, p.rowvec, p.rowvec_div,
             p.rowvec_ld, p.residual, p.ldr, p.res_f32, p.out, p.ldo, p.out_f32, p.geglu, bf16, p.act);
    return check_launch(c, "splitk_reduce");
  }
  // 16-bit output rows 16-byte aligned: the epilogue stores its 32 x 32 chunks with TMA
  p.tma_out = 0;
  if (!p.out_f32 && p.staged && p.splits <= 1 && !p.cs && !p.gstats && !p.dbg && !p.gn_tab && !g_gemm_generic) {
    const uint64_t dims[2] = {(uint64_t)(p.geglu ? p.N / 2 : p.N), (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.ldo * 2};
    const uint32_t box[2] = {32, 32};
    std::string err;
    p.tma_out = make_tmap(&p.tmO, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.out,
                          dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B, &err) ? 1 : 0;
  }
  return dispatch_variant(c, p, bn, bf16, pair);
}

static CUtensorMapDataType tdt(int dtype) {
  return dtype == DI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// 2-D K-major operand map: rows x cols(K), row stride ld elements, box 64 x box_rows.
bool tmap_kmajor(CUtensorMap* m, int dtype, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows, std::string* err) {
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {ld * 2};
  uint32_t box[2] = {64, box_rows};
  return make_tmap(m, tdt(dtype), 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, err);
}

// Conv tile geometry: 128 output pixels = bn images x bh rows x Wo columns.
// Rows wider than 128 pixels (multiples of 128) are cut into 128-pixel tiles: box {64, 128, 1, 1}.
static uint32_t conv_box_w(int Wo) { return (uint32_t)std::min(Wo, 128); }
static bool conv_box(int Ho, int Wo, uint32_t* bh, uint32_t* bn) {
  if (Wo > 128 && Wo % 128 == 0) {
    *bh = 1;
    *bn = 1;
    return true;
  }
  if (Wo <= 0 || Wo > 128 || (128 % Wo) != 0) return false;
  const int rows = std::min(Ho, 128 / Wo);
  if ((128 / Wo) % rows != 0) return false;
  if (Ho % rows != 0) return false;
  *bh = rows;
  *bn = 128 / (Wo * rows);
  return true;
}

static bool tmap_conv_s1(CUtensorMap* m, int dtype, const void* base, int N, int H, int W, int C, uint32_t bh,
                         uint32_t bn, std::string* err) {
  uint64_t dims[4] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)N};
  uint64_t strides[3] = {(uint64_t)C * 2, (uint64_t)W * C * 2, (uint64_t)H * W * C * 2};
  uint32_t box[4] = {64, conv_box_w(W), bh, bn};
  return make_tmap(m, tdt(dtype), 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, err);
}

static bool tmap_conv_s2(CUtensorMap* m, int dtype, const void* base, int N, int H, int W, int C, int py, int px,
                         uint32_t bh, uint32_t bn, std::string* err) {
  const uint16_t* b = static_cast<const uint16_t*>(base) + ((size_t)py * W + px) * C;
  uint64_t dims[4] = {(uint64_t)C, (uint64_t)(W / 2), (uint64_t)(H / 2), (uint64_t)N};
  uint64_t strides[3] = {(uint64_t)C * 4, (uint64_t)W * C * 4, (uint64_t)H * W * C * 2};
  uint32_t box[4] = {64, conv_box_w(W / 2), bh, bn};
  return make_tmap(m, tdt(dtype), 4, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, err);
}

static bool vec_rows_ok(const void* p, int ld, int esz) {
  return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && ((size_t)ld * esz) % 16 == 0;
}

static GemmParams base_params() {
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.rowvec_div = 1;
  p.splits = 1;
  return p;
}

// Public building blocks used by the fused blocks and the U-Net plan ---------------------------
int gemm_linear(Ctx* c, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
                const float* bias, const void* R, int res_f32, void* Y, int out_f32, int geglu, const float* rowvec,
                int rowvec_div, void* splitk_ws, const GnFuse* gnf, int gnf_hw, int act) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 64 || (X2 && (K1 <= 0 || K1 % 64 || K1 >= K)))
    return set_error(c, DI_EINVAL, "linear: K and K1 must be multiples of 64");
  if (geglu && (N % 128)) return set_error(c, DI_EINVAL, "linear_geglu: F must be a multiple of 64");
  GemmParams p = base_params();
  std::string err;
  const int ks = X2 ? K1 : K;
  if (!tmap_kmajor(&p.tmA[0], dtype, X1, M, ks, ks, 128, &err)) return set_error(c, DI_EINVAL, err);
  if (X2) {
    if (!tmap_kmajor(&p.tmA[1], dtype, X2, M, K - K1, K - K1, 128, &err)) return set_error(c, DI_EINVAL, err);
  } else {
    p.tmA[1] = p.tmA[0];
  }
  p.tmA[2] = p.tmA[0];
  p.tmA[3] = p.tmA[0];
  const int bn = geglu ? 128 : 0;
  p.mode = 0;
  p.M = M;
  p.N = N;
  p.num_k = K / 64;
  p.k_split = ks / 64;
  p.bias = bias;
  p.rowvec = rowvec;
  p.rowvec_div = rowvec_div > 0 ? rowvec_div : 1;
  p.rowvec_ld = N;
  p.residual = R;
  p.ldr = N;
  p.res_f32 = res_f32;
  p.out = Y;
  p.ldo = geglu ? N / 2 : N;
  p.out_f32 = out_f32;
  p.geglu = geglu;
  p.act = geglu ? 0 : act;
  p.vec_ok = vec_rows_ok(Y, p.ldo, out_f32 ? 4 : 2) && (!R || vec_rows_ok(R, N, res_f32 ? 4 : 2));
  (void)bn;
  if (gnf && gnf->tab) {  // rows are pixels of images of gnf_hw pixels (GnFuse on a 1x1 projection)
    if (gnf_hw <= 0) return set_error(c, DI_EINVAL, "linear: fused GroupNorm needs the pixels per image");
    p.gn_tab = gnf->tab;
    p.gn_silu = gnf->silu;
    p.gn_C = K;
    p.gn_HW = gnf_hw;
  }
  int chosen, splits;
  int pair, cs;
  choose_tiling(c, M, N, p.num_k, geglu, &chosen, &splits, &pair, &cs);
  if (!tmap_kmajor(&p.tmB, dtype, W, N, K, K, pair ? chosen / 2 : chosen, &err)) return set_error(c, DI_EINVAL, err);
  return launch_gemm(c, p, dtype == DI_BF16, chosen, splits, pair, cs, splitk_ws);
}

int gemm_conv3x3(Ctx* c, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W, int stride,
                 const void* Wt, int Co, const float* bias, const float* temb, const void* residual, int res_f32,
                 void* y, int out_f32, int temb_ld, void* splitk_ws, const GnFuse* gnf, int act) {
  if (C1 <= 0 || C1 % 64 || (x2 && (C2 <= 0 || C2 % 64)) || Co % 16 || (stride != 1 && stride != 2))
    return set_error(c, DI_EINVAL, "conv3x3: channels must be multiples of 64 (Co of 16), stride 1 or 2");
  if (stride == 2 && (x2 || (H % 2) || (W % 2)))
    return set_error(c, DI_EUNSUPPORTED, "conv3x3 stride 2: single input with even H, W");
  const int Ho = stride == 1 ? H : H / 2, Wo = stride == 1 ? W : W / 2;
  uint32_t bh, bn;
  if (!conv_box(Ho, Wo, &bh, &bn)) return set_error(c, DI_EUNSUPPORTED, "conv3x3: output tile geometry");
  GemmParams p = base_params();
  std::string err;
  const int Cin = C1 + (x2 ? C2 : 0);
  if (stride == 1) {
    if (!tmap_conv_s1(&p.tmA[0], dtype, x1, N, H, W, C1, bh, bn, &err)) return set_error(c, DI_EINVAL, err);
    if (x2) {
      if (!tmap_conv_s1(&p.tmA[1], dtype, x2, N, H, W, C2, bh, bn, &err)) return set_error(c, DI_EINVAL, err);
    } else p.tmA[1] = p.tmA[0];
    p.tmA[2] = p.tmA[0];
    p.tmA[3] = p.tmA[0];
    p.mode = 1;
  } else {
    for (int py = 0; py < 2; ++py)
      for (int px = 0; px < 2; ++px)
        if (!tmap_conv_s2(&p.tmA[py * 2 + px], dtype, x1, N, H, W, C1, py, px, bh, bn, &err))
          return set_error(c, DI_EINVAL, err);
    p.mode = 2;
  }
  p.M = N * Ho * Wo;
  p.N = Co;
  p.cin_blocks = Cin / 64;
  p.k_split = C1 / 64;
  p.num_k = 9 * p.cin_blocks;
  p.HWo = Ho * Wo;
  p.Wo = Wo;
  p.bias = bias;
  p.rowvec = temb;
  p.rowvec_div = Ho * Wo;
  p.rowvec_ld = temb_ld > 0 ? temb_ld : Co;
  p.residual = residual;
  p.ldr = Co;
  p.res_f32 = res_f32;
  p.out = y;
  p.ldo = Co;
  p.out_f32 = out_f32;
  p.vec_ok = vec_rows_ok(y, Co, out_f32 ? 4 : 2) && (!residual || vec_rows_ok(residual, Co, res_f32 ? 4 : 2));
  p.act = act;
  if (gnf && gnf->tab) {
    if (stride != 1) return set_error(c, DI_EUNSUPPORTED, "conv3x3: fused GroupNorm needs stride 1");
    p.gn_tab = gnf->tab;
    p.gn_silu = gnf->silu;
    p.gn_C = Cin;
    p.gn_HW = H * W;
    p.conv_bh = (int)bh;
  }
  int chosen, splits;
  int pair, cs;
  choose_tiling(c, p.M, Co, p.num_k, 0, &chosen, &splits, &pair, &cs);
  if (!tmap_kmajor(&p.tmB, dtype, Wt, Co, 9 * Cin, 9 * Cin, pair ? chosen / 2 : chosen, &err))
    return set_error(c, DI_EINVAL, err);
  if (p.gn_tab) cs = 0;  // the fused-GroupNorm transform keeps its table in the epilogue slabs
  return launch_gemm(c, p, dtype == DI_BF16, chosen, splits, pair, cs, splitk_ws);
}

// Weight repack: [Co][Ci][3][3] fp32 -> [Co][3][3][Ci] fp16/bf16.
__global__ void pack_conv3x3_kernel(const float* __restrict__ w, int Co, int Ci, void* out, int bf16) {
  pdl_begin();
  const size_t n = (size_t)Co * Ci * 9;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int ci = i % Ci;
    const int tap = (i / Ci) % 9;
    const int co = i / ((size_t)Ci * 9);
    const float v = w[((size_t)co * Ci + ci) * 9 + tap];
    if (bf16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else static_cast<__half*>(out)[i] = __float2half_rn(v);
  }
}

int pack_conv3x3(Ctx* c, int dtype, const float* w, int Co, int Ci, void* out) {
  launch_k(pack_conv3x3_kernel, std::min<size_t>(((size_t)Co * Ci * 9 + 255) / 256, 4096), 256, 0, c->stream, 
      w, Co, Ci, out, dtype == DI_BF16);
  return check_launch(c, "pack_conv3x3");
}

}  // namespace di

using namespace di;

extern "C" {

int di_debug_gemm_trace(unsigned long long* buf, int ctas) {
  if (ctas < 0 || (ctas > 0 && !buf)) return DI_EINVAL;
  g_trace = ctas ? buf : nullptr;
  g_trace_ctas = ctas;
  return DI_OK;
}

int di_linear(di_ctx_t h, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
              const float* bias, const void* R, void* Y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  return gemm_linear(c, dtype, X1, K1, X2, M, K, W, N, bias, R, 0, Y, 0, 0, nullptr, 1, nullptr, nullptr, 0, 0);
}

int di_linear_act(di_ctx_t h, int dtype, const void* X, int M, int K, const void* W, int N, const float* bias,
                  const void* R, int act, void* Y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16) || act < 0 || act > 2) return DI_EINVAL;
  return gemm_linear(c, dtype, X, K, nullptr, M, K, W, N, bias, R, 0, Y, 0, 0, nullptr, 1, nullptr, nullptr, 0, act);
}

int di_linear_geglu(di_ctx_t h, int dtype, const void* X, int M, int K, const void* W, int F, const float* bias,
                    void* Y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16) || F % 64) return DI_EINVAL;
  return gemm_linear(c, dtype, X, K, nullptr, M, K, W, 2 * F, bias, nullptr, 0, Y, 0, 1, nullptr, 1, nullptr, nullptr,
                     0, 0);
}

int di_conv3x3_nhwc(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W,
                    int stride, const void* Wt, int Co, const float* bias, const float* temb, const void* residual,
                    void* y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  return gemm_conv3x3(c, dtype, x1, C1, x2, C2, N, H, W, stride, Wt, Co, bias, temb, residual, 0, y, 0, Co, nullptr,
                      nullptr, 0);
}

int di_conv3x3_nhwc_act(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W,
                        int stride, const void* Wt, int Co, const float* bias, const float* temb,
                        const void* residual, int act, void* y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16) || act < 0 || act > 1) return DI_EINVAL;
  return gemm_conv3x3(c, dtype, x1, C1, x2, C2, N, H, W, stride, Wt, Co, bias, temb, residual, 0, y, 0, Co, nullptr,
                      nullptr, act);
}

int di_conv3x3_nhwc_gn(di_ctx_t h, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W,
                       const void* Wt, int Co, const float* bias, const float* temb, const void* residual,
                       const float* gn_table, int silu, void* y) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16) || !gn_table) return DI_EINVAL;
  const GnFuse f{reinterpret_cast<const float2*>(gn_table), silu ? 1 : 0};
  return gemm_conv3x3(c, dtype, x1, C1, x2, C2, N, H, W, 1, Wt, Co, bias, temb, residual, 0, y, 0, Co, nullptr, &f, 0);
}

int di_pack_conv3x3(di_ctx_t h, int dtype, const float* w, int Co, int Ci, void* out) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  return pack_conv3x3(c, dtype, w, Co, Ci, out);
}

}  // extern "C"
