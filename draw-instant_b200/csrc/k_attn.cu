// k_attn.cu — flash attention, head dim 64, on tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's per-query-row workgroups (WGSL_FUSED_ATTN fused-attn.js:199-307, which
// re-reads all of K for every query row and holds a full score row in workgroup memory, and the
// cross-attention kernel fused-cross-attn.js:112-173 with its single-thread softmax) by a tiled,
// online-softmax kernel: one CTA per (128 queries, head, image), keys in tiles of 64.
//
//   warp 0      TMA: Q tile once, then K/V tiles of 64 keys into a 3-stage ring
//   warp 1      MMA: S_j = Q K_j^T (M=128, N=64, K=64) into a double-buffered TMEM tile, so the product
//               for tile j+1 runs while the softmax warps work on tile j; then O += P_j V_j
//               (M=128, N=64, K=64) with O resident in TMEM for the whole row block
//   warps 2..5  softmax, one query row per thread (= one TMEM lane): running max / sum in the exp2
//               domain, P written to shared memory as fp16/bf16 in the 128B-swizzled K-major layout the
//               MMA reads (two P buffers, so P_{j+1} is written while P_j.V_j runs); finally O / l.
//
// Softmax cost, which bounds this kernel rather than the tensor pipe:
//   * lazy rescaling: the running max used for the exponentials only moves when a row's true max
//     exceeds it by more than 8 (log2 units), so O in TMEM is rescaled rarely; P then stays <= 2^8,
//     well inside fp16 / bf16 range, and l uses the same stale max, so O / l is exact;
//   * the softmax warps' instruction issue, not the MUFU unit, is the limit: the max runs on raw
//     scores with 3-input max, the scale and max subtraction are one packed f32x2 FMA per two scores,
//     the row sum is packed f32x2 adds, and key masking runs only on the last, partial tile.
//
// Footprint: ~97 KB shared memory and 256 TMEM columns (S0 [0,64), S1 [64,128), O [128,192)), so two
// CTAs share an SM: one CTA's softmax overlaps the other's tensor-core work, and the U-Net's
// 160-CTA attention grids are resident in a single wave.
// Scores are scaled by 1/sqrt(64) as in the reference.  Keys past Skv (the zero-filled tail of the last
// TMA box) are masked to -inf.  All waits are time-bounded; no multicast loads.
#include <algorithm>

#include "di_common.cuh"

namespace di {

struct AttnParams {
  CUtensorMap tmQ, tmK, tmV;
  void* out;
  long long o_sb, o_ss, o_sh;  // output strides in elements (image, token, head)
  int Sq, Skv, H;
  int layout;                  // 0: dims {64, H, S, B}; 1: dims {64, S, H, B}
  int causal;                  // 1: query i attends to keys 0..i only (CLIP text encoder)
  float scale_log2;            // (1/sqrt(d)) * log2(e)
  int* err;
};

namespace {

constexpr int QT = 128, KT = 64, HD = 64, KV_STAGES = 3;
constexpr uint32_t Q_BYTES = QT * HD * 2;   // 16 KB
constexpr uint32_t KV_BYTES = KT * HD * 2;  // 8 KB per K or V tile
constexpr uint32_t P_BYTES = QT * KT * 2;   // 16 KB
constexpr uint32_t SMEM_ATTN = 1024 + Q_BYTES + 2 * KV_STAGES * KV_BYTES + 2 * P_BYTES + 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Packed two-lane fp32 arithmetic (sm_100): halves the FMA / FADD instruction count of the softmax.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float ex2_approx(float x) {  // MUFU 2^x; -inf -> +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__global__ void __launch_bounds__(192, 2) attn_fwd_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;               // KV_STAGES tiles
  uint8_t* sV = sK + KV_STAGES * KV_BYTES;  // KV_STAGES tiles
  uint8_t* sP = sV + KV_STAGES * KV_BYTES;  // [2] x (128 x 64), 128B-swizzled K-major blocks
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                // [KV_STAGES]
  uint64_t* kv_empty = kv_full + KV_STAGES;    // [KV_STAGES]
  uint64_t* s_full = kv_empty + KV_STAGES;     // [2]
  uint64_t* p_full = s_full + 2;               // [2] P_j written (buffer j & 1)
  uint64_t* pv_done = p_full + 2;              // [2] P_j.V_j complete (buffer j & 1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  // causal: the CTA's last query row q0 + QT - 1 sees keys up to that index only
  const int nt = (min(p.Skv, p.causal ? q0 + QT : p.Skv) + KT - 1) / KT;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_begin();  // set-up above touches no global memory
  const uint32_t tS0 = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&p.tmQ);
      tma_prefetch_desc(&p.tmK);
      tma_prefetch_desc(&p.tmV);
      const int c1q = p.layout == 0 ? h : q0, c2q = p.layout == 0 ? q0 : h;
      mbar_arrive_expect_tx(q_full, Q_BYTES);
      tma_load_4d(sQ, &p.tmQ, q_full, 0, c1q, c2q, b);
      for (int j = 0; j < nt; ++j) {
        const int st = j % KV_STAGES;
        if (*abort_flag || !mbar_wait(&kv_empty[st], ((j / KV_STAGES) & 1) ^ 1, p.err, DEVERR_WAIT_TMA)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
        const int k0 = j * KT;
        const int c1 = p.layout == 0 ? h : k0, c2 = p.layout == 0 ? k0 : h;
        tma_load_4d(sK + st * KV_BYTES, &p.tmK, &kv_full[st], 0, c1, c2, b);
        tma_load_4d(sV + st * KV_BYTES, &p.tmV, &kv_full[st], 0, c1, c2, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_f16(128, KT, BF16);
      constexpr uint32_t idO = idesc_f16(128, HD, BF16, false, true);  // B = V is MN-major (d contiguous)
      const uint32_t aQ = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.err, DEVERR_WAIT_MMA);
      auto issue_pv = [&](int jj) {
        const int st = jj % KV_STAGES;
        const uint32_t aV = smem_u32(sV + st * KV_BYTES);
        const uint32_t aP = smem_u32(sP + (jj & 1) * P_BYTES);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(aP + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(aV + kk * 2048, 8192, 1024);
          umma_f16(tO, ad, bd, idO, (jj | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&pv_done[jj & 1]);
        umma_commit(&kv_empty[st]);
      };
      for (int j = 0; ok && j < nt; ++j) {
        const int st = j % KV_STAGES;
        if (*abort_flag || !mbar_wait(&kv_full[st], (j / KV_STAGES) & 1, p.err, DEVERR_WAIT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(aQ + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(aK + kk * 32, 16, 1024);
          umma_f16(tS0 + (j & 1) * KT, ad, bd, idS, kk != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        if (j > 0) {
          if (!mbar_wait(&p_full[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, DEVERR_WAIT_MMA)) { ok = false; break; }
          tc_fence_after();
          issue_pv(j - 1);
        }
      }
      if (ok && mbar_wait(&p_full[(nt - 1) & 1], ((nt - 1) >> 1) & 1, p.err, DEVERR_WAIT_MMA)) {
        tc_fence_after();
        issue_pv(nt - 1);
      } else {
        *abort_flag = 1;
        umma_commit(&pv_done[0]);  // release the softmax warps promptly
        umma_commit(&pv_done[1]);
      }
    }
  } else {
    // ---------------- softmax warps ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int sb = j & 1;
      ok = ok && mbar_wait(&s_full[sb], (j >> 1) & 1, p.err, DEVERR_WAIT_SOFTMAX);
      tc_fence_after();
      float s[KT];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < KT / 32; ++c) {
          tmem_ld32(tS0 + sb * KT + lane_off + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      int kvalid = p.Skv - j * KT;
      if (p.causal) kvalid = min(kvalid, q0 + row + 1 - j * KT);  // key index <= query index
      if (kvalid < KT) {
#pragma unroll
        for (int i = 0; i < KT; ++i)
          if (i >= kvalid) s[i] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < KT; i += 2) mx = max3f(mx, s[i], s[i + 1]);
      mx *= p.scale_log2;  // the scale is positive: max of the scaled scores
      // lazy rescale: move the reference max only when the row max exceeds it by the threshold
      const bool move = mx > m_run + kRescaleThreshold;
      const float m_new = move ? mx : m_run;
      const float alpha = move ? ex2_approx(m_run - m_new) : 1.0f;
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nm2 = f2_pack(-m_new, -m_new);
      uint64_t acc2 = 0;
#pragma unroll
      for (int i = 0; i < KT; i += 2) {
        const uint64_t x = fma2(f2_pack(s[i], s[i + 1]), sc2, nm2);
        s[i] = ex2_approx(lo_f(x));
        s[i + 1] = ex2_approx(hi_f(x));
        acc2 = add2(acc2, f2_pack(s[i], s[i + 1]));
      }
      const float sum = lo_f(acc2) + hi_f(acc2);
      l_run = l_run * alpha + sum;
      m_run = m_new;
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // O is rescaled only after P_{j-1}.V_{j-1} has landed in it
        ok = ok && mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, DEVERR_WAIT_SOFTMAX);
        tc_fence_after();
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tO + lane_off + c * 32, r);
        }
        tmem_wait_st();
      }
      if (j > 1) {
        // P buffer j & 1 is free once P_{j-2}.V_{j-2} has completed
        ok = ok && mbar_wait(&pv_done[sb], ((j - 2) >> 1) & 1, p.err, DEVERR_WAIT_SOFTMAX);
      }
      // P row -> shared memory, 128B swizzle: 16-byte chunk c of row r lands at chunk c ^ (r % 8).
      uint8_t* prow = sP + sb * P_BYTES + row * 128;
#pragma unroll
      for (int c = 0; c < KT / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = s[c * 8 + 2 * e], hi = s[c * 8 + 2 * e + 1];
          if (BF16) {
            __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
            w[e] = *reinterpret_cast<uint32_t*>(&v);
          } else {
            __half2 v = __floats2half2_rn(lo, hi);
            w[e] = *reinterpret_cast<uint32_t*>(&v);
          }
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    ok = ok && mbar_wait(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, p.err, DEVERR_WAIT_SOFTMAX);
    tc_fence_after();
    uint32_t r0[32], r1[32];
    tmem_ld32(tO + lane_off, r0);
    tmem_ld32(tO + lane_off + 32, r1);
    tmem_wait_ld();
    const int qi = q0 + row;
    if (ok && qi < p.Sq) {
      const float inv = 1.0f / l_run;
      uint16_t* o = static_cast<uint16_t*>(p.out) + b * p.o_sb + (long long)qi * p.o_ss + h * p.o_sh;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = c * 8 + 2 * e;
          const float lo = __uint_as_float(i < 32 ? r0[i] : r1[i - 32]) * inv;
          const float hi = __uint_as_float(i + 1 < 32 ? r0[i + 1] : r1[i + 1 - 32]) * inv;
          if (BF16) {
            __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
            w[e] = *reinterpret_cast<uint32_t*>(&v);
          } else {
            __half2 v = __floats2half2_rn(lo, hi);
            w[e] = *reinterpret_cast<uint32_t*>(&v);
          }
        }
        reinterpret_cast<uint4*>(o)[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// layout 0: token-major rows of ld elements holding H heads of 64; layout 1: [B][H][S][64].
bool attn_map(CUtensorMap* m, int dtype, const void* base, int B, int H, int S, int layout, long long ld,
              uint32_t rows) {
  const CUtensorMapDataType dt =
      dtype == DI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  if (layout == 0) {
    dims[0] = 64; dims[1] = H; dims[2] = S; dims[3] = B;
    strides[0] = 128; strides[1] = (uint64_t)ld * 2; strides[2] = (uint64_t)S * ld * 2;
    box[0] = 64; box[1] = 1; box[2] = rows; box[3] = 1;
  } else {
    dims[0] = 64; dims[1] = S; dims[2] = H; dims[3] = B;
    strides[0] = 128; strides[1] = (uint64_t)S * 128; strides[2] = (uint64_t)H * S * 128;
    box[0] = 64; box[1] = rows; box[2] = 1; box[3] = 1;
  }
  std::string err;
  return make_tmap(m, dt, 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &err);
}

}  // namespace

// ld_* = token row stride in elements for layout 0 (H*64 when packed); ignored for layout 1.
int attention(Ctx* c, int dtype, const void* Q, const void* K, const void* V, void* O, int B, int H, int Sq, int Skv,
              int layout, long long ld_q, long long ld_k, long long ld_v, long long ld_o, int causal) {
  if (B <= 0 || H <= 0 || Sq <= 0 || Skv <= 0 || (layout != 0 && layout != 1))
    return set_error(c, DI_EINVAL, "attention: bad shape");
  if (causal && Sq != Skv) return set_error(c, DI_EINVAL, "attention: causal needs Sq == Skv");
  AttnParams p;
  memset(&p, 0, sizeof p);
  if (!attn_map(&p.tmQ, dtype, Q, B, H, Sq, layout, ld_q, QT) || !attn_map(&p.tmK, dtype, K, B, H, Skv, layout, ld_k, KT) ||
      !attn_map(&p.tmV, dtype, V, B, H, Skv, layout, ld_v, KT))
    return set_error(c, DI_EINVAL, "attention: tensor map (pointers and row strides must be 16-byte aligned)");
  p.out = O;
  if (layout == 0) { p.o_sb = (long long)Sq * ld_o; p.o_ss = ld_o; p.o_sh = 64; }
  else { p.o_sb = (long long)H * Sq * 64; p.o_ss = 64; p.o_sh = (long long)Sq * 64; }
  p.Sq = Sq;
  p.Skv = Skv;
  p.H = H;
  p.layout = layout;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  p.err = c->d_err;
  auto kern = dtype == DI_BF16 ? attn_fwd_kernel<true> : attn_fwd_kernel<false>;
  static unsigned attr_done[2] = {0, 0};
  const int di = dtype == DI_BF16;
  if (!(attr_done[di] & (1u << (c->device & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_ATTN) != cudaSuccess)
      return set_error(c, DI_ECUDA, "attention: smem attribute");
    attr_done[di] |= 1u << (c->device & 31);
  }
  dim3 grid((Sq + QT - 1) / QT, H, B);
  launch_k(kern, grid, 192, SMEM_ATTN, c->stream, p);
  return check_launch(c, "attention");
}

}  // namespace di

using namespace di;

extern "C" int di_attention(di_ctx_t h, int dtype, const void* Q, const void* K, const void* V, void* O, int B, int H,
                            int Sq, int Skv, int layout) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  const long long ld = (long long)H * 64;
  return attention(c, dtype, Q, K, V, O, B, H, Sq, Skv, layout, ld, ld, ld, ld, 0);
}

extern "C" int di_attention_causal(di_ctx_t h, int dtype, const void* Q, const void* K, const void* V, void* O, int B,
                                   int H, int S, int layout) {
  Ctx* c = ctx_of(h);
  if (!c || (dtype != DI_F16 && dtype != DI_BF16)) return DI_EINVAL;
  const long long ld = (long long)H * 64;
  return attention(c, dtype, Q, K, V, O, B, H, S, S, layout, ld, ld, ld, ld, 1);
}
