/* di.h — C ABI of libdi, the B200 (sm_100a) kernels for draw-instant's SD-Turbo denoising hot path.
 *
 * Plain C: opaque handles, raw device pointers, sizes and the reference's own packed cfg blocks.
 * Every entry returns DI_OK (0) or a negative DI_E* code and never traps; di_last_error() holds the
 * message.  Launches are asynchronous on the context's stream; di_wait() is the only host sync
 * (the analogue of device.queue.onSubmittedWorkDone()).
 *
 * Each declaration cites the reference interface it replaces (file:line in abgnydn/draw-instant).
 */
#ifndef DI_H_
#define DI_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DI_API __attribute__((visibility("default")))
#else
#define DI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DI_OK 0
#define DI_EINVAL (-1)       /* bad argument / shape (the reference throws an Error) */
#define DI_ECUDA (-2)        /* CUDA runtime / launch error */
#define DI_ENOMEM (-3)       /* device allocation failed */
#define DI_EUNSUPPORTED (-4) /* shape outside what a kernel handles (e.g. wgsl-executor.js:1082) */
#define DI_EFAULT (-5)       /* sticky device fault: a kernel reported a timed-out wait */

/* element types for the fast (NHWC) path */
#define DI_F32 0
#define DI_F16 1
#define DI_BF16 2

typedef struct di_ctx_s* di_ctx_t;
typedef struct di_buf_s* di_buf_t;

/* ---------------------------------------------------------------------------------------------
 * Device, buffers, submission — unet-wgsl.js:64-84 (requestDevice + lost/error hooks),
 * wgsl-ops.js:1172-1210 (createStorage/createOutput/readBack), wgsl-executor.js:1424-1425 (submit).
 * ------------------------------------------------------------------------------------------- */
DI_API int di_init(int device_ordinal, di_ctx_t* out);
DI_API void di_destroy(di_ctx_t ctx);
DI_API int di_set_stream(di_ctx_t ctx, void* cuda_stream); /* caller's cudaStream_t; NULL = default stream */
DI_API void* di_get_stream(di_ctx_t ctx);
DI_API int di_buf_alloc(di_ctx_t ctx, size_t bytes, di_buf_t* out);            /* createOutput */
DI_API int di_buf_free(di_buf_t buf);                                          /* GPUBuffer.destroy */
DI_API void* di_buf_ptr(di_buf_t buf);
DI_API size_t di_buf_size(di_buf_t buf);
DI_API int di_buf_upload(di_buf_t buf, const void* src, size_t bytes, size_t offset);  /* createStorage */
DI_API int di_buf_download(di_buf_t buf, void* dst, size_t bytes, size_t offset);      /* readBack */
DI_API int di_wait(di_ctx_t ctx);                                              /* onSubmittedWorkDone */
DI_API const char* di_last_error(di_ctx_t ctx);
/* getUNetGpuFault analogue (unet-wgsl.js:32-38): reads the device error word; >0 = fault flags. */
DI_API int di_device_fault(di_ctx_t ctx);
DI_API int di_clear_fault(di_ctx_t ctx);

/* Diagnostics (no counterpart in the reference): while set, every tensor-core GEMM launch with at most
 * `ctas` CTAs writes 16 %globaltimer stamps per CTA to buf[cta * 16 + i] (device memory): entry, set-up
 * done, dependency wait passed, first stage landed, last MMA issued, accumulator ready, epilogue done,
 * exit, then epilogue detail (TMEM load issue / done for chunks 0 and 1, store issued for chunks 0, 1).  ctas = 0 switches it off.  Launches in flight keep the pointer they were given. */
DI_API int di_debug_gemm_trace(unsigned long long* buf, int ctas);
/* Fault-path probe (test support for the sticky fault of unet-wgsl.js:32-38): enqueues one kernel whose
 * bounded mbarrier wait (the helper every pipeline kernel uses) waits on a phase nothing completes, gives
 * up after timeout_us (1 .. 1e6) microseconds, sets flag 64 in the device error word and returns: the
 * context stays usable, di_device_fault reports the flag and di_clear_fault clears it.  No trap, no
 * unbounded wait. */
DI_API int di_debug_wait_timeout(di_ctx_t ctx, int timeout_us);

/* ---------------------------------------------------------------------------------------------
 * wgsl-ops.js op families: fp32 tensors in the reference's layouts, cfg blocks exactly as the
 * executor packs them (wgsl-executor.js OPS.* bodies).  Pointers are device pointers.
 * ------------------------------------------------------------------------------------------- */
/* unary ops, wgsl-ops.js:58-72 / :110-122 */
#define DI_SIGMOID 0
#define DI_SQRT 1
#define DI_NEG 2
#define DI_ABS 3
#define DI_SIN 4
#define DI_COS 5
#define DI_EXP 6
#define DI_LOG 7
#define DI_SILU 8
#define DI_GELU 9
#define DI_ERF 10
/* binary ops, wgsl-ops.js:130-134 */
#define DI_ADD 0
#define DI_SUB 1
#define DI_MUL 2
#define DI_DIV 3
#define DI_POW 4
#define DI_MAX 5
#define DI_MIN 6

/* WeightCache's fp16 -> fp32 conversion of raw little-endian fp16 bytes (wgsl-unet.js:23-47), bit-exact
 * for every input including subnormals, Inf and NaN payloads; n halves. */
DI_API int di_f16_bytes_to_f32(di_ctx_t ctx, const void* src, float* dst, size_t n);
DI_API int di_unary(di_ctx_t ctx, int op, const float* X, float* Y, uint32_t n);                 /* wgsl-ops.js:110 */
/* operands wrap at their own length (i % nA, i % nB), wgsl-ops.js:147-151 */
DI_API int di_binary(di_ctx_t ctx, int op, const float* A, uint32_t nA, const float* B, uint32_t nB, float* Y,
              uint32_t n);                                                                 /* wgsl-ops.js:250 */
DI_API int di_binary_bcast(di_ctx_t ctx, int op, const float* A, const float* B, float* Y,
                    const uint32_t cfg[20]);                                               /* wgsl-ops.js:191 */
DI_API int di_affine_bcast(di_ctx_t ctx, const float* A, const float* gamma, const float* beta, float* Y,
                    const uint32_t cfg[20]);                                               /* wgsl-ops.js:239 */
DI_API int di_softmax(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[2]);             /* wgsl-ops.js:285 */
DI_API int di_instance_norm(di_ctx_t ctx, const float* X, const float* gamma, const float* beta, float* Y,
                     const uint32_t cfg[4]);                                               /* wgsl-ops.js:374 */
/* cfg32 = {u32 N, u32 G, u32 cpg, u32 HW, f32 eps, pad x3} (wgsl-executor.js:738-743); fuse_silu applies
 * x/(1+exp(-x)) after the affine (fused-resnet.js:121-166). */
DI_API int di_group_norm(di_ctx_t ctx, const float* X, const float* gamma, const float* beta, float* Y,
                  const void* cfg32, int fuse_silu);                                       /* wgsl-ops.js:460 */
DI_API int di_layer_norm(di_ctx_t ctx, const float* X, const float* gamma, const float* beta, float* Y,
                  const uint32_t cfg[2]);                                                  /* wgsl-ops.js:803 */
/* cfg = {M, N, K, bBatched}; Y[z] = A[z] . B[z|0] (wgsl-ops.js:477-556). */
DI_API int di_matmul(di_ctx_t ctx, const float* A, const float* B, float* Y, const uint32_t cfg[4], uint32_t batch);
/* cfg = {M, N, K, transB}; Y = A . B(^T) + C[col] (wgsl-ops.js:821-897). */
DI_API int di_gemm(di_ctx_t ctx, const float* A, const float* B, const float* C, float* Y, const uint32_t cfg[4]);
/* cfg = {C_in, C_out, K, K*K, H, W, PAD, S, H_out, W_out, 0, 0} (wgsl-executor.js:1088); NCHW, any batch
 * (the reference computes batch 0 only, wgsl-executor.js:1082). */
DI_API int di_conv(di_ctx_t ctx, const float* X, const float* W, const float* bias, float* Y, const uint32_t cfg[12],
            uint32_t n_batch);                                                             /* wgsl-ops.js:700 */
DI_API int di_resize_nearest(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[8]);     /* wgsl-ops.js:945 */
DI_API int di_reduce_mean(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[2]);        /* wgsl-ops.js:975 */
DI_API int di_transpose(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[20]);         /* wgsl-ops.js:1035 */
DI_API int di_pow_scalar(di_ctx_t ctx, const float* X, float* Y, float exponent, uint32_t n);    /* wgsl-ops.js:1076 */
DI_API int di_slice(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[20]);             /* wgsl-ops.js:1126 */
DI_API int di_concat_copy(di_ctx_t ctx, const float* X, float* Y, const uint32_t cfg[4]);        /* wgsl-ops.js:1159 */

/* ---------------------------------------------------------------------------------------------
 * Fast path: NHWC / token-major activations in fp16 or bf16 (dtype DI_F16 / DI_BF16), fp32
 * accumulation on the tcgen05 tensor cores.  These are the kernels the fused blocks and the U-Net
 * plan are built from.
 * ------------------------------------------------------------------------------------------- */
/* GroupNorm over channels-last x = concat(x1[..., C1], x2[..., C2]) per image (x2 may be NULL),
 * y = (x - mean_g) * rsqrt(var_g + eps) * gamma + beta, optional SiLU; var = E[x^2] - mean^2
 * clamped at 0 (wgsl-ops.js:390-458).  y has C1+C2 channels; in and out dtype = dtype. */
DI_API int di_group_norm_nhwc(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW,
                       int G, float eps, const float* gamma, const float* beta, int fuse_silu, void* y);

/* Same as di_group_norm_nhwc, but it allocates no device memory, for callers that cannot let a library
 * call cudaMalloc (a fixed, pre-reserved memory budget, an external allocator that owns the device
 * memory, or latency-critical code that must not take allocation locks).  No counterpart in the
 * reference.  Its scratch is a fixed 1 MiB array inside the library (kept on every GPU that loads the
 * library until the process exits): sizes needing more than N * max(1, min(16, HW/256)) * G * 8 =
 * 1 MiB are rejected with DI_EINVAL.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and loads the GroupNorm kernels' device code; under CUDA's lazy module loading
 * that may allocate.  So make one call per device
 * at start-up, before any stream capture and before the no-allocation period begins; later calls
 * allocate nothing.  The looked-up address is forgotten when a context on that device is destroyed
 * (di_destroy) and looked up again by the next call; do not call it across a device reset without
 * destroying the contexts first.  All calls share the one
 * array: calls that may overlap on the GPU (different streams or contexts on the same device) race and
 * must be serialised by the caller. */
DI_API int di_group_norm_nhwc_noalloc(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N,
                                      int HW, int G, float eps, const float* gamma, const float* beta, int fuse_silu,
                                      void* y);

/* Linear / 1x1 conv: Y[M,N] = X[M,K] . W[N,K]^T (+ bias[N]) (+ R[M,N]); X = concat(X1[M,K1], X2[M,K-K1])
 * along K when X2 != NULL (skip-connection concat without a copy).  K, K1 multiples of 64, N multiple of 16.
 * Replaces the Gemm/MatMul epilogue variants of fused-block-full.js:128-186. */
DI_API int di_linear(di_ctx_t ctx, int dtype, const void* X1, int K1, const void* X2, int M, int K, const void* W, int N,
              const float* bias, const void* R, void* Y);
/* GEGLU feed-forward up-projection: Y[M,F] = (X.Wv^T + bv) * gelu_erf(X.Wg^T + bg), W = [Wv; Wg] as [2F,K]
 * (diffusers GEGLU; erf GELU of wgsl-ops.js:69).  F multiple of 64. */
/* Linear with an activation after the bias, before the residual: act 0 none, 1 SiLU, 2 erf GELU
 * (wgsl-ops.js:69, the text encoder's MLP).  K multiple of 64. */
DI_API int di_linear_act(di_ctx_t ctx, int dtype, const void* X, int M, int K, const void* W, int N, const float* bias,
                         const void* R, int act, void* Y);
DI_API int di_linear_geglu(di_ctx_t ctx, int dtype, const void* X, int M, int K, const void* W, int F, const float* bias,
                    void* Y);
/* 3x3 conv, pad 1, stride 1 or 2, NHWC: x = concat(x1[...,C1], x2[...,C2]) (x2 may be NULL), W packed
 * [Co][ky][kx][C1+C2]; y[N,Ho,Wo,Co] = conv + bias (+ temb[n][co] broadcast) (+ residual).  C1, C2 multiples
 * of 64, Co multiple of 16, W and Ho*Wo powers of two with Wo <= 128.  (wgsl-ops.js:584-711 + the
 * fused-resnet.js:173-208 epilogues.) */
DI_API int di_conv3x3_nhwc(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H, int W,
                    int stride, const void* Wt, int Co, const float* bias, const float* temb, const void* residual,
                    void* y);
/* Packs a reference-layout fp32 conv weight [Co][Ci][3][3] into the [Co][3][3][Ci] dtype layout used above. */
/* di_conv3x3_nhwc with an activation in the epilogue: act 1 = y = silu(conv + bias + temb) + residual
 * (fused-conv.js:50-100 epilogue 'silu_fn(sum) + residual'); act 0 = di_conv3x3_nhwc. */
DI_API int di_conv3x3_nhwc_act(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H,
                               int W, int stride, const void* Wt, int Co, const float* bias, const float* temb,
                               const void* residual, int act, void* y);
/* GroupNorm fused into the conv's operand load (no normalised tensor in memory).  di_gn_table_nhwc
 * reduces concat(x1, x2) [N, HW, C1 + C2] to table[N][C] = (scale, shift) float pairs (8 bytes per
 * channel) with scale = gamma * rstd, shift = beta - mean * scale (fused-groupnorm.js:145-227
 * statistics).  di_conv3x3_nhwc_gn is di_conv3x3_nhwc (stride 1) applied to silu?(x * scale + shift)
 * of the raw x1/x2, the normalisation done in shared memory between the TMA load and the tensor core
 * (fused-resnet.js:121-208 chain: GN -> SiLU -> conv3x3 -> +temb / +residual). */
DI_API int di_gn_table_nhwc(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int HW,
                            int G, float eps, const float* gamma, const float* beta, float* table);
DI_API int di_conv3x3_nhwc_gn(di_ctx_t ctx, int dtype, const void* x1, int C1, const void* x2, int C2, int N, int H,
                              int W, const void* Wt, int Co, const float* bias, const float* temb,
                              const void* residual, const float* gn_table, int silu, void* y);
DI_API int di_pack_conv3x3(di_ctx_t ctx, int dtype, const float* w_oihw, int Co, int Ci, void* w_packed);

/* Attention, head dim 64: O = softmax(Q K^T / 8) V per (b, h).  layout 0 = token-major [B,S,H,64]
 * (fused-attn.js:46-48), 1 = head-major [B,H,S,64] (fused-cross-attn.js:134).  Any Sq, Skv >= 1.
 * Replaces WGSL_FUSED_ATTN (fused-attn.js:199-307) and the cross-attention kernel (fused-cross-attn.js:112-173). */
DI_API int di_attention(di_ctx_t ctx, int dtype, const void* Q, const void* K, const void* V, void* O, int B, int H, int Sq,
                 int Skv, int layout);
/* Causal attention (query i sees keys 0..i; the CLIP text encoder's self-attention), Sq = Skv = S. */
DI_API int di_attention_causal(di_ctx_t ctx, int dtype, const void* Q, const void* K, const void* V, void* O, int B,
                               int H, int S, int layout);

/* Timestep embedding, fused-tembed.js:73-130: y[b] = W2 . silu(W1 . [cos||sin](t_b f) + b1) + b2 with
 * f_i = exp(-ln(1e4) i / (Din/2)); W1 [Dh,Din], W2 [Dh,Dh] row-major fp32; t, y fp32. */
DI_API int di_tembed(di_ctx_t ctx, const float* t, int B, const float* W1, const float* b1, const float* W2,
              const float* b2, int Din, int Dh, float* y);

/* ---------------------------------------------------------------------------------------------
 * Planned fused blocks and the U-Net.  A plan is built once (weights drawn from the seeded generator
 * or supplied per parameter name by `fn`, packed fp16; every buffer and launch fixed) and replayed as
 * one CUDA graph.  Parameter names follow diffusers' UNet2DConditionModel ("down_blocks.0.resnets.0.
 * conv1.weight", ...), values in the reference (PyTorch / ONNX) layouts; `fn` returns 0 when it filled
 * dst with n floats, nonzero to fall back to the generator.
 * ------------------------------------------------------------------------------------------- */
typedef struct di_unet_s* di_unet_t;
typedef struct di_resnet_s* di_resnet_t;
typedef struct di_tblock_s* di_tblock_t;
typedef struct di_vae_s* di_vae_t;
typedef struct di_text_s* di_text_t;
typedef struct di_t2i_s* di_t2i_t;
typedef int (*di_weight_fn)(const char* name, size_t n, float* dst, void* user);

/* The seeded parameter generator: key = mix64(seed*0x9E3779B97F4A7C15 + fnv1a64(name)),
 * u_i = (mix64(key + (i+1)*0x9E3779B97F4A7C15) >> 40) * 2^-24; uniform = (2u-1)*bound (float);
 * normal = Box-Muller (double) on (u_2j, u_2j+1).  Host-only; no GPU needed. */
DI_API void di_synth_uniform(uint64_t seed, const char* name, size_t n, float bound, float* out);
DI_API void di_synth_normal(uint64_t seed, const char* name, size_t n, float mean, float stdv, float* out);
/* The Euler-discrete schedule the one-step pipeline uses (scheduler.js:27-89: scaled-linear betas,
 * trailing timesteps, sigmas rounded to float, last sigma 0): sigmas[n + 1], timesteps[n].  Host-only. */
DI_API int di_euler_sigmas(int n, float* sigmas, float* timesteps);

/* SD-Turbo (SD2.1) U-Net, fp16 weights / activations, fp32 accumulation: replaces unetForwardWGSL
 * (unet-wgsl.js:145-195) and the Executor.run walk it drives (wgsl-executor.js:1248-1466).
 * Latent [B,4,H,W] fp32 NCHW, t [B] fp32, context [B,ctx_len,1024] fp32, output [B,4,H,W] fp32. */
DI_API int di_unet_create(di_ctx_t ctx, int B, int H, int W, int ctx_len, uint64_t seed, di_weight_fn fn, void* user,
                          di_unet_t* out);
DI_API int di_unet_io(di_unet_t u, float** latent, float** t, float** context, float** out); /* device buffers */
DI_API int di_unet_info(di_unet_t u, int* launches, size_t* weight_bytes, size_t* act_bytes);
/* Per-op metadata of the plan (kind 0 GEMM/conv, 1 attention, 2 norm, 3 other; algorithmic FLOPs and HBM
 * bytes; kernels launched).  Arrays may be NULL; call with NULLs first to get n_ops. */
DI_API int di_unet_ops(di_unet_t u, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels);
/* LOG.profile analogue (wgsl-executor.js:1380-1390): replays a graph with an event between every op
 * `reps` times and writes each op's mean device time (ms) to op_ms[n_ops]. */
DI_API int di_unet_profile(di_unet_t u, int reps, float* op_ms);
/* Mean device ms of all ops of one kind replayed alone, in plan order (a graph of just those launches). */
DI_API int di_unet_profile_kind(di_unet_t u, int kind, int reps, float* ms);
DI_API int di_unet_forward(di_unet_t u);  /* enqueue one forward on the context stream (graph replay) */
/* host buffers in, host buffer out, synchronous: the unetForwardWGSL(sample, timestep, cond) shape */
DI_API int di_unet_forward_host(di_unet_t u, const float* latent, const float* t, const float* context, float* out);
DI_API void di_unet_destroy(di_unet_t u);
/* Scheduler on the device (scheduler.js:95-110): the U-Net feeds float(double(latent) * in_scale) to
 * conv_in (scaleModelInput) and writes next = float(double(latent) + dt * double(eps)) (the Euler step,
 * dt = sigma_{i+1} - sigma_i) beside its noise prediction.  Defaults: in_scale 1, dt 0.  *next receives
 * the device buffer [B,4,H,W] fp32. */
DI_API int di_unet_sched(di_unet_t u, double in_scale, double dt, float** next);

/* OpenCLIP ViT-H text encoder (SD2.x / SD-Turbo; run by ONNX Runtime in the reference, text-encoder.js:
 * 69-174): token ids [B,S] int32 (S <= 77, ids in [0, 49408)) -> last_hidden_state [B,S,1024] fp32.
 * `layers` pre-LN blocks (causal 16-head self-attention, MLP 1024->4096->1024 with erf GELU), final
 * LayerNorm; HF CLIPTextModel parameter names (text_model.embeddings.token_embedding.weight, ...). */
DI_API int di_text_create(di_ctx_t ctx, int B, int S, int layers, uint64_t seed, di_weight_fn fn, void* user,
                          di_text_t* out);
DI_API int di_text_io(di_text_t t, int** ids, float** hidden);
DI_API int di_text_info(di_text_t t, int* launches, size_t* weight_bytes, size_t* act_bytes);
DI_API int di_text_ops(di_text_t t, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels);
DI_API int di_text_forward(di_text_t t);
DI_API int di_text_forward_host(di_text_t t, const int* ids, float* hidden);
DI_API void di_text_destroy(di_text_t t);

/* Batched one-step text-to-image (config 5, pipeline.js's SD-Turbo generate path): text encoder ->
 * U-Net at t = 999 with scaleModelInput and the Euler step on the device -> VAE decoder (in chunks of up
 * to 8 images), on shared device buffers.  ids [B,77] int32; latent [B,4,h,w] fp32 = the noise already
 * scaled by initNoiseSigma (sampleNoiseLatent); image [B,3,8h,8w] fp32.  One parameter seed for all
 * three models. */
DI_API int di_t2i_create(di_ctx_t ctx, int B, int h, int w, int text_layers, uint64_t seed, di_weight_fn fn,
                         void* user, di_t2i_t* out);
DI_API int di_t2i_io(di_t2i_t t, int** ids, float** latent, float** image, float** context, float** eps);
DI_API int di_t2i_info(di_t2i_t t, int* launches, size_t* weight_bytes, size_t* act_bytes, float* sigma0);
/* stage -1: the whole pipeline; 0 text encoder, 1 U-Net + scheduler, 2 VAE decoder */
DI_API int di_t2i_forward(di_t2i_t t, int stage);
DI_API int di_t2i_forward_host(di_t2i_t t, const int* ids, const float* latent, float* image);
DI_API void di_t2i_destroy(di_t2i_t t);

/* SD VAE decoder (config 5's image decode; vae-wgsl.js:99-118 runs it through the same executor):
 * diffusers AutoencoderKL decode = latent / 0.18215 -> post_quant_conv -> Decoder (conv_in 4->512, mid
 * ResNet / single-head attention / ResNet, up blocks 512, 512, 256, 128 with 3 ResNets each and 2x
 * nearest upsample + conv, GroupNorm(32, 1e-6) + SiLU, conv_out 128->3).  Latent [B,4,h,w] fp32 NCHW
 * (h*w a multiple of 64), image [B,3,8h,8w] fp32 NCHW; parameter names are diffusers' (post_quant_conv.*,
 * decoder.*).  Activations reuse a ring of buffers (the decoder is a chain). */
DI_API int di_vae_create(di_ctx_t ctx, int B, int h, int w, uint64_t seed, di_weight_fn fn, void* user, di_vae_t* out);
DI_API int di_vae_io(di_vae_t v, float** latent, float** image);
DI_API int di_vae_info(di_vae_t v, int* launches, size_t* weight_bytes, size_t* act_bytes);
DI_API int di_vae_ops(di_vae_t v, int* n_ops, int* kinds, double* flops, double* bytes, int* kernels);
DI_API int di_vae_profile_kind(di_vae_t v, int kind, int reps, float* ms);
DI_API int di_vae_forward(di_vae_t v);
DI_API int di_vae_forward_host(di_vae_t v, const float* latent, float* image);
DI_API void di_vae_destroy(di_vae_t v);
/* Diagnostics: copy `bytes` at `off` of activation-ring buffer idx (idx < 0: temporary arena) to host. */
DI_API int di_vae_debug_copy(di_vae_t v, int idx, size_t off, void* dst, size_t bytes);

/* Config-1 ResNet block, fp32 NCHW in and out (fused-resnet.js:121-208 + the timestep add it omits,
 * fused-resnet.js:9-12): y = conv2(silu(gn2(conv1(silu(gn1(x))) + Wt.act(temb) + bt))) + x;
 * act = SiLU when temb_silu (diffusers), identity otherwise.  Names: norm1/conv1/time_emb_proj/norm2/conv2. */
DI_API int di_resnet_block_create(di_ctx_t ctx, int N, int C, int H, int W, int Tdim, uint64_t seed, float eps,
                                  int temb_silu, di_weight_fn fn, void* user, di_resnet_t* out);
DI_API int di_resnet_block_io(di_resnet_t r, float** x, float** temb, float** y);
DI_API int di_resnet_block_run(di_resnet_t r); /* runResNetBench's fused path (fused-resnet.js:340-350) */
DI_API void di_resnet_block_destroy(di_resnet_t r);

/* Config-2 SD2.1 transformer block (GN + proj_in, self-attn, cross-attn, GEGLU FF, proj_out + residual),
 * fp16 token-major hidden [B,S,C] and context [B,Sk,Cctx]; parameter names prefixed "block."
 * (runBlockBench's fused path, fused-block-full.js:456-686). */
DI_API int di_transformer_block_create(di_ctx_t ctx, int B, int S, int C, int Sk, int Cctx, uint64_t seed,
                                       di_weight_fn fn, void* user, di_tblock_t* out);
DI_API int di_transformer_block_io(di_tblock_t t, void** hidden, void** context, void** out);
DI_API int di_transformer_block_run(di_tblock_t t);
DI_API void di_transformer_block_destroy(di_tblock_t t);

#ifdef __cplusplus
}
#endif
#endif /* DI_H_ */
