/*
 * glt_graft.h -- C ABI of the B200-native grafted-MLP training library.
 *
 * Drop-in boundary for the hot path of Hinedes/GLT ("grafting"): a frozen
 * bf16 decoder whose SwiGLU MLPs carry trainable fp32 graft slices (gate/up/
 * down deltas), trained with graft-only AdamW, optionally shadow-baked into
 * the base weights for inference.
 *
 * The reference exposes no FFI; its internal API is free C++ functions
 * taking VramArena& / GraftWeights& plus raw device pointers.  Each entry
 * point below names the reference function(s) it replaces (path:line inside
 * the reference project).  Conventions:
 *   - plain pointers and sizes only; device pointers are marked "dev",
 *     host pointers "host";
 *   - every function returns a GltStatus (0 = ok) and never throws; the
 *     message of the last failure on the calling thread is glt_last_error();
 *     the reference logs file:line and throws std::runtime_error
 *     (src/checks.hpp:10-44) or returns [[nodiscard]] bool for I/O
 *     (src/checkpoint_impl.inc:170, src/data_impl.inc:9);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - handles are not thread-safe; use one handle per rank thread.
 */
#ifndef GLT_GRAFT_H_
#define GLT_GRAFT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GLT_API __attribute__((visibility("default")))
#else
#define GLT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status                                                                   */
/* ------------------------------------------------------------------------ */
typedef enum GltStatus {
  GLT_OK = 0,
  GLT_EINVAL = 1,   /* bad argument / shape / alignment                   */
  GLT_ECUDA = 2,    /* CUDA runtime or driver error                       */
  GLT_ENCCL = 3,    /* NCCL error                                         */
  GLT_EIO = 4,      /* file I/O or format error                           */
  GLT_ETIMEOUT = 5, /* a kernel gave up a bounded device wait (glt_device_error) */
  GLT_ESTATE = 6,   /* call not legal in the current state (e.g. double bake) */
  GLT_ENOMEM = 7    /* allocation failed                                  */
} GltStatus;

/* Message of the last failing call on this thread ("" if none). */
GLT_API const char* glt_last_error(void);
/* Library version string. */
GLT_API const char* glt_version(void);
/* Reads and clears the device error words of the current device (the one
 * every kernel uses and the one of glt_graft_op_noalloc): 1 = a bounded
 * mbarrier wait ran out, 2 = a kernel saw a bad shape.  Synchronises.
 * The model calls report these codes themselves: glt_model_step_stats (and
 * glt_train_step with stats), glt_model_eval and glt_block_step with a loss
 * collect the word on their stream at the end of the work they read back
 * (also covering the model's earlier glt_forward calls and pipelined steps)
 * and return GLT_ETIMEOUT (code 1) or GLT_EINVAL (code 2) with the results.
 * A kernel that gives up a wait leaves its outputs incomplete, writes the
 * code, waits for its own copies and tensor-core work in flight, frees its
 * tensor memory and exits; the next launch starts clean (no code is
 * consulted by later launches).  The reference throws from its CHECK macros
 * (src/checks.hpp:10-44). */
GLT_API int glt_device_error(unsigned int* out_code);
/* Failure-path self-test (no counterpart in the reference): runs one small
 * GEMM in which CTA 0 never receives its first k-block, so that CTA's waits
 * run out after timeout_ms (1..2000) and it takes the abort path above; the
 * other CTAs finish normally.  mode 0: reads and clears the device word and
 * returns GLT_ETIMEOUT (the expected result); mode 1: returns GLT_OK and
 * leaves the code in the device word for the next model call to report;
 * mode 2: the same with the word of glt_graft_op_noalloc, which
 * glt_device_error reports.  Synchronises. */
GLT_API int glt_selftest_wait_timeout(int timeout_ms, int mode, void* stream);
/* Copies `bytes` between any host/device pointers on `stream` (cudaMemcpyDefault);
 * synchronises the stream when sync != 0.  Lets bindings move data in and out
 * of library-owned buffers without their own CUDA runtime binding. */
GLT_API int glt_memcpy(void* dst, const void* src, int64_t bytes, void* stream, int sync);
/* Device allocation for bindings that have no CUDA runtime of their own. */
GLT_API int glt_malloc(void** ptr, int64_t bytes);
GLT_API int glt_free(void* ptr);
/* Number of kernels this library has launched in the process so far. */
GLT_API int glt_launch_count(uint64_t* out);
/* Device memory in use and in total on the current device (cudaMemGetInfo);
 * the reference samples hipMemGetInfo for peak_train_vram_mb (grafting.hip:807-821). */
GLT_API int glt_device_memory(int64_t* used_bytes, int64_t* total_bytes);

/* ------------------------------------------------------------------------ */
/* Generic tensor-core GEMM (bf16 x bf16 -> fp32 accumulate)                */
/* Replaces gemm_core (src/gemm_impl.inc:21-58): one sm_100a tcgen05 kernel */
/* instead of rocblas_gemm_ex.  Row-major view:                            */
/*   C[M,N] = alpha * A[M,K] * B[N,K]^T + beta * C                          */
/* a_mn = 0: A stored [M][lda] (K contiguous); a_mn = 1: A stored [K][lda].   */
/* b_mn = 0: B stored [N][ldb] (K contiguous); b_mn = 1: B stored [K][ldb].   */
/* c_dtype: 0 = fp32, 1 = bf16 (beta must be 0 for bf16).                   */
/* ------------------------------------------------------------------------ */
GLT_API int glt_gemm(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
             void* C, int64_t ldc, int c_dtype, int M, int N, int K, float alpha, float beta,
             void* stream);
/* Tile shape of the library's 256-column GEMMs (every call above and every */
/* GEMM of a model step): mode 1 runs them on CTA pairs                     */
/* (tcgen05.mma.cta_group::2, 256 x 256 tiles, 128 rows of A and B staged   */
/* per CTA), mode 0 on single CTAs (128 x 256 tiles).  -1 only queries.     */
/* Returns the mode in force.  Default 1; the environment variable          */
/* GLT_GEMM_PAIR=0 at the first call makes it 0.  Process-wide; change it   */
/* only while no GEMM is being enqueued.                                    */
GLT_API int glt_gemm_pair_mode(int mode);


/* ------------------------------------------------------------------------ */
/* Workspace for the stand-alone graft ops (the reference's arena scratch,  */
/* arena.d_bf16_temp, src/arena_impl.inc:14-126).                           */
/* ------------------------------------------------------------------------ */
typedef struct GltArena GltArena;
GLT_API int glt_arena_create(int64_t scratch_bytes, GltArena** out);
GLT_API int glt_arena_destroy(GltArena* arena);

/* ------------------------------------------------------------------------ */
/* The six graft GEMMs in general (overlay) geometry, one tcgen05 kernel.   */
/* W is one projection's delta in storage orientation [S, H] row-major:     */
/* fp32 (w_f32, rounded to bf16 like graft_gemm_fwd, gemm_impl.inc:398-405) */
/* or its bf16 mirror (w_bf16, used when non-NULL).  x / dy are bf16        */
/* (x_is_f32 / dy_is_f32 = 0) or fp32 (rounded to bf16 first, as           */
/* grad_gemm does with dy, gemm_impl.inc:455, 525), with row strides in     */
/* elements; out is fp32: out = alpha * (product) + beta * out.  Operands   */
/* TMA cannot read in place are packed into `arena` (GLT_ENOMEM with the    */
/* needed size if it is too small).                                         */
/*   EXPAND_FWD     out[M,S] = x_h[M,H] . W^T   execute_expand_forward      */
/*                                                (graft_ops_impl.inc:14-24) */
/*   CONTRACT_FWD   out[M,H] = x_i[M,S] . W     execute_contract_forward    */
/*                                                (graft_ops_impl.inc:33-114)*/
/*   EXPAND_WGRAD   out[S,H] = dy[M,S]^T . x_h  execute_expand_grad_gemm    */
/*                                                (graft_ops_impl.inc:120-132)*/
/*   CONTRACT_WGRAD out[S,H] = x_i[M,S]^T . dy[M,H]                         */
/*                  execute_contract_backward_storage_canonical (:214-228)  */
/*   EXPAND_DGRAD   out[M,H] = dy[M,S] . W      ExpandInputGrad             */
/*                  (layer_backward_impl.inc:277-342; this is the math of   */
/*                  docs/test_contract_audit.py op 3 and of the reference's */
/*                  ATen path)                                              */
/*   CONTRACT_DGRAD out[M,S] = dy_h[M,H] . W^T  ContractInputGrad           */
/*                  (layer_backward_impl.inc:117-155)                       */
/* ------------------------------------------------------------------------ */
#define GLT_GRAFT_EXPAND_FWD 0
#define GLT_GRAFT_CONTRACT_FWD 1
#define GLT_GRAFT_EXPAND_WGRAD 2
#define GLT_GRAFT_CONTRACT_WGRAD 3
#define GLT_GRAFT_EXPAND_DGRAD 4
#define GLT_GRAFT_CONTRACT_DGRAD 5
GLT_API int glt_graft_op(int op, int M, int S, int H, const float* w_f32, const uint16_t* w_bf16,
                         const void* x, int x_is_f32, int64_t x_stride, const void* dy,
                         int dy_is_f32, int64_t dy_stride, float* out, int64_t out_stride,
                         float alpha, float beta, GltArena* arena, void* stream);

/* Allocation-free variant of glt_graft_op (same ops and arguments, no     */
/* arena).  It has no counterpart in the reference.  It is for callers that */
/* must not call cudaMalloc -- code inside a framework whose caching        */
/* allocator owns the device memory, or latency-critical paths that cannot  */
/* afford cudaMalloc's implicit device synchronisation.  Operands that need */
/* staging go to a fixed 16 MiB workspace compiled into the library (held  */
/* by every GPU that loads it until exit); larger staging needs return      */
/* GLT_EINVAL.  The first call on a device looks up the workspace address   */
/* (cudaGetSymbolAddress) and should come before any stream capture.  All   */
/* calls on a device share the workspace: calls that may overlap on the GPU */
/* race and must be serialised by the caller.                               */
GLT_API int glt_graft_op_noalloc(int op, int M, int S, int H, const float* w_f32,
                                 const uint16_t* w_bf16, const void* x, int x_is_f32,
                                 int64_t x_stride, const void* dy, int dy_is_f32,
                                 int64_t dy_stride, float* out, int64_t out_stride, float alpha,
                                 float beta, void* stream);

/* ------------------------------------------------------------------------ */
/* Shadow bake (src/shadow_bake_impl.inc:15-128).                           */
/* glt_shadow_bake: one projection, in place, bit-exact with the reference: */
/*   mode 0 (expand):   base[i0+s, h0+h] = bf16(base + graft[s,h])          */
/*   mode 1 (contract): base[h0+h, i0+s] = bf16(base + graft[s,h])          */
/* glt_apply_graft_to_shadow: every grafted layer and projection of a model  */
/* given per-layer device pointers (host arrays, NULL to skip a kind), the  */
/* flat [3L,S,H] graft, and the caller's guard flag (g_shadow_baked): a    */
/* second bake with the flag set returns GLT_ESTATE.  Synchronises.         */
/* ------------------------------------------------------------------------ */
GLT_API int glt_shadow_bake(uint16_t* base, int64_t base_stride, const float* graft, int S, int H,
                            int i0, int h0, int mode, void* stream);
/* (declared after GltModelConfig below) */

/* ------------------------------------------------------------------------ */
/* SwiGLU as stand-alone ops (the fused training step computes both inside  */
/* its GEMM epilogues).  bf16 = uint16 bit patterns; fp32 gradients.        */
/* glt_swiglu_fwd replaces fused_silu_product_strided_kernel                */
/*   (kernels_elementwise_impl.inc:411-448): out[r, c] =                    */
/*   bf16(silu(gate_pre[r, c]) * up[r, c]) over rows x width, each operand  */
/*   with its own row stride (elements).  width and strides multiples of 8, */
/*   pointers 16-byte aligned, else GLT_EINVAL.                             */
/* glt_swiglu_bwd replaces fused_gate_up_bwd_kernel                         */
/*   (kernels_elementwise_impl.inc:80-124): with sg = sigmoid(gp),          */
/*   grad_gate_pre = grad_h * up * sg * (1 + gp * (1 - sg)),                */
/*   grad_up = grad_h * gp * sg, over n contiguous elements (n % 8 == 0).   */
/* ------------------------------------------------------------------------ */
GLT_API int glt_swiglu_fwd(const uint16_t* gate_pre, const uint16_t* up, uint16_t* out, int rows,
                           int width, int64_t gate_ld, int64_t up_ld, int64_t out_ld, void* stream);
GLT_API int glt_swiglu_bwd(float* grad_gate_pre, float* grad_up, const float* grad_h,
                           const uint16_t* up, const uint16_t* gate_pre, int64_t n, void* stream);

/* ------------------------------------------------------------------------ */
/* Layer kernels for callers that run their own layer loop.                 */
/* qkv: packed rows [q heads | k heads | v heads] of B*T tokens (ld_qkv     */
/* elements per row), bf16; o / dout: [B*T, nh*hd] rows with ld_o; lse:     */
/* [B, nh, T] fp32 natural-log sum-exp of the scaled scores.               */
/* Attention = causal GQA SDPA (layer_forward_impl.inc:41-49; K/V heads     */
/* indexed, not repeat_interleave'd); backward = attention_bwd_autograd's  */
/* gradient (attention_autograd_impl.inc:1-39) into dqkv (same packing),   */
/* with fp32 workspaces dq_acc [B*T, nh*hd] and dsum [B*nh*T]; the        */
/* tcgen05 backward at hd 64 needs dq_acc of B*T*(nh + 2*nkv)*hd floats     */
/* (its dK/dV accumulators follow dQ).                                      */
/* impl: GLT_ATTN_TCGEN05 (tcgen05/TMEM kernels, seq_len % 128 == 0) or     */
/* GLT_ATTN_MMA_SYNC (seq_len % 64 == 0).  hd: 64 or 128.                   */
/* RoPE: half-split rotation in place on q and k (rope_impl.inc:8-64);      */
/* inverse = 1 applies the transpose (its backward).                        */
/* RMSNorm: rms_norm_fwd_kernel / rms_norm_bwd_kernel                       */
/* (kernels_rmsnorm_kernels.inc:8-126); bwd adds resid (may be NULL).       */
/* ------------------------------------------------------------------------ */
#define GLT_ATTN_TCGEN05 0
#define GLT_ATTN_MMA_SYNC 1
GLT_API int glt_attention_fwd(const uint16_t* qkv, int64_t ld_qkv, uint16_t* o, int64_t ld_o,
                              float* lse, int B, int T, int nh, int nkv, int hd, int impl,
                              void* stream);
GLT_API int glt_attention_bwd(const uint16_t* qkv, int64_t ld_qkv, const uint16_t* o,
                              const uint16_t* dout, int64_t ld_o, const float* lse, uint16_t* dqkv,
                              float* dq_acc, float* dsum, int B, int T, int nh, int nkv, int hd,
                              int impl, void* stream);
GLT_API int glt_rope(uint16_t* qkv, int64_t ld_qkv, int B, int T, int nh, int nkv, int hd,
                     float theta, int inverse, void* stream);
GLT_API int glt_rmsnorm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, float* var, int M,
                            int D, float eps, void* stream);
GLT_API int glt_rmsnorm_bwd(const float* dy, const uint16_t* x, const uint16_t* w,
                            const float* var, const float* resid, float* dx, int M, int D,
                            float eps, void* stream);

/* ------------------------------------------------------------------------ */
/* Configuration                                                            */
/* Mirrors GraftConfig (src/config.hpp:40-91) plus the CLI-level values of  */
/* grafting.hip:274-292.  layout selects the graft geometry:                */
/*   GLT_LAYOUT_OVERLAY (0): the reference's own semantics -- deltas added  */
/*     into slice [domain*S, +S) x [domain*H, +H), H = hidden/max_domains   */
/*     (src/layer_forward_impl.inc:21-22);                                  */
/*   GLT_LAYOUT_CONCAT (1): [base | graft] intermediate, i.e. overlay on a  */
/*     base zero-padded from F to F+S with i0 = F, h0 = 0, H = hidden.      */
/* ------------------------------------------------------------------------ */
#define GLT_LAYOUT_OVERLAY 0
#define GLT_LAYOUT_CONCAT 1

typedef struct GltModelConfig {
  int hidden_dim, intermediate_dim, slice_dim, vocab_size;
  int num_layers, num_heads, num_kv_heads, head_dim; /* head_dim 0: hidden/heads */
  int max_domains, domain_id, layout, tie_embeddings;
  float rms_norm_eps, lm_loss_scale, lambda_silence, rope_theta;
  int graft_layer_start, graft_layer_end; /* inclusive range */
  int graft_proj_gate, graft_proj_up, graft_proj_down, allow_expansion_trap;
  float adam_beta1, adam_beta2, adam_eps, adam_weight_decay, gradient_clip_norm;
  int lr_warmup_steps;
  float lr_peak;
  int no_rope_mask_len;            /* 0 or num_layers */
  int no_rope_mask[256];           /* per layer: nonzero = apply RoPE (layer_forward_impl.inc:37) */
} GltModelConfig;

/* Reference defaults (src/config.hpp:42-90; lr 2e-4 from grafting.hip:281). */
GLT_API int glt_config_default(GltModelConfig* cfg);
/* Host-only validation of the reference CLI rules (grafting.hip:364-444,
 * 715-786: positivity, divisibility, projection flags, expansion-trap
 * refusal, even batch).  mode: 0 = train, 1 = eval/shadow-eval. */
GLT_API int glt_config_validate(const GltModelConfig* cfg, int batch_size, int mode);
/* LR schedule: linear warm-up then cosine decay (src/config.hpp:122-129). */
GLT_API float glt_get_lr(const GltModelConfig* cfg, int step, int total_steps);
/* Flat offset of projection p of layer l in [3L,S,H] (src/graft_ops_impl.inc:5-7). */
GLT_API int64_t glt_delta_offset(int layer, int proj, int slice_dim, int h_slice_dim);
/* glt_stack_grafts: a stack of n sibling grafts of the overlay geometry     */
/* (domains 0..n-1 of one session, each a flat [3L, S, H] fp32 device       */
/* buffer, H = hidden / max_domains) -> one [3L, n*S, n*H] graft whose       */
/* projections are block-diagonal: domain d at rows [dS, (d+1)S) and columns */
/* [dH, (d+1)H), zeros elsewhere.  Loaded as the graft of a model with       */
/* slice_dim n*S, max_domains 1 and domain_id 0, it injects every domain's   */
/* delta into the reference's slice for that domain -- the explicit stack of */
/* tests/test6_stack_vs_bake_f32.cpp -- and glt_model_shadow_bake bakes all  */
/* n at once (zero blocks leave the bf16 base bits unchanged).  grafts is a  */
/* host array of n (<= 8) device pointers; out is device memory; H % 4 == 0. */
GLT_API int glt_stack_grafts(const float* const* grafts, int n, int num_layers, int S, int H,
                             float* out, void* stream);
/* glt_grad_clip replaces the clip of grafting.hip:1150-1164 (reduce_l2 /   */
/* calc_scale / apply_scale, kernels_elementwise_impl.inc:125-213): with     */
/* norm = sqrt(sum g^2 + 1e-8) over the n fp32 grads (16-byte aligned),      */
/* writes scale = clip_norm / norm if norm > clip_norm else 1 to *scale_out */
/* (device), the norm to *norm_out (device, nullable), and with              */
/* apply_in_place = 1 multiplies the grads by it; with 0 pass scale_out as   */
/* glt_adamw_all's grad_scale instead.  The sum of squares is fp64.          */
/* workspace: device memory of at least 8192 bytes (8-byte aligned).         */
GLT_API int glt_grad_clip(float* grads, int64_t n, float clip_norm, int apply_in_place,
                          void* workspace, int64_t workspace_bytes, float* scale_out,
                          float* norm_out, void* stream);
/* glt_adamw_all replaces execute_adamw_all + adamw_fused_kernel             */
/* (kernels_optimizer_impl.inc:11-77): one AdamW step over the flat          */
/* [3L, S, H] graft (weights, grads, adam_m, adam_v fp32, 16-byte aligned), */
/* bias corrections 1/(1-beta^(step+1)), decoupled weight decay, projection */
/* kinds disabled in cfg skipped entirely.  weights_bf16 (nullable, 8-byte  */
/* aligned) receives the RNE bf16 image at the same flat index.  grad_scale */
/* (nullable device pointer) multiplies every gradient (the clip scale).    */
/* Hyper-parameters come from cfg (adam_beta1/2, adam_eps,                  */
/* adam_weight_decay); S * H must be a multiple of 4.                       */
GLT_API int glt_adamw_all(float* weights, uint16_t* weights_bf16, const float* grads,
                          float* adam_m, float* adam_v, const float* grad_scale,
                          const GltModelConfig* cfg, int step, float lr, void* stream);

/* apply_graft_to_shadow (src/shadow_bake_impl.inc:58-128); see glt_shadow_bake. */
GLT_API int glt_apply_graft_to_shadow(const GltModelConfig* cfg, uint16_t* const* gate,
                                      uint16_t* const* up, uint16_t* const* down,
                                      int64_t gate_up_stride, int64_t down_stride,
                                      const float* graft, int* baked_flag, void* stream);

/* ------------------------------------------------------------------------ */
/* Model (frozen bf16 base + fp32 graft, one CUDA device per handle)        */
/* Replaces load_base_model_safetensors/ModelWeights (src/model_io_impl.inc) */
/* allocate_arena/VramArena (src/arena_impl.inc:14-126) and                 */
/* allocate_graft_weights/GraftWeights (src/graft_weights_impl.inc:6-62).   */
/* kind: GLT_MODEL_DECODER runs the full decoder step; GLT_MODEL_MLP_BLOCK  */
/* runs one pre-RMSNorm grafted MLP block with residual.                   */
/* ------------------------------------------------------------------------ */
#define GLT_MODEL_DECODER 0
#define GLT_MODEL_MLP_BLOCK 1

typedef struct GltModel GltModel;

GLT_API int glt_model_create(const GltModelConfig* cfg, int batch_size, int seq_len, int kind,
                             GltModel** out);
GLT_API int glt_model_destroy(GltModel* m);
/* Bytes of device memory held by the model (arena + graft buffers). */
GLT_API int glt_model_memory(const GltModel* m, int64_t* arena_bytes, int64_t* graft_bytes);
/* Stored MLP activations.  No counterpart in the reference, whose backward
 * recomputes gate_pre/up per layer (recompute_ffn,
 * src/layer_recompute_impl.inc:8-91).  With the store on, the training
 * forward keeps the bf16 gate_pre/up of every layer (num_layers * M * 2F' * 2
 * bytes, F' = intermediate + slice columns rounded up) and the backward
 * fuses SwiGLU's backward into the dh GEMM: no recompute GEMM.  mode 0:
 * recompute (the reference's memory profile); 1: store, allocated now
 * (GLT_ENOMEM when it does not fit); 2: auto, the default -- decided at the
 * next training step, store when free device memory exceeds the store plus
 * max(8 GiB, 1/16 of the device); -1: query only.  Both geometries (overlay
 * stores the pre-activations after the delta injection).  GLT_MLP_STORE=0|1|2
 * in the environment sets the mode at glt_model_create.  *active (nullable)
 * = 1 while the store is allocated, *bytes (nullable) = its size.
 * Synchronizes the device. */
GLT_API int glt_model_mlp_store(GltModel* m, int mode, int* active, int64_t* bytes);

/* load_base_model_safetensors (src/model_io_impl.inc:57-190): path is one
 * .safetensors file or a directory of shards (read in sorted order); HF
 * tensor names; BF16/F16/F32 converted to bf16 (RNE); lm_head.weight absent
 * means tied (the model must be created with tie_embeddings = 1, and with 0
 * when it is present); lm_head stored [D, V] is transposed. */
GLT_API int glt_model_load_safetensors(GltModel* m, const char* path, void* stream);
/* Looks a tensor up by name in a safetensors file or directory: found = 0/1,
 * ndim and up to 8 dims of its shape.  Host only (no device work). */
GLT_API int glt_safetensors_tensor_info(const char* path, const char* name, int* found,
                                        int64_t* shape, int* ndim);

/* Seeded N(0, std) base init (norm weights 1), graft gate/up N(0, graft_std),
 * graft down N(0, graft_down_std); Adam state zeroed. */
GLT_API int glt_model_init_random(GltModel* m, uint64_t seed, float std, float graft_std,
                                  float graft_down_std);

/* Base weights, HF shapes, bf16.  layer = -1 for the model-level tensors. */
#define GLT_W_EMBED 0      /* [V, D]     */
#define GLT_W_LM_HEAD 1    /* [V, D]     */
#define GLT_W_FINAL_NORM 2 /* [D]        */
#define GLT_W_IN_NORM 3    /* [D]        */
#define GLT_W_Q 4          /* [nh*hd, D] */
#define GLT_W_K 5          /* [nkv*hd, D]*/
#define GLT_W_V 6          /* [nkv*hd, D]*/
#define GLT_W_O 7          /* [D, nh*hd] */
#define GLT_W_POST_NORM 8  /* [D]        */
#define GLT_W_GATE 9       /* [F, D]     */
#define GLT_W_UP 10        /* [F, D]     */
#define GLT_W_DOWN 11      /* [D, F]     */
GLT_API int glt_model_set_weight(GltModel* m, int layer, int which, const void* src_bf16,
                                 int64_t numel, int src_is_host, void* stream);

/* Device pointers of the fp32 graft buffers, each [3L, S, H] (delta_offset
 * layout); m/v are the AdamW moments (arena.d_adam_m/v). */
GLT_API int glt_model_graft_buffers(GltModel* m, float** weight, float** grad, float** adam_m,
                                    float** adam_v, int64_t* numel);
/* Re-derives the bf16 graft copies inside the fused weights after the fp32
 * graft weights were written externally (refresh_graft_weight_bf16). */
GLT_API int glt_model_refresh_graft(GltModel* m, void* stream);

typedef struct GltStepStats {
  float lm_loss, silence_loss, domain_graft_energy, ood_graft_energy;
  float domain_ood_energy_ratio, total_loss, lr, grad_norm;
} GltStepStats;

/* One training step (grafting.hip:954-1172): forward with saved activations,
 * CE on domain tokens + OOD silence loss, backward (from stored or
 * recomputed FFN pre-activations, glt_model_mlp_store), global-norm clip,
 * graft-only AdamW.  ids/ood_mask are [B*T] int32; with host_inputs = 1 they
 * are host pointers copied inside the call (the host buffers may be reused
 * as soon as it returns).  If stats is non-NULL the call waits for the step
 * and fills it; with NULL it only enqueues the step. */
GLT_API int glt_train_step(GltModel* m, const int32_t* ids, const int32_t* ood_mask,
                           int host_inputs, int step, int total_steps, GltStepStats* stats,
                           void* stream);
/* The stats of an enqueued training step (one of the last two): waits for
 * that step only, so a caller can enqueue step k+1 before reading step k's
 * stats and keep the device busy while it logs (the reference reads them
 * with .item() host syncs).  GLT_EINVAL for an older step. */
GLT_API int glt_model_step_stats(GltModel* m, int step, GltStepStats* stats);

/* Forward only; writes bf16 logits [B*T, V] (device) when logits != NULL.
 * use_graft = 0 runs the base model (graft columns skipped). */
GLT_API int glt_forward(GltModel* m, const int32_t* ids, int host_inputs, int use_graft,
                        uint16_t* logits, void* stream);

/* Eval-only / shadow-eval metrics (grafting.hip:446-713): the deterministic
 * forward over num_sequences sequences of the model's seq_len tokens
 * (ids [num_sequences, seq_len] int32, host or device), in batches of the
 * model's batch size (a shorter last batch is run as is).
 *   mean_ce   mean next-token cross entropy over every position t < T-1 of
 *             every sequence (no OOD mask), ppl = exp(mean_ce)
 *   logits_sum / logits_l2  sum and L2 norm of all logits read as fp32
 *   logits_hash  FNV-1a 64 over the little-endian fp32 bytes of the logits in
 *             [sequence, position, vocab] order, chained across batches
 *   graft_forward_calls  layers run with graft GEMMs (the reference's
 *             g_graft_fwd_calls; 0 for a base-only or shadow eval)
 * use_graft = 1 is the explicit-graft eval (--eval-only with a checkpoint),
 * 0 the base model or, after glt_model_shadow_bake, the shadow model.
 * Synchronises the stream. */
typedef struct GltEvalStats {
  int64_t tokens;
  double total_nll, mean_ce, ppl, logits_sum, logits_l2;
  uint64_t logits_hash;
  int64_t graft_forward_calls;
} GltEvalStats;
GLT_API int glt_model_eval(GltModel* m, const int32_t* ids, int64_t num_sequences, int host_ids,
                           int use_graft, GltEvalStats* out, void* stream);

/* apply_graft_to_shadow for the model's own graft (shadow_bake_impl.inc:58-128):
 * bakes the enabled projections of the grafted layer range into the base
 * weights (bf16 round-to-nearest-even of base + delta), then frees the graft
 * storage as --shadow-eval does before its first forward (grafting.hip:483-490).
 * A second call fails (g_shadow_baked guard); training, graft access and
 * use_graft = 1 forwards fail afterwards.  Synchronises the stream. */
GLT_API int glt_model_shadow_bake(GltModel* m, void* stream);

/* MLP-block step: out = x + MLP(rms_norm(x)),
 * loss = mean((out - y)^2), backward to the graft, AdamW with lr.
 * x: bf16 [M, D] device; y: fp32 [M, D] device.  Optional outputs: out (bf16),
 * dx (fp32 grad wrt x), loss (host float, synchronises). */
GLT_API int glt_block_step(GltModel* m, const uint16_t* x, const float* y, float lr, int step,
                           float* loss, uint16_t* out, float* dx, void* stream);

/* Saved activations for tests: which = 0 residual input of layer, 1 qkv,
 * 2 attention output, 3 x_post_attn, 4 x_ffn, 5 per-token energy sums
 * [3][M] fp32 (sum of squares of the gate/up/down deltas), 6 final hidden;
 * concat geometry only: 7 the layer's fused gate/up weights [2F' x D] bf16
 * (intermediate column c at row 256*(c/128) + c%128, +128 for up; graft
 * column s at c = F_pad + s, F_pad = F rounded up to 256), 8 its fused down
 * weights [D x F'] bf16 (F' = F_pad + S rounded up to 128). */
GLT_API int glt_model_activation(GltModel* m, int which, int layer, void** ptr, int64_t* numel);

/* Per-kind kernel timing: CUDA events recorded on the launching stream around
 * each launch of the kinds below while enabled -- the counterpart of the
 * reference's --profile-graft-gemms per-kind stats (src/gemm_impl.inc:153-199,
 * 408-444).  read: ms[k] total milliseconds and launches[k] launch counts per
 * kind since the last reset (synchronises the model's recorded work). */
#define GLT_PROF_GATE_UP_FWD 0   /* x.W_gu^T + SwiGLU epilogue              */
#define GLT_PROF_DOWN_FWD 1      /* h.W_d^T + residual                      */
#define GLT_PROF_DELTA_DOWN 2    /* h_graft.Delta_down (+ energy)           */
#define GLT_PROF_QKV 3
#define GLT_PROF_OPROJ 4
#define GLT_PROF_ATTN_FWD 5
#define GLT_PROF_DH 6            /* dy.W_d                                  */
#define GLT_PROF_RECOMPUTE 7     /* x.W_gu^T recompute + SwiGLU backward    */
#define GLT_PROF_WGRAD_DOWN 8
#define GLT_PROF_WGRAD_GATE_UP 9
#define GLT_PROF_DX_GATE_UP 10   /* dgu.W_gu                                */
#define GLT_PROF_DO 11
#define GLT_PROF_ATTN_BWD 12
#define GLT_PROF_DX_QKV 13
#define GLT_PROF_LM_HEAD 14
#define GLT_PROF_LM_DX 15
#define GLT_PROF_CE 16
#define GLT_PROF_DELTA_EXPAND 17 /* overlay: x_h.Delta_{gate,up}^T (+ energy) */
#define GLT_PROF_GRAFT_DGRAD 18  /* overlay: dyh.Delta_down^T, dys.Delta_gu  */
#define GLT_PROF_RMSNORM 19      /* RMSNorm forward and backward            */
#define GLT_PROF_ROPE 20         /* RoPE on q/k and its transpose on dq/dk  */
#define GLT_PROF_ADAMW 21        /* grad clip norm + AdamW + bf16 image     */
#define GLT_PROF_KINDS 22
GLT_API int glt_model_profile(GltModel* m, int enable);
GLT_API int glt_model_profile_read(GltModel* m, double* ms, int64_t* launches, int reset);

/* ------------------------------------------------------------------------ */
/* Graft weights outside any arena: allocate_graft_weights /                */
/* free_graft_weights_noexcept (src/graft_weights_impl.inc:6-62).          */
/* alloc: the fp32 master [3L, S, H] (delta_offset layout; H = hidden for   */
/* the concat layout, hidden / max_domains for overlay) and, with           */
/* with_bf16_mirror, its bf16 mirror, both zeroed; active = 0 (the caller   */
/* sets it once a checkpoint, init or training load is applied).  A struct */
/* still allocated is freed first.  free: releases both buffers and resets  */
/* every field (safe on a freed or zeroed struct).                          */
/* ------------------------------------------------------------------------ */
typedef struct GltGraftWeights {
  float* weight;          /* device fp32 [3L, S, H]         (d_weight)      */
  uint16_t* weight_bf16;  /* device bf16 mirror, or NULL    (d_weight_bf16) */
  int64_t weight_elems;
  int domain_id;
  int allocated;
  int active;
} GltGraftWeights;
GLT_API int glt_graft_weights_alloc(const GltModelConfig* cfg, int domain_id, int with_bf16_mirror,
                                    GltGraftWeights* g);
GLT_API int glt_graft_weights_free(GltGraftWeights* g);

/* ------------------------------------------------------------------------ */
/* Layer-level grafted MLP, for callers that keep the reference's own layer */
/* loop: the MLP halves of forward_layer (src/layer_forward_impl.inc:53-285), */
/* recompute_ffn (src/layer_recompute_impl.inc:8-91) and backward_layer     */
/* (src/layer_backward_impl.inc:36-367), in the same fused tcgen05 GEMMs as */
/* glt_train_step.  A GltMlp holds, for cfg.num_layers layers, the frozen   */
/* bf16 post-attention norm and gate/up/down weights in the fused layout    */
/* with the graft's bf16 image inside, and the scratch of one layer for     */
/* `tokens` rows (M = batch * seq).  The caller owns the activations, the   */
/* saved tensors (GltMlpSaved, the MLP fields of LayerActivations), the     */
/* graft weights (GltGraftWeights) and their gradients.  All device         */
/* pointers 16-byte aligned; calls are stream-ordered and do not            */
/* synchronise (a device timeout is reported by glt_device_error).          */
/* ------------------------------------------------------------------------ */
typedef struct GltMlp GltMlp;
typedef struct GltMlpSaved {
  uint16_t* x_ffn;       /* [M, D] bf16 post-attention RMSNorm output (x_ffn_input)   */
  float* variance;       /* [M] fp32 mean square of x_post (rms_norm_variance)        */
  float* energy_sq;      /* [3, M] fp32 per-token sums of squares of the gate, up and */
                         /* down delta outputs (energy = sqrt(esq + 1e-8) / sqrt(width)) */
  uint16_t* delta_down;  /* [M, H] bf16 delta_down_out (needed when down is grafted)  */
} GltMlpSaved;
GLT_API int glt_mlp_create(const GltModelConfig* cfg, int tokens, GltMlp** out);
GLT_API int glt_mlp_destroy(GltMlp* m);
/* which: GLT_W_POST_NORM [D], GLT_W_GATE / GLT_W_UP [F, D], GLT_W_DOWN [D, F], bf16. */
GLT_API int glt_mlp_set_weight(GltMlp* m, int layer, int which, const void* src_bf16, int64_t numel,
                               int src_is_host, void* stream);
/* Copies the bf16 image (reference rounding) of g->weight into the fused    */
/* weights the GEMMs read, and into g->weight_bf16 when present: after a    */
/* load or an optimizer step (refresh_graft_weight_bf16).                   */
GLT_API int glt_mlp_set_graft(GltMlp* m, const GltGraftWeights* g, void* stream);
/* Forward of layer `layer`: x_out = x_post + MLP(rms_norm(x_post)) with the */
/* graft's expand deltas injected into gate/up and its contract delta into   */
/* the output (use_graft = 0: base only), bf16 [M, D]; fills saved.          */
GLT_API int glt_mlp_fwd(GltMlp* m, int layer, const uint16_t* x_post, uint16_t* x_out,
                        const GltMlpSaved* saved, int use_graft, void* stream);
/* recompute_ffn: the layer's bf16 gate_pre/up (deltas injected) from       */
/* saved->x_ffn into gate_up, a private blocked layout of                   */
/* glt_mlp_recompute_bytes bytes that glt_mlp_bwd reads.                    */
GLT_API int glt_mlp_recompute_bytes(const GltMlp* m, int64_t* bytes);
GLT_API int glt_mlp_recompute(GltMlp* m, int layer, const GltMlpSaved* saved, void* gate_up,
                              void* stream);
/* Backward of layer `layer`'s MLP half and post-attention RMSNorm: dx (fp32 */
/* [M, D], in/out) enters as the gradient of x_out and leaves as that of     */
/* x_post (the residual included); x_post is the forward's input.  The       */
/* layer's three [S, H] slices of grad ([3L, S, H] fp32) are overwritten     */
/* with the graft gradients, the OOD silence term included (ood_mask [M]     */
/* int32 device, lambda_effective = lambda / (ood_count * active_grafts) as  */
/* grafting.hip:1104).  gate_up: this layer's glt_mlp_recompute output, or   */
/* NULL to recompute gate/up inside the backward's own GEMM.                 */
GLT_API int glt_mlp_bwd(GltMlp* m, int layer, float* dx, const uint16_t* x_post,
                        const GltMlpSaved* saved, const void* gate_up, const int32_t* ood_mask,
                        float lambda_effective, float* grad, void* stream);

/* ------------------------------------------------------------------------ */
/* GRFT checkpoint (src/checkpoint_impl.inc).  Bytes: u32 "GRFT" LE | u8 4  */
/* | u64 header size (JSON NUL-padded to 8) | safetensors JSON | bf16      */
/* delta_weights [3L,S,H] (bias-trick rounding, checkpoint_impl.inc:49-57). */
/* save: save_safetensors (:32-89), refuses a directory or a missing parent */
/* directory.  load: load_safetensors_checkpoint (:170-285): accepts the    */
/* GRFT prefix or a legacy plain safetensors file, checks dtype, shape,     */
/* session_id (when both are set) and domain_id (when present; the file's   */
/* value is returned in *file_domain_id, -1 if missing).  Host-only when    */
/* the weight buffers are host buffers (src_is_host / dst_is_host = 1).     */
/* ------------------------------------------------------------------------ */
GLT_API int glt_checkpoint_save(const char* path, const float* weights, int64_t numel,
                                int src_is_host, const char* session_id, int domain_id,
                                int slice_dim, int h_slice_dim, int hidden_dim, int num_layers);
GLT_API int glt_checkpoint_load(const char* path, float* weights, int64_t numel, int dst_is_host,
                                int expected_domain_id, const char* session_id,
                                int total_projections, int slice_dim, int h_slice_dim,
                                int* file_domain_id);
/* Model-level save/load of its fp32 graft (load also refreshes the bf16 graft
 * copies in the fused weights and leaves the Adam state untouched, like --checkpoint). */
GLT_API int glt_model_save_checkpoint(GltModel* m, const char* path, const char* session_id,
                                      int domain_id);
GLT_API int glt_model_load_checkpoint(GltModel* m, const char* path, const char* session_id,
                                      int expected_domain_id);

/* ------------------------------------------------------------------------ */
/* Training state: no counterpart in the reference, whose checkpoint holds  */
/* only the bf16 deltas, so that --checkpoint restarts Adam's moments, its  */
/* bias correction and the LR schedule (grafting.hip:876-880).  This file   */
/* resumes a run exactly: the fp32 master graft, both Adam moments and the  */
/* index of the next step.  Bytes: u32 "GLTS" LE | u8 1 | u64 header size  */
/* (JSON NUL-padded to 8) | JSON {"__metadata__": {format "glt-train-state",*/
/* session_id, domain_id, slice_dim, h_slice_dim, hidden_dim, num_layers,   */
/* step}, "weights" / "adam_m" / "adam_v": F32 [3L,S,H] with data_offsets}  */
/* | fp32 LE data.  load checks format, dtype, shape, session_id (when both */
/* are set) and domain_id, and leaves the destination untouched on failure  */
/* (host destinations; device ones are written tensor by tensor).           */
/* ------------------------------------------------------------------------ */
GLT_API int glt_train_state_save(const char* path, const float* weights, const float* adam_m,
                                 const float* adam_v, int64_t numel, int src_is_host,
                                 const char* session_id, int domain_id, int slice_dim,
                                 int h_slice_dim, int hidden_dim, int num_layers, int64_t step);
GLT_API int glt_train_state_load(const char* path, float* weights, float* adam_m, float* adam_v,
                                 int64_t numel, int dst_is_host, const char* session_id,
                                 int expected_domain_id, int total_projections, int slice_dim,
                                 int h_slice_dim, int64_t* step);
/* Sibling grafts of a stack, one GRFT file each (the reference trains and
 * ships one graft per domain; test6_stack_vs_bake_f32.cpp runs N of them at
 * once).  The model's graft holds the N siblings, slice_dim = N * S_sib:
 * concat geometry side by side over the full hidden width (sibling d on
 * graft rows [d*S_sib, (d+1)*S_sib) -- N slices trained jointly), or the
 * overlay stack geometry of glt_stack_grafts (max_domains = 1, domain_id 0;
 * block-diagonal, sibling d also on hidden columns [d*H_sib, (d+1)*H_sib),
 * H_sib = H / N).  save writes sibling d to paths[d] as GRFT v4 with
 * domain_id d and its own [3L, S_sib, H_sib] shape; load checks and reads
 * all N files (domain_id d each, session_id when both are set), then sets the
 * graft to their assembly (zeros elsewhere) and refreshes its bf16 copies;
 * the Adam state is untouched. */
GLT_API int glt_model_save_stack(GltModel* m, const char* const* paths, int n, const char* session_id);
GLT_API int glt_model_load_stack(GltModel* m, const char* const* paths, int n, const char* session_id);
/* Model-level: its fp32 graft and Adam state; load also refreshes the bf16
 * graft copies in the fused weights.  `step` is the index of the next
 * training step (glt_train_step's step argument). */
GLT_API int glt_model_save_train_state(GltModel* m, const char* path, const char* session_id,
                                       int domain_id, int64_t step);
GLT_API int glt_model_load_train_state(GltModel* m, const char* path, const char* session_id,
                                       int expected_domain_id, int64_t* step);

/* ------------------------------------------------------------------------ */
/* Token data (host).  .bin = [i32 nseq][i32 seq_len][i32 tokens...] with   */
/* the checks of load_bin (src/data_impl.inc:9-58); tokens = NULL reads and */
/* validates only the header.  The batch walk is grafting.hip:924-988:      */
/* splitmix64-seeded start positions, then per step the first B/2 rows from */
/* the domain corpus (mask 0) and the last B/2 from the OOD corpus (mask 1). */
/* ------------------------------------------------------------------------ */
GLT_API int glt_load_bin(const char* path, int32_t* num_sequences, int32_t* seq_len,
                         int32_t* tokens, int64_t capacity);
GLT_API int glt_batch_walk_start(uint64_t seed, int n_domain, int n_ood, int* domain_pos,
                                 int* ood_pos);
GLT_API int glt_batch_step(const int32_t* domain_tokens, int n_domain, const int32_t* ood_tokens,
                           int n_ood, int seq_len, int batch_size, int* domain_pos, int* ood_pos,
                           int32_t* ids_out, int32_t* ood_mask_out);

/* ------------------------------------------------------------------------ */
/* Data parallelism (new: the reference is single-GPU).  One process per   */
/* GPU; each rank trains on its own microbatch and the graft gradients are */
/* sum-all-reduced per layer over NCCL (NVLink/NVSwitch), overlapped with  */
/* the backward of the remaining layers; clip + AdamW use the mean.        */
/* Rank 0 creates the id and shares it with the others out of band.       */
/* ------------------------------------------------------------------------ */
GLT_API int glt_dp_unique_id(void* out, int out_bytes); /* out_bytes >= 128 */
GLT_API int glt_dp_init(GltModel* m, const void* unique_id, int rank, int world);
GLT_API int glt_dp_finalize(GltModel* m);
/* Failure handling between steps.  glt_dp_async_error: the communicator's  */
/* asynchronous state (ncclCommGetAsyncError) in *nccl_result; GLT_ENCCL    */
/* when a collective failed.  glt_dp_abort: tears the communicator down     */
/* without waiting for the other ranks (ncclCommAbort), for a rank that     */
/* learned on the host that a peer has left (glt_b200.graft.PeerMonitor);   */
/* call it with no step in flight.  The model then trains on its own GPU.   */
GLT_API int glt_dp_async_error(GltModel* m, int* nccl_result);
GLT_API int glt_dp_abort(GltModel* m);

#ifdef __cplusplus
}
#endif

#endif /* GLT_GRAFT_H_ */
