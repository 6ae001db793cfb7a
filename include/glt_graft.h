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
  GLT_ETIMEOUT = 5, /* a bounded device wait gave up (see glt_device_error) */
  GLT_ESTATE = 6,   /* call not legal in the current state (e.g. double bake) */
  GLT_ENOMEM = 7    /* allocation failed                                  */
} GltStatus;

/* Message of the last failing call on this thread ("" if none). */
GLT_API const char* glt_last_error(void);
/* Library version string. */
GLT_API const char* glt_version(void);
/* Reads and clears the device error word of the current device
 * (1 = mbarrier wait timed out, 2 = bad shape seen by a kernel). */
GLT_API int glt_device_error(unsigned int* out_code);
/* Copies `bytes` between any host/device pointers on `stream` (cudaMemcpyDefault);
 * synchronises the stream when sync != 0.  Lets bindings move data in and out
 * of library-owned buffers without their own CUDA runtime binding. */
GLT_API int glt_memcpy(void* dst, const void* src, int64_t bytes, void* stream, int sync);
/* Number of kernels this library has launched in the process so far. */
GLT_API int glt_launch_count(uint64_t* out);

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

/* ------------------------------------------------------------------------ */
/* Model (frozen bf16 base + fp32 graft, one CUDA device per handle)        */
/* Replaces load_base_model_safetensors/ModelWeights (src/model_io_impl.inc) */
/* allocate_arena/VramArena (src/arena_impl.inc:14-126) and                 */
/* allocate_graft_weights/GraftWeights (src/graft_weights_impl.inc:6-62).   */
/* kind: GLT_MODEL_DECODER runs the full decoder step; GLT_MODEL_MLP_BLOCK  */
/* runs one pre-RMSNorm grafted MLP block with residual. */
/* ------------------------------------------------------------------------ */
#define GLT_MODEL_DECODER 0
#define GLT_MODEL_MLP_BLOCK 1

typedef struct GltModel GltModel;

GLT_API int glt_model_create(const GltModelConfig* cfg, int batch_size, int seq_len, int kind,
                             GltModel** out);
GLT_API int glt_model_destroy(GltModel* m);
/* Bytes of device memory held by the model (arena + graft buffers). */
GLT_API int glt_model_memory(const GltModel* m, int64_t* arena_bytes, int64_t* graft_bytes);

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
 * CE on domain tokens + OOD silence loss, backward with FFN recompute,
 * global-norm clip, graft-only AdamW.  ids/ood_mask are [B*T] int32; with
 * host_inputs = 1 they are host pointers copied inside the call.  If stats
 * is non-NULL the call synchronises the stream and fills it. */
GLT_API int glt_train_step(GltModel* m, const int32_t* ids, const int32_t* ood_mask,
                           int host_inputs, int step, int total_steps, GltStepStats* stats,
                           void* stream);

/* Forward only; writes bf16 logits [B*T, V] (device) when logits != NULL.
 * use_graft = 0 runs the base model (graft columns skipped). */
GLT_API int glt_forward(GltModel* m, const int32_t* ids, int host_inputs, int use_graft,
                        uint16_t* logits, void* stream);

/* MLP-block step: out = x + MLP(rms_norm(x)),
 * loss = mean((out - y)^2), backward to the graft, AdamW with lr.
 * x: bf16 [M, D] device; y: fp32 [M, D] device.  Optional outputs: out (bf16),
 * dx (fp32 grad wrt x), loss (host float, synchronises). */
GLT_API int glt_block_step(GltModel* m, const uint16_t* x, const float* y, float lr, int step,
                           float* loss, uint16_t* out, float* dx, void* stream);

/* Saved activations for tests: which = 0 residual input of layer, 1 qkv,
 * 2 attention output, 3 x_post_attn, 4 x_ffn, 5 per-token energy sums
 * [3][M] fp32 (sum of squares of the gate/up/down deltas), 6 final hidden. */
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
#define GLT_PROF_KINDS 17
GLT_API int glt_model_profile(GltModel* m, int enable);
GLT_API int glt_model_profile_read(GltModel* m, double* ms, int64_t* launches, int reset);

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

#ifdef __cplusplus
}
#endif

#endif /* GLT_GRAFT_H_ */
