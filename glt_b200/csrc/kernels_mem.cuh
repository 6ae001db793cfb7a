// Declarations of the bandwidth-bound kernels' host launchers (kernels_mem.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace glt {

// RMSNorm forward: y = bf16(x * rsqrt(mean(x^2) + eps) * w), var = mean(x^2).
// Reference: rms_norm_fwd_kernel (src/kernels_rmsnorm_kernels.inc:8-60).
int rmsnorm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, float* var, int M, int D,
                float eps, cudaStream_t st);

// RMSNorm backward fused with the residual add:
//   out = resid + dy*r*w - x*mean(dy*x*w)*r^3,   r = rsqrt(var + eps)
// (src/kernels_rmsnorm_kernels.inc:70-126, src/layer_backward_impl.inc:367-368).
// resid may be null or alias out; out_bf16 (optional) receives bf16(out).
int rmsnorm_bwd(const float* dy, const uint16_t* x, const uint16_t* w, const float* var,
                const float* resid, float* out, uint16_t* out_bf16, int M, int D, float eps,
                cudaStream_t st);

// x[t,:] = E[ids[t],:]   (at::embedding, grafting.hip:233)
int embedding_fwd(const int32_t* ids, const uint16_t* E, uint16_t* x, int M, int D, int V,
                  cudaStream_t st);

// Step-level device scalars (one per model).
struct DevStats {
  double ce_sum;            // sum over domain label positions of CE
  double dom_energy_sum;    // sum_l,p sum_t energy * (1 - ood)
  double ood_energy_sum;    // sum_l,p sum_t energy * ood
  double grad_sq;           // sum of squared graft grads
  float in_count;           // domain label positions (clamped to >= 1)
  float ood_count;          // OOD tokens
  float lambda_eff;         // lambda / (ood_count * active_grafts) or 0
  float clip_scale;         // global-norm clip factor
  float lm_loss, silence, domain_energy, ood_energy, ratio, total_loss, grad_norm;
  unsigned int dev_err;     // device error word collected at the end of the step
  float pad[2];
};

// Counts domain label positions and OOD tokens.
int count_tokens(const int32_t* ood, int B, int T, DevStats* stats, cudaStream_t st);

// Cross-entropy over one chunk of rows of bf16 logits [rows, V]; adds the
// masked CE sum to stats->ce_sum and overwrites the logits with bf16
// dlogits = (softmax - onehot) * mask * scale / in_count  (grafting.hip:1027-1135).
int cross_entropy_chunk(uint16_t* logits, int64_t ld, int rows, int row0, int V,
                        const int32_t* ids, const int32_t* ood, int T, float scale,
                        DevStats* stats, cudaStream_t st,
                        const int* row_map = nullptr, const int* n_rows = nullptr);
// Rows whose next-token label counts in the LM loss (t % T < T-1 and
// ood[t+1] == 0), in order, into rows[0, *n_rows) (one CTA).
int live_rows(const int32_t* ood, int M, int T, int* rows, int* n_rows, cudaStream_t st);
// dst[i] = src[rows[i]] for i < *n_rows (bf16 rows of D).
int gather_rows(const uint16_t* src, uint16_t* dst, const int* rows, const int* n_rows, int M, int D,
                cudaStream_t st);

// Silence bookkeeping.  esq holds per-token sum of squares of each grafted
// projection's delta output, laid out [L][3][M].
int silence_stats(const float* esq, const int* proj_enabled /*[L*3] dev*/, int L, int M,
                  int S, int H, const int32_t* ood, DevStats* stats, cudaStream_t st);
// MSE gradient of the MLP-block config: dx = 2 (out - y) / numel, loss sum -> stats->ce_sum.
int mse_grad(const uint16_t* out, const float* y, float* dx, DevStats* stats, int M, int D,
             cudaStream_t st);
int set_clip_scale(DevStats* stats, float v, cudaStream_t st);
// stats->lambda_eff = v (a caller-supplied silence weight for a layer-level backward).
int set_lambda_eff(DevStats* stats, float v, cudaStream_t st);
// Stream-ordered collection of the device error word (kernels that give up a
// bounded wait set it): v = *word | *accum, then *word = 0; with dst, *dst = v
// and *accum = 0, else *accum = v.  No host synchronisation.
int collect_device_error(unsigned int* word, unsigned int* accum, unsigned int* dst, cudaStream_t st);
// Finalises losses and lambda_eff on the device (grafting.hip:1097-1117).
int finalize_loss(DevStats* stats, float lambda_silence, int active_grafts, float lm_loss_scale,
                  cudaStream_t st);

// dy = bf16(dx) over all D columns;  on the graft's hidden window [h0, h0+H):
// dyg[:, j] = bf16(dx[:, h0+j] + s_t * delta_down[:, j]) with
// s_t = ood_t * lambda_eff / (sqrt(esq_t + 1e-8) * sqrt(H))  (silence_blend_kernel,
// src/kernels_elementwise_impl.inc:8-67).  delta_down may be null (no down
// graft).  h0 and H are multiples of 8; concat geometry is h0 = 0, H = D.
int silence_down_prep(const float* dx, const uint16_t* delta_down, int64_t ld_dd,
                      const float* esq_down, const int32_t* ood, const DevStats* stats,
                      uint16_t* dy, uint16_t* dyg, int64_t ld_dyg, int M, int D, int h0, int H,
                      cudaStream_t st);

// Global L2 norm of gscale * grads -> stats->clip_scale = gscale * min(1, clip/norm)
// (reduce_l2/calc_scale, src/kernels_elementwise_impl.inc:133-197; gscale = 1/world
// turns all-reduced sums into means).
int grad_clip_scale(const float* grad, int64_t n, float clip_norm, float gscale,
                    DevStats* stats, cudaStream_t st);

// Where the bf16 mirror of each graft projection lives: inside the fused
// concat weights (w_gu / w_d), or, for the overlay geometry, a plain bf16
// [3L, S, H] copy in the delta_offset layout (`plain`).  Both may be null.
struct MirrorTargets {
  uint16_t* plain;   // overlay: bf16 image at the same flat index, or null
  uint16_t** w_gu;   // [L] device pointers to W_gu_cat (2F' x D, interleaved 128-blocks)
  uint16_t** w_d;    // [L] device pointers to W_d_cat (D x F')
  int f_pad;         // first graft column in the intermediate index space
  int ffn;           // F' (row count of W_gu_cat / 2 and ld of W_d_cat)
  int D;
  int layer_begin, layer_end;  // grafted layer range (inclusive)
  int kinds[3];                // grafted projection kinds
};

// Fused AdamW over all 3L projections with the clip scale read on the device;
// disabled projection kinds are skipped (kernels_optimizer_impl.inc:11-77).
// Also refreshes the bf16 mirror inside the concat weights.
// bf16 image of the grafted down projections in W_d_cat (a shared-memory
// staged transpose of the [S, H] fp32 graft).
int mirror_down(const float* w, int L, int S, int H, const MirrorTargets& mt, cudaStream_t st);
int adamw_step(float* w, const float* grad, float* m, float* v, int L, int S, int H, float lr,
               float beta1, float beta2, float eps, float wd, int step, const int* kinds_enabled,
               const DevStats* stats, const MirrorTargets* mirror, cudaStream_t st);

// Copies the bf16 image of the fp32 graft weights into the concat weights.
int refresh_mirror(const float* w, int L, int S, int H, const MirrorTargets& mirror,
                   cudaStream_t st);

// Shadow bake (shadow_bake_kernel, src/shadow_bake_impl.inc:15-51):
// mode 0: base[i0+s, h0+h] = bf16(base + g[s,h]);  mode 1: base[h0+h, i0+s] = ...
int shadow_bake(uint16_t* base, int64_t base_stride, const float* g, int S, int H, int i0, int h0,
                int mode, cudaStream_t st);

// Shadow bake of every enabled (layer, projection) of the graft straight into
// the fused layer weights (W_gu interleaved 128-row gate/up blocks, W_d
// [D, ffn]) of the overlay geometry: intermediate index i0+s, hidden index
// h0+h; same bf16 round-to-nearest-even of base + delta as shadow_bake.
int shadow_bake_fused(const float* g, int L, int S, int H, int i0, int h0,
                      const MirrorTargets& mt, cudaStream_t st);

// Deterministic N(0, std) init (counter-based hash + Box-Muller).
int init_normal_bf16(uint16_t* p, int64_t n, uint64_t seed, float std, cudaStream_t st);
int init_normal_f32(float* p, int64_t n, uint64_t seed, float std, cudaStream_t st);
int fill_bf16(uint16_t* p, int64_t n, float v, cudaStream_t st);

// Packs a strided [rows, cols] matrix (fp32 or bf16 source) into bf16 rows of
// length ld_dst (zero padded); used to stage operands for TMA.
int pack_bf16(const void* src, int src_is_f32, int64_t src_ld, int rows, int cols, uint16_t* dst,
              int64_t ld_dst, cudaStream_t st);
int cast_f32_to_bf16(const float* src, uint16_t* dst, int64_t n, cudaStream_t st);

}  // namespace glt
