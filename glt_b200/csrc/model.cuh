// Model handle behind the opaque GltModel* of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/glt_graft.h"
#include "kernels_mem.cuh"

namespace glt {

int config_default(GltModelConfig* c);
int config_validate(const GltModelConfig* c, int batch_size, int mode);
float get_lr(const GltModelConfig* c, int step, int total_steps);

struct Layer {
  // frozen weights (bf16)
  uint16_t* in_norm = nullptr;    // [D]
  uint16_t* wqkv = nullptr;       // [(nh + 2 nkv) hd, D]  q rows, k rows, v rows
  uint16_t* wo = nullptr;         // [D, nh hd]
  uint16_t* post_norm = nullptr;  // [D]
  uint16_t* w_gu = nullptr;       // [2F', D] interleaved gate/up 128-row blocks (+ graft rows)
  uint16_t* w_d = nullptr;        // [D, F'] (+ graft columns = Delta_down^T)
  // saved activations
  float* var1 = nullptr;          // [M] input-norm mean square
  uint16_t* qkv = nullptr;        // [M, QKV] after RoPE
  uint16_t* o = nullptr;          // [M, nh hd]
  float* lse = nullptr;           // [B, nh, T]
  uint16_t* x_post = nullptr;     // [M, D] after attention residual
  uint16_t* x_ffn = nullptr;      // [M, D] post-attention RMSNorm output
  float* var2 = nullptr;          // [M]
  float* esq = nullptr;           // [3][M] per-token sum of squares of gate/up/down deltas
  uint16_t* dd = nullptr;         // [M, H] delta_down (bf16), for the silence gradient
  uint16_t* gu = nullptr;         // [M, 2F'] gate_pre/up (bf16, W_gu's interleaving) while
                                  // the MLP store is on; null: the backward recomputes them
};

// Running eval totals on the device (eval.cu).
struct EvalAccum {
  double nll, sum, sumsq;
  uint64_t hash;
  unsigned int dev_err;   // device error word collected at the end of the eval
  unsigned int pad;
};

struct Model {
  GltModelConfig cfg{};
  int kind = 0;
  int B = 0, T = 0, M = 0, D = 0, F = 0, S = 0, H = 0, V = 0, L = 0;
  int nh = 0, nkv = 0, hd = 0, QKV = 0, AD = 0;
  int F_pad = 0, S_pad = 0, FF = 0;
  // Graft geometry: overlay (the reference's) puts the slice on intermediate
  // columns [i0, i0+S) and hidden columns [h0, h0+H) of the base; concat
  // appends S graft columns at i0 = F_pad with h0 = 0, H = D.
  bool overlay = false;
  int i0 = 0, h0 = 0;
  std::vector<int> enabled;  // [3L] should_graft_proj
  int active_grafts = 0;
  bool shadow_baked = false;

  // parameters
  uint16_t* embed = nullptr;
  uint16_t* lm_head = nullptr;
  uint16_t* final_norm = nullptr;
  std::vector<Layer> layers;
  void* graft_mem = nullptr;
  size_t graft_bytes = 0;
  int64_t graft_numel = 0;
  float* gw = nullptr;
  float* grad = nullptr;
  float* adam_m = nullptr;
  float* adam_v = nullptr;

  // arena
  void* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<uint16_t*> xs;   // [L+1] residual stream at layer boundaries
  float* esq_all = nullptr;    // [L][3][M]
  uint16_t* xn = nullptr;
  uint16_t* h = nullptr;
  float* dx = nullptr;
  float* dtmp = nullptr;
  uint16_t* dy_b = nullptr;
  uint16_t* dyg_b = nullptr;
  uint16_t* dh = nullptr;
  uint16_t* dgu = nullptr;
  uint16_t* hg = nullptr;
  uint16_t* gwb = nullptr;     // overlay: bf16 mirror of the graft [3L, S, H]
  float* dlt = nullptr;        // overlay: expand deltas [M, 2S] fp32 (gate | up)
  uint16_t* dys = nullptr;     // overlay: silence-blended expand grads [M, 2S] bf16
  uint16_t* dqkv = nullptr;
  uint16_t* dout_b = nullptr;
  float* dq_acc = nullptr;
  float* dsum = nullptr;
  uint16_t* xf = nullptr;
  float* varf = nullptr;
  float* var_in = nullptr;
  uint16_t* logits = nullptr;
  int ce_rows = 0;
  int* lm_rows = nullptr;      // token rows that carry LM loss, compacted [M]
  int* n_lm_rows = nullptr;    // their count (device)
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  DevStats* stats = nullptr;
  DevStats* pinned_stats = nullptr;   // [2]: the stats of the last two training steps
  cudaEvent_t stats_ev[2] = {nullptr, nullptr};
  int stats_step[2] = {-1, -1};
  float stats_lr[2] = {0.f, 0.f};
  int step_stats(int step, GltStepStats* out);
  int* d_enabled = nullptr;
  uint16_t** d_gu_ptrs = nullptr;
  uint16_t** d_wd_ptrs = nullptr;
  int32_t* ids = nullptr;
  int32_t* ood = nullptr;
  float last_lr = 0.f;
  // Device error codes of this model's calls that return without a host
  // sync (glt_forward, a pipelined glt_train_step), held until the next call
  // that reads its results back reports them (glt_model_step_stats, eval, a
  // block step with its loss).
  unsigned int* d_err = nullptr;
  // GEMM tile-claim counter of this model's stream, used with
  // GLT_GEMM_SCHEDULE=dynamic (default static: round-robin units)
  int* tile_ctr = nullptr;
  int* gemm_counter() const { return tile_ctr_on ? tile_ctr : nullptr; }
  bool tile_ctr_on = false;

  // Stored MLP activations: the training forward keeps bf16 gate_pre/up of
  // every layer (L * M * 2F' * 2 bytes) so the backward fuses SwiGLU's
  // backward into the dh GEMM instead of recomputing x.W_gu^T.
  void* gu_mem = nullptr;
  size_t gu_bytes = 0;
  int store_mode = 2;          // 0 recompute, 1 store, 2 auto (decided at the next training step)
  bool store_decided = false;
  bool saving = false;         // a training forward is running (writes layers[l].gu)
  int set_mlp_store(int mode);
  int ensure_mlp_store();
  int alloc_mlp_store(bool required);
  void free_mlp_store();

  // data parallel (NCCL, loaded at run time)
  void* nccl_comm = nullptr;
  int dp_rank = 0, dp_world = 1;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> layer_done;
  cudaEvent_t comm_done = nullptr;
  bool own_stream_events = false;

  // Layer-level use (glt_mlp_*, mlp_layers.cu): the caller owns the saved
  // activations, the graft weights and their gradients; the model holds only
  // the fused weights and the scratch of one layer at a time.  The per-layer
  // saved pointers, dx, grad and ood are set by each call.
  bool external_acts = false;
  int ffn_recompute(int l, cudaStream_t st);   // gate_pre/up of layer l into layers[l].gu

  ~Model();
  int setup(const GltModelConfig& c, int batch, int seq, int kind);
  int allocate();
  MirrorTargets mirror() const;
  int set_weight(int layer, int which, const void* src, int64_t numel, int host, cudaStream_t st);
  int init_random(uint64_t seed, float std, float graft_std, float graft_down_std);
  int refresh_graft(cudaStream_t st);
  bool rope_on(int l) const;
  int ffn_forward(int l, const uint16_t* x_in, uint16_t* x_out, float* var_out, bool use_graft,
                  cudaStream_t st);
  int forward_layer(int l, bool use_graft, cudaStream_t st);
  // model_overlay.cu
  int expand_deltas(int l, bool gate, bool up, float* esq_gate, float* esq_up, cudaStream_t st);
  int ffn_forward_overlay(int l, const uint16_t* x_in, uint16_t* x_out, float* var_out,
                          bool use_graft, cudaStream_t st);
  int ffn_backward_overlay(int l, cudaStream_t st);
  int ffn_backward(int l, cudaStream_t st);
  int backward_layer(int l, cudaStream_t st);
  int load_inputs(const int32_t* ids_in, const int32_t* ood_in, int host, cudaStream_t st);
  int forward_all(bool use_graft, cudaStream_t st);
  int train_step(const int32_t* ids_in, const int32_t* ood_in, int host, int step,
                 int total_steps, GltStepStats* out, cudaStream_t st);
  int finish_step(int step, int total_steps, GltStepStats* out, cudaStream_t st);
  int forward_logits(const int32_t* ids_in, int host, int use_graft, uint16_t* out,
                     cudaStream_t st);
  int block_step(const uint16_t* x, const float* y, float lr, int step, float* loss,
                 uint16_t* out, float* dx_out, cudaStream_t st);
  int activation(int which, int layer, void** ptr, int64_t* numel);
  int lm_head_chunk(int r0, int rows, cudaStream_t st);
  int lm_head_live_chunk(int r0, int rows, cudaStream_t st);
  int load_safetensors(const char* path, cudaStream_t st);  // safetensors_io.cu

  // eval.cu: eval-only / shadow-eval metrics and the model's own shadow bake
  void* eval_mem = nullptr;
  uint64_t* ev_tables = nullptr;
  double* ev_rows = nullptr;
  EvalAccum* ev_acc = nullptr;
  EvalAccum* ev_pinned = nullptr;
  int eval_alloc();
  int eval(const int32_t* ids_in, int64_t n_seq, int host, int use_graft, GltEvalStats* out,
           cudaStream_t st);
  int shadow_bake_self(cudaStream_t st);

  // per-kind kernel timing (GLT_PROF_*)
  bool prof_on = false;
  std::vector<cudaEvent_t> ev_free;
  struct LiveEv { int kind; cudaEvent_t a, b; };
  std::vector<LiveEv> ev_live;
  double prof_ms[GLT_PROF_KINDS] = {};
  int64_t prof_n[GLT_PROF_KINDS] = {};
  int prof_begin(int kind, cudaStream_t st);
  void prof_end(int idx, cudaStream_t st);
  int prof_collect();

  // dp.cu
  int dp_init(const void* unique_id, int rank, int world);
  int dp_allreduce_layers(int l0, int l1);   // layers [l0, l1), after layer_done[l0]
  int dp_bucket = 4;                          // layers per graft-gradient all-reduce
  int dp_reserve_sms = 0;                     // SMs the GEMMs after an all-reduce leave to NCCL
  int dp_reserve_gemms = 1;                   // how many GEMMs after each all-reduce do so
  int dp_async_error(int* nccl_result);
  int dp_abort();
  void dp_shutdown();
};

}  // namespace glt

// Runs `expr` (an int status) inside a Model method with stream `st`, timed
// under profiling kind `kind` when the model's profiling is enabled.
#define GLT_PROF(kind, expr)            \
  do {                                  \
    const int _pb = prof_begin(kind, st); \
    const int _ps = (expr);             \
    prof_end(_pb, st);                  \
    if (_ps != GLT_OK) return _ps;      \
  } while (0)

