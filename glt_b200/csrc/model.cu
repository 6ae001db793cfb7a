// Grafted decoder model: memory layout, forward / backward orchestration,
// loss, clip and AdamW.  Host code is C++; every tensor operation is one of
// this library's sm_100a kernels (tcgen05 GEMMs with fused epilogues, flash
// attention, bandwidth-bound row kernels).
//
// Reference mapping (Hinedes/GLT):
//   forward_layer       src/layer_forward_impl.inc:15-291   -> Model::forward_layer
//   recompute_ffn       src/layer_recompute_impl.inc:8-91   -> fused into the
//                        recompute GEMM of Model::backward_layer
//   backward_layer      src/layer_backward_impl.inc:10-385  -> Model::backward_layer
//   attention_bwd_autograd src/attention_autograd_impl.inc:1-39 -> flash_bwd (saved
//                        q/k/v/o/lse instead of an autograd re-run)
//   forward_model + train loop grafting.hip:224-271, 954-1172 -> Model::train_step
//   allocate_arena       src/arena_impl.inc:14-126           -> Model::allocate
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "kernels_mem.cuh"
#include "mlp_epilogues.cuh"
#include "model.cuh"

namespace glt {

static inline int64_t rup(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// ------------------------------ config -------------------------------------
int config_default(GltModelConfig* c) {
  memset(c, 0, sizeof(*c));
  c->hidden_dim = 2048;
  c->intermediate_dim = 11008;
  c->slice_dim = 2752;
  c->vocab_size = 128256;
  c->num_layers = 36;
  c->num_heads = 16;
  c->num_kv_heads = 4;
  c->head_dim = 0;
  c->max_domains = 4;
  c->domain_id = 0;
  c->layout = GLT_LAYOUT_OVERLAY;
  c->tie_embeddings = 1;
  c->rms_norm_eps = 1e-6f;
  c->lm_loss_scale = 1.0f;
  c->lambda_silence = 5.0f;
  c->rope_theta = 5000000.0f;
  c->graft_layer_start = 0;
  c->graft_layer_end = 35;
  c->graft_proj_gate = 0;
  c->graft_proj_up = 0;
  c->graft_proj_down = 1;
  c->allow_expansion_trap = 0;
  c->adam_beta1 = 0.9f;
  c->adam_beta2 = 0.999f;
  c->adam_eps = 1e-8f;
  c->adam_weight_decay = 0.01f;
  c->gradient_clip_norm = 1.0f;
  c->lr_warmup_steps = 20;
  c->lr_peak = 2e-4f;
  c->no_rope_mask_len = 0;
  return GLT_OK;
}

int config_validate(const GltModelConfig* c, int batch_size, int mode) {
  if (!c) return fail(GLT_EINVAL, "null config");
  if (c->num_heads <= 0) return fail(GLT_EINVAL, "--num-heads must be positive");
  if (c->max_domains <= 0) return fail(GLT_EINVAL, "--max-domains must be positive");
  if (c->hidden_dim <= 0 || c->intermediate_dim <= 0 || c->slice_dim <= 0 || c->num_layers <= 0)
    return fail(GLT_EINVAL, "dimensions must be positive");
  if (c->hidden_dim % c->num_heads != 0)
    return fail(GLT_EINVAL, "hidden-dim (%d) not divisible by num-heads (%d)", c->hidden_dim,
                c->num_heads);
  if (c->hidden_dim % c->max_domains != 0)
    return fail(GLT_EINVAL, "hidden-dim (%d) not divisible by max-domains (%d)", c->hidden_dim,
                c->max_domains);
  if (c->domain_id < 0 || c->domain_id >= c->max_domains)
    return fail(GLT_EINVAL, "--domain-id (%d) out of range [0, %d)", c->domain_id,
                c->max_domains);
  if (c->no_rope_mask_len != 0 && c->no_rope_mask_len != c->num_layers)
    return fail(GLT_EINVAL, "--rope-layer-mask expects %d values, got %d", c->num_layers,
                c->no_rope_mask_len);
  if (c->num_layers > 256 && c->no_rope_mask_len) return fail(GLT_EINVAL, "too many layers");
  if (c->layout == GLT_LAYOUT_OVERLAY && c->intermediate_dim % c->slice_dim != 0)
    return fail(GLT_EINVAL, "intermediate-dim (%d) not divisible by slice-dim (%d)",
                c->intermediate_dim, c->slice_dim);
  if (c->slice_dim % 4 != 0) return fail(GLT_EINVAL, "--slice-dim (%d) must be a multiple of 4", c->slice_dim);
  if (c->intermediate_dim % 8 != 0)
    return fail(GLT_EINVAL, "--intermediate-dim (%d) must be a multiple of 8", c->intermediate_dim);
  for (int f : {c->graft_proj_gate, c->graft_proj_up, c->graft_proj_down})
    if (f != 0 && f != 1) return fail(GLT_EINVAL, "--graft-proj-* flags must be 0 or 1");
  if (!c->graft_proj_gate && !c->graft_proj_up && !c->graft_proj_down)
    return fail(GLT_EINVAL, "no graft projection enabled");
  if (c->graft_proj_gate && c->graft_proj_up && !c->allow_expansion_trap)
    return fail(GLT_EINVAL,
                "gate+up enabled: Expansion Quadratic Trap (pass allow_expansion_trap for an "
                "explicit ablation)");
  if (c->layout != GLT_LAYOUT_OVERLAY && c->layout != GLT_LAYOUT_CONCAT)
    return fail(GLT_EINVAL, "unknown graft layout %d", c->layout);
  if (mode == 0) {
    if (batch_size % 2 != 0) return fail(GLT_EINVAL, "--batch-size must be even");
    if (c->layout == GLT_LAYOUT_OVERLAY) {
      const int H = c->hidden_dim / c->max_domains;
      if ((int64_t)c->domain_id * c->slice_dim + c->slice_dim > c->intermediate_dim)
        return fail(GLT_EINVAL, "domain slice exceeds intermediate_dim");
      if ((int64_t)c->domain_id * H + H > c->hidden_dim)
        return fail(GLT_EINVAL, "domain H-slice exceeds hidden_dim");
    }
  }
  return GLT_OK;
}

float get_lr(const GltModelConfig* c, int step, int total_steps) {
  if (step < c->lr_warmup_steps)
    return c->lr_peak * static_cast<float>(step + 1) / static_cast<float>(c->lr_warmup_steps);
  const float denom = static_cast<float>(total_steps - c->lr_warmup_steps);
  const float progress = static_cast<float>(step - c->lr_warmup_steps) / fmaxf(denom, 1.0f);
  return c->lr_peak * (1.0f + cosf(static_cast<float>(M_PI * progress))) * 0.5f;
}

// ------------------------------ GEMM helpers -------------------------------
namespace {

Operand kmaj(const void* p, int64_t ld) { return Operand{p, ld, false}; }
Operand mnmaj(const void* p, int64_t ld) { return Operand{p, ld, true}; }

// C (bf16) = A.B^T (+R)
int g_bf16(const Operand& A, const Operand& B, int M, int N, int K, uint16_t* C, int64_t ldc,
           const uint16_t* R, int64_t ldr, cudaStream_t st, const Operand* A2 = nullptr,
           int a2_col = 0) {
  const bool vec = aligned16(C) && ldc % 8 == 0 && N % 8 == 0 && (!R || (aligned16(R) && ldr % 8 == 0));
  const int v = vec ? 1 : 0;
  if (N >= 1024 && (!A2 || a2_col % 256 == 0)) {
    EpiBF16<256> e{C, ldc, R, ldr, M, N, v};
    if (A.mn_major) return fail(GLT_EINVAL, "g_bf16: MN-major A unsupported here");
    if (B.mn_major)
      return launch_gemm<256, 4, false, true>(A, B, M, N, K, e, st, 1, A2, a2_col / 256);
    return launch_gemm<256, 4, false, false>(A, B, M, N, K, e, st, 1, A2, a2_col / 256);
  }
  EpiBF16<128> e{C, ldc, R, ldr, M, N, v};
  if (B.mn_major)
    return launch_gemm<128, 6, false, true>(A, B, M, N, K, e, st, 1, A2, a2_col / 128);
  return launch_gemm<128, 6, false, false>(A, B, M, N, K, e, st, 1, A2, a2_col / 128);
}

// C (fp32) = A.B^T  (plain store, K-major A)
int g_f32(const Operand& A, const Operand& B, int M, int N, int K, float* C, int64_t ldc,
          cudaStream_t st) {
  const int v = (aligned16(C) && ldc % 4 == 0 && N % 4 == 0) ? 1 : 0;
  if (N >= 1024) {
    EpiF32<256> e{C, ldc, M, N, 1.f, 0.f, 0, v};
    if (B.mn_major) return launch_gemm<256, 4, false, true>(A, B, M, N, K, e, st);
    return launch_gemm<256, 4, false, false>(A, B, M, N, K, e, st);
  }
  EpiF32<128> e{C, ldc, M, N, 1.f, 0.f, 0, v};
  if (B.mn_major) return launch_gemm<128, 6, false, true>(A, B, M, N, K, e, st);
  return launch_gemm<128, 6, false, false>(A, B, M, N, K, e, st);
}

}  // namespace

// ------------------------------ profiling ----------------------------------
int Model::prof_begin(int kind, cudaStream_t st) {
  if (!prof_on) return -1;
  cudaEvent_t ev[2];
  for (int i = 0; i < 2; ++i) {
    if (!ev_free.empty()) {
      ev[i] = ev_free.back();
      ev_free.pop_back();
    } else if (cudaEventCreate(&ev[i]) != cudaSuccess) {
      return -1;
    }
  }
  cudaEventRecord(ev[0], st);
  ev_live.push_back(LiveEv{kind, ev[0], ev[1]});
  return static_cast<int>(ev_live.size()) - 1;
}

void Model::prof_end(int idx, cudaStream_t st) {
  if (idx >= 0) cudaEventRecord(ev_live[idx].b, st);
}

int Model::prof_collect() {
  for (auto& e : ev_live) {
    GLT_CUDA_TRY(cudaEventSynchronize(e.b));
    float ms = 0.f;
    GLT_CUDA_TRY(cudaEventElapsedTime(&ms, e.a, e.b));
    prof_ms[e.kind] += ms;
    prof_n[e.kind] += 1;
    ev_free.push_back(e.a);
    ev_free.push_back(e.b);
  }
  ev_live.clear();
  return GLT_OK;
}

// ------------------------------ allocation ---------------------------------
Model::~Model() {
  for (auto& e : ev_live) { cudaEventDestroy(e.a); cudaEventDestroy(e.b); }
  for (auto e : ev_free) cudaEventDestroy(e);
  if (own_stream_events) {
    for (auto e : layer_done) cudaEventDestroy(e);
    if (comm_done) cudaEventDestroy(comm_done);
    if (comm_stream) cudaStreamDestroy(comm_stream);
  }
  dp_shutdown();
  if (arena) cudaFree(arena);
  if (graft_mem) cudaFree(graft_mem);
  if (gu_mem) cudaFree(gu_mem);
  if (pinned_stats) cudaFreeHost(pinned_stats);
  for (auto e : stats_ev)
    if (e) cudaEventDestroy(e);
  if (eval_mem) cudaFree(eval_mem);
  if (ev_pinned) cudaFreeHost(ev_pinned);
}

int Model::setup(const GltModelConfig& c, int batch, int seq, int k) {
  cfg = c;
  kind = k;
  GLT_TRY(config_validate(&cfg, batch, 1));
  if (kind == GLT_MODEL_DECODER && batch % 2 != 0) return fail(GLT_EINVAL, "--batch-size must be even");
  overlay = cfg.layout == GLT_LAYOUT_OVERLAY;
  B = batch;
  T = seq;
  M = B * T;
  D = cfg.hidden_dim;
  F = cfg.intermediate_dim;
  S = cfg.slice_dim;
  H = overlay ? D / cfg.max_domains : D;  // concat: the graft spans the full hidden dimension
  V = cfg.vocab_size;
  L = cfg.num_layers;
  nh = cfg.num_heads;
  nkv = cfg.num_kv_heads;
  hd = cfg.head_dim ? cfg.head_dim : D / nh;
  QKV = (nh + 2 * nkv) * hd;
  AD = nh * hd;
  F_pad = static_cast<int>(rup(F, 256));
  S_pad = static_cast<int>(rup(S, 128));
  if (overlay) {
    // i0 = domain_id * S, h0 = domain_id * H (layer_forward_impl.inc:21-22)
    FF = F_pad;
    i0 = cfg.domain_id * S;
    h0 = cfg.domain_id * H;
    if (S % 8 || H % 8)
      return fail(GLT_EINVAL, "overlay geometry needs slice_dim (%d) and hidden_dim/max_domains (%d) "
                  "to be multiples of 8", S, H);
    if (i0 + S > F) return fail(GLT_EINVAL, "domain slice exceeds intermediate_dim");
    if (h0 + H > D) return fail(GLT_EINVAL, "domain H-slice exceeds hidden_dim");
  } else {
    FF = F_pad + S_pad;
    i0 = F_pad;
    h0 = 0;
  }
  if (D % 64) return fail(GLT_EINVAL, "hidden_dim must be a multiple of 64");
  if (kind == GLT_MODEL_DECODER) {
    if (T % 64) return fail(GLT_EINVAL, "seq_len must be a multiple of 64");
    if (hd != 64 && hd != 128) return fail(GLT_EINVAL, "head_dim must be 64 or 128");
    if (nkv <= 0 || nh % nkv) return fail(GLT_EINVAL, "num_heads must be a multiple of num_kv_heads");
    if (V % 8) return fail(GLT_EINVAL, "vocab_size must be a multiple of 8");
  }
  for (int l = 0; l < L; ++l)
    for (int p = 0; p < 3; ++p) {
      const bool on = l >= cfg.graft_layer_start && l <= cfg.graft_layer_end &&
                      (p == 0 ? cfg.graft_proj_gate : p == 1 ? cfg.graft_proj_up : cfg.graft_proj_down);
      enabled.push_back(on ? 1 : 0);
      active_grafts += on ? 1 : 0;
    }
  if (const char* e = getenv("GLT_GEMM_SCHEDULE")) {
    if (strcmp(e, "dynamic") == 0) tile_ctr_on = true;
    else if (strcmp(e, "static") != 0)
      return fail(GLT_EINVAL, "GLT_GEMM_SCHEDULE=%s (static or dynamic)", e);
  }
  if (const char* e = getenv("GLT_MLP_STORE")) {
    const int v = atoi(e);
    if (v < 0 || v > 2) return fail(GLT_EINVAL, "GLT_MLP_STORE=%s (0 recompute, 1 store, 2 auto)", e);
    store_mode = v;
  }
  return allocate();
}

// ---------------------- stored MLP activations -----------------------------
namespace {
// Marks a training forward (whose MLPs write the store) for its scope.
struct SavingScope {
  bool& flag;
  explicit SavingScope(bool& f) : flag(f) { flag = true; }
  ~SavingScope() { flag = false; }
};
}  // namespace

void Model::free_mlp_store() {
  if (gu_mem) cudaFree(gu_mem);
  gu_mem = nullptr;
  gu_bytes = 0;
  for (auto& y : layers) y.gu = nullptr;
}

int Model::alloc_mlp_store(bool required) {
  if (gu_mem) return GLT_OK;
  // gu_block_offset layout: 32-row bands
  const size_t per = static_cast<size_t>(rup(rup(M, 32) * 2 * FF * 2, 256));
  const size_t bytes = per * L;
  if (!required) {
    // auto: store only with room to spare for the caller's own buffers
    size_t fr = 0, tot = 0;
    GLT_CUDA_TRY(cudaMemGetInfo(&fr, &tot));
    const size_t reserve = std::max(static_cast<size_t>(8) << 30, tot / 16);
    if (fr < bytes + reserve) return GLT_OK;
  }
  const cudaError_t e = cudaMalloc(&gu_mem, bytes);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    gu_mem = nullptr;
    if (required)
      return fail(GLT_ENOMEM, "stored MLP activations: cudaMalloc(%zu bytes) failed: %s", bytes,
                  cudaGetErrorString(e));
    return GLT_OK;
  }
  gu_bytes = bytes;
  for (int l = 0; l < L; ++l) layers[l].gu = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(gu_mem) + per * l);
  return GLT_OK;
}

int Model::set_mlp_store(int mode) {
  if (mode < 0 || mode > 2) return fail(GLT_EINVAL, "MLP store mode %d (0 recompute, 1 store, 2 auto)", mode);
  GLT_CUDA_TRY(cudaDeviceSynchronize());   // no step may still read the store
  store_mode = mode;
  store_decided = false;
  if (mode == 0) free_mlp_store();
  if (mode == 1) return ensure_mlp_store();
  return GLT_OK;
}

int Model::ensure_mlp_store() {
  if (store_decided) return GLT_OK;
  store_decided = true;
  if (store_mode == 0) return GLT_OK;
  return alloc_mlp_store(store_mode == 1);
}

int Model::allocate() {
  // ---- graft parameters (outside the arena, like GraftWeights) ----
  graft_numel = static_cast<int64_t>(3) * L * S * H;
  if (!external_acts) {
    const size_t bytes = static_cast<size_t>(graft_numel) * 4 * 4;
    GLT_CUDA_TRY(cudaMalloc(&graft_mem, bytes));
    GLT_CUDA_TRY(cudaMemset(graft_mem, 0, bytes));
    gw = static_cast<float*>(graft_mem);
    grad = gw + graft_numel;
    adam_m = grad + graft_numel;
    adam_v = adam_m + graft_numel;
    graft_bytes = bytes;
  }
  // ---- arena: one allocation carved at 256-byte alignment ----
  struct Req { void** p; size_t bytes; };
  std::vector<Req> reqs;
  auto add = [&](void** p, size_t bytes) { reqs.push_back({p, bytes}); };
  const size_t b2 = 2, b4 = 4;
  layers.resize(L);
  const bool dec = kind == GLT_MODEL_DECODER;
  if (dec) {
    add(reinterpret_cast<void**>(&embed), b2 * V * D);
    if (!cfg.tie_embeddings) add(reinterpret_cast<void**>(&lm_head), b2 * V * D);
    add(reinterpret_cast<void**>(&final_norm), b2 * D);
  }
  for (int l = 0; l < L; ++l) {
    Layer& y = layers[l];
    if (dec) {
      add(reinterpret_cast<void**>(&y.in_norm), b2 * D);
      add(reinterpret_cast<void**>(&y.wqkv), b2 * QKV * D);
      add(reinterpret_cast<void**>(&y.wo), b2 * D * AD);
    }
    add(reinterpret_cast<void**>(&y.post_norm), b2 * D);
    add(reinterpret_cast<void**>(&y.w_gu), b2 * 2 * FF * D);
    add(reinterpret_cast<void**>(&y.w_d), b2 * D * FF);
    if (external_acts) continue;   // saved activations belong to the caller
    // saved activations
    add(reinterpret_cast<void**>(&y.x_post), b2 * M * D);
    add(reinterpret_cast<void**>(&y.x_ffn), b2 * M * D);
    add(reinterpret_cast<void**>(&y.var2), b4 * M);
    if (enabled[3 * l + 2]) add(reinterpret_cast<void**>(&y.dd), b2 * M * H);
    if (dec) {
      add(reinterpret_cast<void**>(&y.var1), b4 * M);
      add(reinterpret_cast<void**>(&y.qkv), b2 * M * QKV);
      add(reinterpret_cast<void**>(&y.o), b2 * M * AD);
      add(reinterpret_cast<void**>(&y.lse), b4 * B * nh * T);
    }
  }
  if (!external_acts) {
    add(reinterpret_cast<void**>(&esq_all), b4 * 3 * static_cast<size_t>(L) * M);
    xs.resize(L + 1);
    for (int l = 0; l <= L; ++l) add(reinterpret_cast<void**>(&xs[l]), b2 * M * D);
  }
  add(reinterpret_cast<void**>(&h), b2 * M * FF);
  add(reinterpret_cast<void**>(&dx), b4 * M * D);
  add(reinterpret_cast<void**>(&dtmp), b4 * M * D);
  add(reinterpret_cast<void**>(&dy_b), b2 * M * D);
  add(reinterpret_cast<void**>(&dyg_b), b2 * M * D);
  add(reinterpret_cast<void**>(&dh), b2 * M * FF);
  add(reinterpret_cast<void**>(&dgu), b2 * M * 2 * FF);
  add(reinterpret_cast<void**>(&hg), b2 * M * S_pad);
  if (overlay) {
    add(reinterpret_cast<void**>(&gwb), b2 * static_cast<size_t>(graft_numel));
    add(reinterpret_cast<void**>(&dlt), b4 * M * 2 * static_cast<size_t>(S));
    add(reinterpret_cast<void**>(&dys), b2 * M * 2 * static_cast<size_t>(S));
  }
  add(reinterpret_cast<void**>(&stats), sizeof(DevStats));
  add(reinterpret_cast<void**>(&d_err), sizeof(unsigned int));   // zeroed with the arena
  add(reinterpret_cast<void**>(&tile_ctr), 2 * sizeof(int));   // zeroed with the arena
  add(reinterpret_cast<void**>(&d_enabled), sizeof(int) * 3 * L);
  add(reinterpret_cast<void**>(&d_gu_ptrs), sizeof(void*) * L);
  add(reinterpret_cast<void**>(&d_wd_ptrs), sizeof(void*) * L);
  add(reinterpret_cast<void**>(&ids), b4 * M);
  add(reinterpret_cast<void**>(&ood), b4 * M);
  if (dec) {
    add(reinterpret_cast<void**>(&xn), b2 * M * D);
    add(reinterpret_cast<void**>(&dqkv), b2 * M * QKV);
    add(reinterpret_cast<void**>(&dout_b), b2 * M * AD);
    // fp32 dQ accumulator; with head_dim 64 also the dK/dV accumulators of
    // the tcgen05 backward (flash_bwd_tc64)
    add(reinterpret_cast<void**>(&dq_acc), b4 * M * (AD + (hd == 64 ? 2 * nkv * hd : 0)));
    add(reinterpret_cast<void**>(&dsum), b4 * B * nh * T);
    add(reinterpret_cast<void**>(&xf), b2 * M * D);
    add(reinterpret_cast<void**>(&varf), b4 * M);
    ce_rows = std::min(M, 8192);
    add(reinterpret_cast<void**>(&logits), b2 * static_cast<size_t>(ce_rows) * V);
    add(reinterpret_cast<void**>(&lm_rows), b4 * M);
    add(reinterpret_cast<void**>(&n_lm_rows), b4);
    add(reinterpret_cast<void**>(&cos_t), b4 * T * (hd / 2));
    add(reinterpret_cast<void**>(&sin_t), b4 * T * (hd / 2));
  } else {
    add(reinterpret_cast<void**>(&var_in), b4 * M);
  }
  size_t total = 0;
  for (auto& r : reqs) total += rup(static_cast<int64_t>(r.bytes), 256);
  arena_bytes = total;
  cudaError_t e = cudaMalloc(&arena, total);
  if (e != cudaSuccess)
    return fail(GLT_ENOMEM, "arena cudaMalloc(%zu bytes) failed: %s", total, cudaGetErrorString(e));
  GLT_CUDA_TRY(cudaMemset(arena, 0, total));
  size_t off = 0;
  for (auto& r : reqs) {
    *r.p = static_cast<uint8_t*>(arena) + off;
    off += rup(static_cast<int64_t>(r.bytes), 256);
  }
  if (dec && cfg.tie_embeddings) lm_head = embed;
  if (esq_all)
    for (int l = 0; l < L; ++l) layers[l].esq = esq_all + static_cast<int64_t>(3) * M * l;
  // device-side tables
  GLT_CUDA_TRY(cudaMemcpy(d_enabled, enabled.data(), sizeof(int) * 3 * L, cudaMemcpyHostToDevice));
  std::vector<uint16_t*> gup(L), wdp(L);
  for (int l = 0; l < L; ++l) { gup[l] = layers[l].w_gu; wdp[l] = layers[l].w_d; }
  GLT_CUDA_TRY(cudaMemcpy(d_gu_ptrs, gup.data(), sizeof(void*) * L, cudaMemcpyHostToDevice));
  GLT_CUDA_TRY(cudaMemcpy(d_wd_ptrs, wdp.data(), sizeof(void*) * L, cudaMemcpyHostToDevice));
  if (dec) {
    const int half = hd / 2;
    std::vector<float> c(static_cast<size_t>(T) * half), s(static_cast<size_t>(T) * half);
    for (int i = 0; i < half; ++i) {
      // rope_impl.inc:13-19: inv_freq = 1 / theta^(2i/hd), angle = pos * inv_freq (fp32)
      const float inv = 1.0f / powf(cfg.rope_theta, static_cast<float>(2 * i) / static_cast<float>(hd));
      for (int p = 0; p < T; ++p) {
        const float a = static_cast<float>(p) * inv;
        c[static_cast<size_t>(p) * half + i] = cosf(a);
        s[static_cast<size_t>(p) * half + i] = sinf(a);
      }
    }
    GLT_CUDA_TRY(cudaMemcpy(cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    GLT_CUDA_TRY(cudaMemcpy(sin_t, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  }
  GLT_CUDA_TRY(cudaMallocHost(&pinned_stats, 2 * sizeof(DevStats)));
  for (auto& e : stats_ev) GLT_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  GLT_CUDA_TRY(cudaStreamCreateWithFlags(&comm_stream, cudaStreamNonBlocking));
  layer_done.resize(L);
  for (int l = 0; l < L; ++l) GLT_CUDA_TRY(cudaEventCreateWithFlags(&layer_done[l], cudaEventDisableTiming));
  GLT_CUDA_TRY(cudaEventCreateWithFlags(&comm_done, cudaEventDisableTiming));
  own_stream_events = true;
  return GLT_OK;
}

MirrorTargets Model::mirror() const {
  MirrorTargets mt;
  mt.plain = overlay ? gwb : nullptr;
  mt.w_gu = d_gu_ptrs;
  mt.w_d = d_wd_ptrs;
  mt.f_pad = F_pad;
  mt.ffn = FF;
  mt.D = D;
  mt.layer_begin = cfg.graft_layer_start;
  mt.layer_end = cfg.graft_layer_end;
  mt.kinds[0] = cfg.graft_proj_gate;
  mt.kinds[1] = cfg.graft_proj_up;
  mt.kinds[2] = cfg.graft_proj_down;
  return mt;
}

// ------------------------------ weights ------------------------------------
int Model::set_weight(int layer, int which, const void* src, int64_t numel, int host,
                      cudaStream_t st) {
  const cudaMemcpyKind kindc = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  auto expect = [&](int64_t n) -> int {
    if (numel != n) return fail(GLT_EINVAL, "weight %d: numel %lld != expected %lld", which,
                                (long long)numel, (long long)n);
    return GLT_OK;
  };
  const bool dec = kind == GLT_MODEL_DECODER;
  if (layer < 0) {
    if (!dec) return fail(GLT_EINVAL, "model-level weights need the decoder model");
    if (which == GLT_W_EMBED || (which == GLT_W_LM_HEAD && cfg.tie_embeddings)) {
      GLT_TRY(expect(static_cast<int64_t>(V) * D));
      GLT_CUDA_TRY(cudaMemcpyAsync(embed, src, numel * 2, kindc, st));
    } else if (which == GLT_W_LM_HEAD) {
      GLT_TRY(expect(static_cast<int64_t>(V) * D));
      GLT_CUDA_TRY(cudaMemcpyAsync(lm_head, src, numel * 2, kindc, st));
    } else if (which == GLT_W_FINAL_NORM) {
      GLT_TRY(expect(D));
      GLT_CUDA_TRY(cudaMemcpyAsync(final_norm, src, numel * 2, kindc, st));
    } else {
      return fail(GLT_EINVAL, "weight kind %d is per-layer", which);
    }
    return GLT_OK;
  }
  if (layer >= L) return fail(GLT_EINVAL, "layer %d out of range", layer);
  Layer& y = layers[layer];
  const char* s8 = static_cast<const char*>(src);
  switch (which) {
    case GLT_W_IN_NORM:
      if (!dec) return fail(GLT_EINVAL, "no attention in the MLP-block model");
      GLT_TRY(expect(D));
      GLT_CUDA_TRY(cudaMemcpyAsync(y.in_norm, src, numel * 2, kindc, st));
      break;
    case GLT_W_POST_NORM:
      GLT_TRY(expect(D));
      GLT_CUDA_TRY(cudaMemcpyAsync(y.post_norm, src, numel * 2, kindc, st));
      break;
    case GLT_W_Q:
    case GLT_W_K:
    case GLT_W_V: {
      if (!dec) return fail(GLT_EINVAL, "no attention in the MLP-block model");
      const int rows = which == GLT_W_Q ? AD : nkv * hd;
      const int r0 = which == GLT_W_Q ? 0 : which == GLT_W_K ? AD : AD + nkv * hd;
      GLT_TRY(expect(static_cast<int64_t>(rows) * D));
      GLT_CUDA_TRY(cudaMemcpyAsync(y.wqkv + static_cast<int64_t>(r0) * D, src, numel * 2, kindc, st));
      break;
    }
    case GLT_W_O:
      if (!dec) return fail(GLT_EINVAL, "no attention in the MLP-block model");
      GLT_TRY(expect(static_cast<int64_t>(D) * AD));
      GLT_CUDA_TRY(cudaMemcpyAsync(y.wo, src, numel * 2, kindc, st));
      break;
    case GLT_W_GATE:
    case GLT_W_UP: {
      GLT_TRY(expect(static_cast<int64_t>(F) * D));
      const int add = which == GLT_W_UP ? 128 : 0;
      for (int b = 0; b * 128 < F; ++b) {
        const int rows = std::min(128, F - b * 128);
        GLT_CUDA_TRY(cudaMemcpyAsync(y.w_gu + (static_cast<int64_t>(256) * b + add) * D,
                                     s8 + static_cast<int64_t>(b) * 128 * D * 2,
                                     static_cast<size_t>(rows) * D * 2, kindc, st));
      }
      break;
    }
    case GLT_W_DOWN:
      GLT_TRY(expect(static_cast<int64_t>(D) * F));
      GLT_CUDA_TRY(cudaMemcpy2DAsync(y.w_d, static_cast<size_t>(FF) * 2, src,
                                     static_cast<size_t>(F) * 2, static_cast<size_t>(F) * 2, D,
                                     kindc, st));
      break;
    default:
      return fail(GLT_EINVAL, "unknown weight kind %d", which);
  }
  return GLT_OK;
}

int Model::init_random(uint64_t seed, float std, float graft_std, float graft_down_std) {
  cudaStream_t st = 0;
  const bool dec = kind == GLT_MODEL_DECODER;
  uint64_t k = seed * 1000003ull + 17;
  if (dec) {
    GLT_TRY(init_normal_bf16(embed, static_cast<int64_t>(V) * D, k++, std, st));
    if (!cfg.tie_embeddings) GLT_TRY(init_normal_bf16(lm_head, static_cast<int64_t>(V) * D, k++, std, st));
    GLT_TRY(fill_bf16(final_norm, D, 1.f, st));
  }
  // base gate/up/down are drawn into a scratch copy in HF shapes then packed,
  // so the padding and graft regions of the fused weights stay exact.
  uint16_t* tmp = dgu;  // scratch large enough for [F, D] (M*2FF >= F*D is checked)
  if (static_cast<int64_t>(M) * 2 * FF < static_cast<int64_t>(F) * D)
    return fail(GLT_EINVAL, "init_random: scratch too small");
  for (int l = 0; l < L; ++l) {
    Layer& y = layers[l];
    if (dec) {
      GLT_TRY(fill_bf16(y.in_norm, D, 1.f, st));
      GLT_TRY(init_normal_bf16(y.wqkv, static_cast<int64_t>(QKV) * D, k++, std, st));
      GLT_TRY(init_normal_bf16(y.wo, static_cast<int64_t>(D) * AD, k++, std, st));
    }
    GLT_TRY(fill_bf16(y.post_norm, D, 1.f, st));
    GLT_CUDA_TRY(cudaMemsetAsync(y.w_gu, 0, static_cast<size_t>(2) * FF * D * 2, st));
    GLT_CUDA_TRY(cudaMemsetAsync(y.w_d, 0, static_cast<size_t>(D) * FF * 2, st));
    for (int which : {GLT_W_GATE, GLT_W_UP, GLT_W_DOWN}) {
      GLT_TRY(init_normal_bf16(tmp, static_cast<int64_t>(F) * D, k++, std, st));
      GLT_TRY(set_weight(l, which, tmp, static_cast<int64_t>(F) * D, 0, st));
    }
  }
  // graft: gate/up N(0, graft_std), down N(0, graft_down_std)
  if (!gw) return fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  const int64_t SH = static_cast<int64_t>(S) * H;
  GLT_CUDA_TRY(cudaMemsetAsync(gw, 0, graft_numel * 4, st));
  for (int l = 0; l < L; ++l)
    for (int p = 0; p < 3; ++p) {
      const float sd = p == 2 ? graft_down_std : graft_std;
      if (sd != 0.f) GLT_TRY(init_normal_f32(gw + (3 * l + p) * SH, SH, k++, sd, st));
    }
  GLT_CUDA_TRY(cudaMemsetAsync(adam_m, 0, graft_numel * 4, st));
  GLT_CUDA_TRY(cudaMemsetAsync(adam_v, 0, graft_numel * 4, st));
  GLT_TRY(refresh_graft(st));
  GLT_CUDA_TRY(cudaStreamSynchronize(st));
  return GLT_OK;
}

int Model::refresh_graft(cudaStream_t st) {
  if (!gw) return fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  return refresh_mirror(gw, L, S, H, mirror(), st);
}

// ------------------------------ forward ------------------------------------
bool Model::rope_on(int l) const {
  return cfg.no_rope_mask_len == 0 || cfg.no_rope_mask[l] != 0;
}

int Model::ffn_forward(int l, const uint16_t* x_in, uint16_t* x_out, float* var_out,
                       bool use_graft, cudaStream_t st) {
  if (overlay) return ffn_forward_overlay(l, x_in, x_out, var_out, use_graft, st);
  Layer& y = layers[l];
  const bool any = enabled[3 * l] || enabled[3 * l + 1] || enabled[3 * l + 2];
  const bool grafted = use_graft && any;
  // Non-grafted layers skip the graft columns; after a shadow bake they are
  // base columns and stay in the GEMMs (without the graft-side energies).
  const int ff = (grafted || (shadow_baked && any)) ? FF : F_pad;
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_fwd(x_in, y.post_norm, y.x_ffn, var_out, M, D, cfg.rms_norm_eps, st));
  // gate/up + SwiGLU (+ graft energies)
  {
    EpiSwiGLUFwd e{h, FF, M, F_pad, F_pad + S,
                   (grafted && enabled[3 * l]) ? y.esq : nullptr,
                   (grafted && enabled[3 * l + 1]) ? y.esq + M : nullptr,
                   saving ? y.gu : nullptr, 2 * static_cast<int64_t>(FF) / 8};
    GLT_PROF(GLT_PROF_GATE_UP_FWD,
             (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * ff, D, e, st)));
  }
  // down + residual
  GLT_PROF(GLT_PROF_DOWN_FWD, g_bf16(kmaj(h, FF), kmaj(y.w_d, FF), M, D, ff, x_out, D, x_in, D, st));
  // delta_down = h_graft . Delta_down (energy + saved copy for the silence gradient)
  if (grafted && enabled[3 * l + 2]) {
    if (D >= 1024) {
      EpiDeltaDown<256> e{y.dd, D, y.esq + 2 * static_cast<int64_t>(M), M, D};
      GLT_PROF(GLT_PROF_DELTA_DOWN, (launch_gemm<256, 4, false, false>(kmaj(h + F_pad, FF), kmaj(y.w_d + F_pad, FF), M, D, S, e, st)));
    } else {
      EpiDeltaDown<128> e{y.dd, D, y.esq + 2 * static_cast<int64_t>(M), M, D};
      GLT_PROF(GLT_PROF_DELTA_DOWN, (launch_gemm<128, 6, false, false>(kmaj(h + F_pad, FF), kmaj(y.w_d + F_pad, FF), M, D, S, e, st)));
    }
  }
  return GLT_OK;
}

// recompute_ffn (layer_recompute_impl.inc:8-91): the gate/up GEMM of layer l
// from its saved x_ffn, with the graft deltas injected, writing only the
// bf16 gate_pre/up store (layers[l].gu) that the fused backward reads.
int Model::ffn_recompute(int l, cudaStream_t st) {
  Layer& y = layers[l];
  if (!y.gu || !y.x_ffn) return fail(GLT_EINVAL, "recompute: no store or no x_ffn for layer %d", l);
  const bool g = enabled[3 * l], u = enabled[3 * l + 1];
  const bool grafted = g || u || enabled[3 * l + 2];
  if (overlay) {
    if (g || u) GLT_TRY(expand_deltas(l, g, u, nullptr, nullptr, st));
    EpiSwiGLUFwdOv e{h, FF, M, g ? dlt : nullptr, u ? dlt + S : nullptr, 2 * static_cast<int64_t>(S),
                     i0, i0 + S, y.gu, 2 * static_cast<int64_t>(FF) / 8};
    GLT_PROF(GLT_PROF_RECOMPUTE,
             (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * FF, D, e, st)));
    return GLT_OK;
  }
  const int ff = grafted ? FF : F_pad;
  EpiSwiGLUFwd e{h, FF, M, F_pad, F_pad + S, nullptr, nullptr, y.gu, 2 * static_cast<int64_t>(FF) / 8};
  GLT_PROF(GLT_PROF_RECOMPUTE,
           (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * ff, D, e, st)));
  return GLT_OK;
}

int Model::forward_layer(int l, bool use_graft, cudaStream_t st) {
  Layer& y = layers[l];
  AttnShape as{B, T, nh, nkv, hd, QKV, AD, 1.0f / sqrtf(static_cast<float>(hd))};
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_fwd(xs[l], y.in_norm, xn, y.var1, M, D, cfg.rms_norm_eps, st));
  if (rope_on(l)) {
    // RoPE on q and k in the QKV GEMM's epilogue (no extra pass over qkv)
    EpiBF16Rope<256> e{y.qkv, QKV, M, QKV, (nh + nkv) * hd, T, hd, cos_t, sin_t};
    GLT_PROF(GLT_PROF_QKV, (launch_gemm<256, 4, false, false>(kmaj(xn, D), kmaj(y.wqkv, D), M, QKV, D, e, st)));
  } else {
    GLT_PROF(GLT_PROF_QKV, g_bf16(kmaj(xn, D), kmaj(y.wqkv, D), M, QKV, D, y.qkv, QKV, nullptr, 0, st));
  }
  // tcgen05/TMEM kernel for 128-token tiles; the mma.sync kernel covers seq_len % 128 != 0
  if (T % 128 == 0)
    GLT_PROF(GLT_PROF_ATTN_FWD, flash_fwd_tc(y.qkv, y.o, y.lse, as, st));
  else
    GLT_PROF(GLT_PROF_ATTN_FWD, flash_fwd(y.qkv, y.o, y.lse, as, st));
  GLT_PROF(GLT_PROF_OPROJ, g_bf16(kmaj(y.o, AD), kmaj(y.wo, AD), M, D, AD, y.x_post, D, xs[l], D, st));
  return ffn_forward(l, y.x_post, xs[l + 1], y.var2, use_graft, st);
}

// ------------------------------ backward -----------------------------------
// dx (fp32, grad wrt the FFN output / residual stream) -> dtmp = grad wrt x_ffn;
// graft weight grads accumulated into `grad`.
int Model::ffn_backward(int l, cudaStream_t st) {
  if (overlay) return ffn_backward_overlay(l, st);
  Layer& y = layers[l];
  const bool gate = enabled[3 * l], up = enabled[3 * l + 1], down = enabled[3 * l + 2];
  const bool grafted = gate || up || down;
  const int ff = grafted ? FF : F_pad;
  const int64_t SH = static_cast<int64_t>(S) * H;
  // dy = bf16(dx); dyg = bf16(dx + silence_down)
  GLT_TRY(silence_down_prep(dx, down ? y.dd : nullptr, D, y.esq + 2 * static_cast<int64_t>(M), ood,
                            stats, dy_b, dyg_b, D, M, D, 0, D, st));
  if (y.gu) {
    // dh = [dy | dyg] . W_d with SwiGLU's backward in its epilogue, from the
    // gate_pre/up the forward stored -> dgu (+ graft h for the down grad)
    Operand a2 = kmaj(dyg_b, D);
    const int64_t ld2 = 2 * static_cast<int64_t>(FF);
    if (ff >= 1024) {
      EpiSwiGLUBwdStored<256> e{y.gu, ld2 / 8, dgu, ld2, down ? hg : nullptr, S_pad, M, ff, F_pad, F_pad + S, S,
                                gate ? y.esq : nullptr, up ? y.esq + M : nullptr, ood, stats};
      GLT_PROF(GLT_PROF_DH, (launch_gemm<256, 4, false, true>(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, ff, D, e, st,
                                                               1, &a2, F_pad / 256)));
    } else {
      EpiSwiGLUBwdStored<128> e{y.gu, ld2 / 8, dgu, ld2, down ? hg : nullptr, S_pad, M, ff, F_pad, F_pad + S, S,
                                gate ? y.esq : nullptr, up ? y.esq + M : nullptr, ood, stats};
      GLT_PROF(GLT_PROF_DH, (launch_gemm<128, 6, false, true>(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, ff, D, e, st,
                                                               1, &a2, F_pad / 128)));
    }
  } else {
    // dh = [dy | dyg] . W_d   (graft columns read the silence-blended gradient)
    {
      Operand a2 = kmaj(dyg_b, D);
      GLT_PROF(GLT_PROF_DH, g_bf16(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, ff, D, dh, FF, nullptr, 0, st, &a2, F_pad));
    }
    // recompute gate/up and SwiGLU backward -> dgu (+ graft h for the down grad)
    EpiSwiGLUBwd e{dh, FF, dgu, 2 * static_cast<int64_t>(FF), down ? hg : nullptr, S_pad, M,
                   F_pad, F_pad + S, S, gate ? y.esq : nullptr, up ? y.esq + M : nullptr, ood,
                   stats};
    GLT_PROF(GLT_PROF_RECOMPUTE,
             (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * ff, D, e, st)));
  }
  // graft weight gradients (K = tokens, split-K with atomic accumulation).
  // 128x256 tiles: at the config-3 shapes they ran 1.5x faster than 128x128
  // (half the L2 operand traffic per FLOP), with splits for ~1.5 waves.
  if (down) {
    const int sp = pick_k_splits(S, D, M, 256, 3);
    EpiF32<256> e{grad + (3 * l + 2) * SH, H, S, D, 1.f, 0.f, 1, 1};
    GLT_PROF(GLT_PROF_WGRAD_DOWN, (launch_gemm<256, 4, true, true>(mnmaj(hg, S_pad), mnmaj(dyg_b, D), S, D, M, e, st, sp)));
  }
  if (gate || up) {
    const int rows = 2 * S_pad;
    const int sp = pick_k_splits(rows, D, M, 256, 3);
    EpiGradGateUp<256> e{gate ? grad + (3 * l) * SH : nullptr, up ? grad + (3 * l + 1) * SH : nullptr,
                         H, S, D};
    GLT_PROF(GLT_PROF_WGRAD_GATE_UP,
             (launch_gemm<256, 4, true, true>(mnmaj(dgu + 2 * static_cast<int64_t>(F_pad), 2 * static_cast<int64_t>(FF)),
                                              mnmaj(y.x_ffn, D), rows, D, M, e, st, sp)));
  }
  // input grad through the fused gate/up weights
  GLT_PROF(GLT_PROF_DX_GATE_UP, g_f32(kmaj(dgu, 2 * static_cast<int64_t>(FF)), mnmaj(y.w_gu, D), M, D, 2 * ff, dtmp, D, st));
  return GLT_OK;
}

int Model::backward_layer(int l, cudaStream_t st) {
  Layer& y = layers[l];
  AttnShape as{B, T, nh, nkv, hd, QKV, AD, 1.0f / sqrtf(static_cast<float>(hd))};
  GLT_TRY(ffn_backward(l, st));
  if (dp_world > 1 && l % dp_bucket == 0) {
    // graft grads of layers [l, l + dp_bucket) are final (layers run L-1 .. 0)
    GLT_CUDA_TRY(cudaEventRecord(layer_done[l], st));
    GLT_TRY(dp_allreduce_layers(l, std::min(L, l + dp_bucket)));
    gemm_sm_reserve() = SmReserve{dp_reserve_sms, dp_reserve_gemms};
  }
  // post-attention RMSNorm backward + residual: dx = grad wrt x_post
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_bwd(dtmp, y.x_post, y.post_norm, y.var2, dx, dx, dy_b, M, D, cfg.rms_norm_eps, st));
  // attention: do = dx_post . Wo ; flash backward ; RoPE^T ; dxn = dqkv . Wqkv
  if (T % 128 == 0 && (hd == 128 || hd == 64)) {
    // tcgen05 backward: dsum from the dO GEMM's epilogue; the inverse RoPE of
    // dq (and, head_dim 64, of dk) in the fp32 -> bf16 conversion, that of dk
    // at head_dim 128 in rope_apply
    EpiBF16Dsum<256> e{dout_b, AD, M, AD, y.o, AD, dsum, T, nh, hd};
    GLT_PROF(GLT_PROF_DO, (launch_gemm<256, 4, false, true>(kmaj(dy_b, D), mnmaj(y.wo, AD), M, AD, D, e, st)));
    const bool rope = rope_on(l);
    if (hd == 64) {
      GLT_PROF(GLT_PROF_ATTN_BWD, flash_bwd_tc64(y.qkv, y.o, dout_b, y.lse, dqkv, dq_acc, dsum, as, st, true,
                                                 rope ? cos_t : nullptr, rope ? sin_t : nullptr));
    } else {
      GLT_PROF(GLT_PROF_ATTN_BWD, flash_bwd_tc(y.qkv, y.o, dout_b, y.lse, dqkv, dq_acc, dsum, as, st, true,
                                               rope ? cos_t : nullptr, rope ? sin_t : nullptr));
      if (rope) GLT_PROF(GLT_PROF_ROPE, rope_apply(dqkv, as, cos_t, sin_t, 1, 0, 1, st));
    }
  } else {
    GLT_PROF(GLT_PROF_DO, g_bf16(kmaj(dy_b, D), mnmaj(y.wo, AD), M, AD, D, dout_b, AD, nullptr, 0, st));
    GLT_PROF(GLT_PROF_ATTN_BWD, flash_bwd(y.qkv, y.o, dout_b, y.lse, dqkv, dq_acc, dsum, as, st));
    if (rope_on(l)) GLT_PROF(GLT_PROF_ROPE, rope_apply(dqkv, as, cos_t, sin_t, 1, 1, 1, st));
  }
  GLT_PROF(GLT_PROF_DX_QKV, g_f32(kmaj(dqkv, QKV), mnmaj(y.wqkv, D), M, D, QKV, dtmp, D, st));
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_bwd(dtmp, xs[l], y.in_norm, y.var1, dx, dx, nullptr, M, D, cfg.rms_norm_eps, st));
  return GLT_OK;
}

// ------------------------------ steps --------------------------------------
int Model::load_inputs(const int32_t* ids_in, const int32_t* ood_in, int host, cudaStream_t st) {
  const cudaMemcpyKind k = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  GLT_CUDA_TRY(cudaMemcpyAsync(ids, ids_in, sizeof(int32_t) * M, k, st));
  if (ood_in) GLT_CUDA_TRY(cudaMemcpyAsync(ood, ood_in, sizeof(int32_t) * M, k, st));
  else GLT_CUDA_TRY(cudaMemsetAsync(ood, 0, sizeof(int32_t) * M, st));
  return GLT_OK;
}

int Model::forward_all(bool use_graft, cudaStream_t st) {
  GLT_TRY(embedding_fwd(ids, embed, xs[0], M, D, V, st));
  for (int l = 0; l < L; ++l) GLT_TRY(forward_layer(l, use_graft, st));
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_fwd(xs[L], final_norm, xf, varf, M, D, cfg.rms_norm_eps, st));
  return GLT_OK;
}

int Model::train_step(const int32_t* ids_in, const int32_t* ood_in, int host, int step,
                      int total_steps, GltStepStats* out, cudaStream_t st) {
  ScopedTileCounter tile_claims(gemm_counter());
  ScopedSmReserveReset sm_reserve_reset;
  if (kind != GLT_MODEL_DECODER) return fail(GLT_ESTATE, "train_step needs the decoder model");
  if (shadow_baked) return fail(GLT_ESTATE, "backward on a shadow-baked model is forbidden");
  GLT_TRY(load_inputs(ids_in, ood_in, host, st));
  GLT_CUDA_TRY(cudaMemsetAsync(stats, 0, sizeof(DevStats), st));
  GLT_CUDA_TRY(cudaMemsetAsync(grad, 0, graft_numel * 4, st));
  GLT_CUDA_TRY(cudaMemsetAsync(esq_all, 0, sizeof(float) * 3 * static_cast<size_t>(L) * M, st));
  GLT_TRY(count_tokens(ood, B, T, stats, st));
  GLT_TRY(ensure_mlp_store());
  {
    SavingScope sv(saving);
    GLT_TRY(forward_all(true, st));
  }
  // LM head + cross-entropy + dlogits . E over the rows that carry LM loss
  // only: a position whose label is OOD (or that has no label) contributes
  // nothing to the loss, and its logit gradient is zero (cross_entropy's
  // mask), so its logits are never computed.  The live rows are compacted on
  // the device (the final-norm rows gathered into xn, free after the
  // forward); the two GEMMs read the row count from device memory, and the
  // dx GEMM scatters back into the zeroed dtmp.  Same values as computing
  // every row; about half the LM-head work in the reference's batch layout.
  GLT_TRY(live_rows(ood, M, T, lm_rows, n_lm_rows, st));
  GLT_TRY(gather_rows(xf, xn, lm_rows, n_lm_rows, M, D, st));
  GLT_CUDA_TRY(cudaMemsetAsync(dtmp, 0, sizeof(float) * static_cast<size_t>(M) * D, st));
  for (int r0 = 0; r0 < M; r0 += ce_rows) {
    const int rows = std::min(ce_rows, M - r0);
    GLT_TRY(lm_head_live_chunk(r0, rows, st));
    GLT_PROF(GLT_PROF_CE, cross_entropy_chunk(logits, V, rows, r0, V, ids, ood, T, cfg.lm_loss_scale,
                                              stats, st, lm_rows, n_lm_rows));
    if (D >= 1024) {
      EpiF32Rows<256> e{dtmp, D, lm_rows + r0, n_lm_rows, r0, D};
      GLT_PROF(GLT_PROF_LM_DX, (launch_gemm<256, 4, false, true>(kmaj(logits, V), mnmaj(lm_head, D), rows, D, V,
                                                                   e, st, 1, nullptr, INT_MAX, 32, n_lm_rows, r0)));
    } else {
      EpiF32Rows<128> e{dtmp, D, lm_rows + r0, n_lm_rows, r0, D};
      GLT_PROF(GLT_PROF_LM_DX, (launch_gemm<128, 6, false, true>(kmaj(logits, V), mnmaj(lm_head, D), rows, D, V,
                                                                   e, st, 1, nullptr, INT_MAX, 32, n_lm_rows, r0)));
    }
  }
  GLT_TRY(silence_stats(esq_all, d_enabled, L, M, S, H, ood, stats, st));
  GLT_TRY(finalize_loss(stats, cfg.lambda_silence, active_grafts, cfg.lm_loss_scale, st));
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_bwd(dtmp, xs[L], final_norm, varf, nullptr, dx, nullptr, M, D, cfg.rms_norm_eps, st));
  for (int l = L - 1; l >= 0; --l) GLT_TRY(backward_layer(l, st));
  return finish_step(step, total_steps, out, st);
}

// logits[0:rows] = gathered live rows [r0, r0+rows) . lm_head^T (bf16); the
// GEMM runs min(rows, n_live - r0) rows, n_live read on the device.
int Model::lm_head_live_chunk(int r0, int rows, cudaStream_t st) {
  const bool vec = V % 8 == 0;
  if (V >= 1024) {
    EpiBF16<256> e{logits, V, nullptr, 0, rows, V, vec ? 1 : 0};
    GLT_PROF(GLT_PROF_LM_HEAD, (launch_gemm<256, 4, false, false>(kmaj(xn + static_cast<int64_t>(r0) * D, D),
                                                                    kmaj(lm_head, D), rows, V, D, e, st, 1, nullptr,
                                                                    INT_MAX, 32, n_lm_rows, r0)));
  } else {
    EpiBF16<128> e{logits, V, nullptr, 0, rows, V, vec ? 1 : 0};
    GLT_PROF(GLT_PROF_LM_HEAD, (launch_gemm<128, 6, false, false>(kmaj(xn + static_cast<int64_t>(r0) * D, D),
                                                                    kmaj(lm_head, D), rows, V, D, e, st, 1, nullptr,
                                                                    INT_MAX, 32, n_lm_rows, r0)));
  }
  return GLT_OK;
}

// logits[0:rows] = final-norm rows [r0, r0+rows) . lm_head^T (bf16)
int Model::lm_head_chunk(int r0, int rows, cudaStream_t st) {
  GLT_PROF(GLT_PROF_LM_HEAD, g_bf16(kmaj(xf + static_cast<int64_t>(r0) * D, D), kmaj(lm_head, D), rows, V,
                                    D, logits, V, nullptr, 0, st));
  return GLT_OK;
}

int Model::finish_step(int step, int total_steps, GltStepStats* out, cudaStream_t st) {
  if (dp_world > 1) {
    GLT_CUDA_TRY(cudaEventRecord(comm_done, comm_stream));
    GLT_CUDA_TRY(cudaStreamWaitEvent(st, comm_done, 0));
  }
  // DP: the all-reduce summed the ranks' grads; 1/world turns the sum into the mean.
  GLT_PROF(GLT_PROF_ADAMW, grad_clip_scale(grad, graft_numel, cfg.gradient_clip_norm, 1.0f / dp_world, stats, st));
  const float lr = get_lr(&cfg, step, total_steps);
  last_lr = lr;
  const int kinds[3] = {cfg.graft_proj_gate, cfg.graft_proj_up, cfg.graft_proj_down};
  MirrorTargets mt = mirror();
  GLT_PROF(GLT_PROF_ADAMW, adamw_step(gw, grad, adam_m, adam_v, L, S, H, lr, cfg.adam_beta1, cfg.adam_beta2,
                     cfg.adam_eps, cfg.adam_weight_decay, step, kinds, stats, &mt, st));
  // The step's stats go to a pinned slot without a host sync; the next step
  // overwrites the device copy, two steps later the slot is reused.  The
  // device error word travels with them (any kernel of this step, or of an
  // earlier forward, that gave up a bounded wait).
  GLT_TRY(collect_device_error(device_error_word(), d_err, &stats->dev_err, st));
  const int slot = step & 1;
  GLT_CUDA_TRY(cudaMemcpyAsync(pinned_stats + slot, stats, sizeof(DevStats), cudaMemcpyDeviceToHost, st));
  GLT_CUDA_TRY(cudaEventRecord(stats_ev[slot], st));
  stats_step[slot] = step;
  stats_lr[slot] = lr;
  return out ? step_stats(step, out) : GLT_OK;
}

int Model::step_stats(int step, GltStepStats* out) {
  const int slot = step & 1;
  if (step < 0 || stats_step[slot] != step)
    return fail(GLT_EINVAL, "the stats of step %d are not kept (the last two training steps are)", step);
  GLT_CUDA_TRY(cudaEventSynchronize(stats_ev[slot]));
  const DevStats& s = pinned_stats[slot];
  out->lm_loss = s.lm_loss;
  out->silence_loss = s.silence;
  out->domain_graft_energy = s.domain_energy;
  out->ood_graft_energy = s.ood_energy;
  out->domain_ood_energy_ratio = s.ratio;
  out->total_loss = s.total_loss;
  out->lr = stats_lr[slot];
  out->grad_norm = s.grad_norm;
  return status_from_device_error(s.dev_err, "glt_train_step");
}

int Model::forward_logits(const int32_t* ids_in, int host, int use_graft, uint16_t* out,
                          cudaStream_t st) {
  ScopedTileCounter tile_claims(gemm_counter());
  if (kind != GLT_MODEL_DECODER) return fail(GLT_ESTATE, "forward needs the decoder model");
  if (use_graft && !gw) return fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_TRY(load_inputs(ids_in, nullptr, host, st));
  GLT_CUDA_TRY(cudaMemsetAsync(esq_all, 0, sizeof(float) * 3 * static_cast<size_t>(L) * M, st));
  GLT_TRY(forward_all(use_graft != 0, st));
  if (out)
    GLT_TRY(g_bf16(kmaj(xf, D), kmaj(lm_head, D), M, V, D, out, V, nullptr, 0, st));
  // no host sync here: a timeout is reported by the model's next call that
  // reads results back
  return collect_device_error(device_error_word(), d_err, nullptr, st);
}

int Model::block_step(const uint16_t* x, const float* y_t, float lr, int step, float* loss,
                      uint16_t* out, float* dx_out, cudaStream_t st) {
  ScopedTileCounter tile_claims(gemm_counter());
  if (kind != GLT_MODEL_MLP_BLOCK) return fail(GLT_ESTATE, "block_step needs the MLP-block model");
  if (!gw) return fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_CUDA_TRY(cudaMemsetAsync(stats, 0, sizeof(DevStats), st));
  GLT_CUDA_TRY(cudaMemsetAsync(grad, 0, graft_numel * 4, st));
  GLT_CUDA_TRY(cudaMemsetAsync(ood, 0, sizeof(int32_t) * M, st));
  GLT_CUDA_TRY(cudaMemsetAsync(layers[0].esq, 0, sizeof(float) * 3 * M, st));
  GLT_CUDA_TRY(cudaMemcpyAsync(xs[0], x, static_cast<size_t>(M) * D * 2, cudaMemcpyDeviceToDevice, st));
  GLT_TRY(ensure_mlp_store());
  {
    SavingScope sv(saving);
    GLT_TRY(ffn_forward(0, xs[0], xs[1], var_in, true, st));
  }
  GLT_TRY(mse_grad(xs[1], y_t, dx, stats, M, D, st));
  GLT_TRY(ffn_backward(0, st));
  GLT_TRY(rmsnorm_bwd(dtmp, xs[0], layers[0].post_norm, var_in, dx, dx, nullptr, M, D, cfg.rms_norm_eps, st));
  if (out) GLT_CUDA_TRY(cudaMemcpyAsync(out, xs[1], static_cast<size_t>(M) * D * 2, cudaMemcpyDeviceToDevice, st));
  if (dx_out) GLT_CUDA_TRY(cudaMemcpyAsync(dx_out, dx, static_cast<size_t>(M) * D * 4, cudaMemcpyDeviceToDevice, st));
  const int kinds[3] = {cfg.graft_proj_gate, cfg.graft_proj_up, cfg.graft_proj_down};
  MirrorTargets mt = mirror();
  GLT_TRY(set_clip_scale(stats, 1.0f, st));
  GLT_PROF(GLT_PROF_ADAMW, adamw_step(gw, grad, adam_m, adam_v, L, S, H, lr, cfg.adam_beta1, cfg.adam_beta2,
                     cfg.adam_eps, cfg.adam_weight_decay, step, kinds, stats, &mt, st));
  if (loss) {
    GLT_TRY(collect_device_error(device_error_word(), d_err, &stats->dev_err, st));
    GLT_CUDA_TRY(cudaMemcpyAsync(pinned_stats, stats, sizeof(DevStats), cudaMemcpyDeviceToHost, st));
    GLT_CUDA_TRY(cudaStreamSynchronize(st));
    *loss = static_cast<float>(pinned_stats->ce_sum / (static_cast<double>(M) * D));
    return status_from_device_error(pinned_stats->dev_err, "glt_block_step");
  }
  return collect_device_error(device_error_word(), d_err, nullptr, st);
}

int Model::activation(int which, int layer, void** ptr, int64_t* numel) {
  if (layer < 0 || layer > L) return fail(GLT_EINVAL, "layer out of range");
  const bool dec = kind == GLT_MODEL_DECODER;
  const Layer* y = layer < L ? &layers[layer] : nullptr;
  switch (which) {
    case 0: *ptr = xs[layer]; *numel = static_cast<int64_t>(M) * D; return GLT_OK;
    case 1: if (!dec || !y) break; *ptr = y->qkv; *numel = static_cast<int64_t>(M) * QKV; return GLT_OK;
    case 2: if (!dec || !y) break; *ptr = y->o; *numel = static_cast<int64_t>(M) * AD; return GLT_OK;
    case 3: if (!y) break; *ptr = y->x_post; *numel = static_cast<int64_t>(M) * D; return GLT_OK;
    case 4: if (!y) break; *ptr = y->x_ffn; *numel = static_cast<int64_t>(M) * D; return GLT_OK;
    case 5: if (!y) break; *ptr = y->esq; *numel = static_cast<int64_t>(M) * 3; return GLT_OK;
    case 6: if (!dec) break; *ptr = xf; *numel = static_cast<int64_t>(M) * D; return GLT_OK;
    case 7: if (!y || overlay) break; *ptr = y->w_gu; *numel = 2 * static_cast<int64_t>(FF) * D; return GLT_OK;
    case 8: if (!y || overlay) break; *ptr = y->w_d; *numel = static_cast<int64_t>(D) * FF; return GLT_OK;
    default: break;
  }
  return fail(GLT_EINVAL, "activation %d unavailable for layer %d", which, layer);
}

}  // namespace glt

// =============================== C ABI =====================================
using glt::Model;

extern "C" int glt_config_default(GltModelConfig* cfg) {
  if (!cfg) return glt::fail(GLT_EINVAL, "null config");
  return glt::config_default(cfg);
}
extern "C" int glt_config_validate(const GltModelConfig* cfg, int batch_size, int mode) {
  return glt::config_validate(cfg, batch_size, mode);
}
extern "C" float glt_get_lr(const GltModelConfig* cfg, int step, int total_steps) {
  return cfg ? glt::get_lr(cfg, step, total_steps) : 0.f;
}
extern "C" int64_t glt_delta_offset(int layer, int proj, int slice_dim, int h_slice_dim) {
  return (static_cast<int64_t>(layer) * 3 + proj) * slice_dim * static_cast<int64_t>(h_slice_dim);
}

extern "C" int glt_model_create(const GltModelConfig* cfg, int batch_size, int seq_len, int kind,
                                GltModel** out) {
  if (!cfg || !out) return glt::fail(GLT_EINVAL, "null argument");
  if (kind != GLT_MODEL_DECODER && kind != GLT_MODEL_MLP_BLOCK)
    return glt::fail(GLT_EINVAL, "unknown model kind %d", kind);
  if (batch_size <= 0 || seq_len <= 0) return glt::fail(GLT_EINVAL, "batch/seq must be positive");
  Model* m = new (std::nothrow) Model();
  if (!m) return glt::fail(GLT_ENOMEM, "host allocation failed");
  int s = m->setup(*cfg, batch_size, seq_len, kind);
  if (s != GLT_OK) {
    delete m;
    return s;
  }
  *out = reinterpret_cast<GltModel*>(m);
  return GLT_OK;
}

extern "C" int glt_model_destroy(GltModel* m) {
  delete reinterpret_cast<Model*>(m);
  return GLT_OK;
}

extern "C" int glt_model_memory(const GltModel* m, int64_t* arena_bytes, int64_t* graft_bytes) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  const Model* mm = reinterpret_cast<const Model*>(m);
  if (arena_bytes) *arena_bytes = static_cast<int64_t>(mm->arena_bytes);
  if (graft_bytes) *graft_bytes = static_cast<int64_t>(mm->graft_bytes);
  return GLT_OK;
}

extern "C" int glt_model_mlp_store(GltModel* m, int mode, int* active, int64_t* bytes) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  Model* mm = reinterpret_cast<Model*>(m);
  if (mode != -1) GLT_TRY(mm->set_mlp_store(mode));
  if (active) *active = mm->gu_mem ? 1 : 0;
  if (bytes) *bytes = static_cast<int64_t>(mm->gu_bytes);
  return GLT_OK;
}

extern "C" int glt_model_init_random(GltModel* m, uint64_t seed, float std, float graft_std,
                                     float graft_down_std) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<Model*>(m)->init_random(seed, std, graft_std, graft_down_std);
}

extern "C" int glt_model_set_weight(GltModel* m, int layer, int which, const void* src,
                                    int64_t numel, int src_is_host, void* stream) {
  if (!m || !src) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->set_weight(layer, which, src, numel, src_is_host,
                                                 static_cast<cudaStream_t>(stream));
}

extern "C" int glt_model_graft_buffers(GltModel* m, float** weight, float** grad, float** adam_m,
                                       float** adam_v, int64_t* numel) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  Model* mm = reinterpret_cast<Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  if (weight) *weight = mm->gw;
  if (grad) *grad = mm->grad;
  if (adam_m) *adam_m = mm->adam_m;
  if (adam_v) *adam_v = mm->adam_v;
  if (numel) *numel = mm->graft_numel;
  return GLT_OK;
}

extern "C" int glt_model_refresh_graft(GltModel* m, void* stream) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<Model*>(m)->refresh_graft(static_cast<cudaStream_t>(stream));
}

extern "C" int glt_train_step(GltModel* m, const int32_t* ids, const int32_t* ood_mask,
                              int host_inputs, int step, int total_steps, GltStepStats* stats,
                              void* stream) {
  if (!m || !ids || !ood_mask) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->train_step(ids, ood_mask, host_inputs, step, total_steps,
                                                 stats, static_cast<cudaStream_t>(stream));
}

extern "C" int glt_model_step_stats(GltModel* m, int step, GltStepStats* stats) {
  if (!m || !stats) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->step_stats(step, stats);
}

extern "C" int glt_forward(GltModel* m, const int32_t* ids, int host_inputs, int use_graft,
                           uint16_t* logits, void* stream) {
  if (!m || !ids) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->forward_logits(ids, host_inputs, use_graft, logits,
                                                     static_cast<cudaStream_t>(stream));
}

extern "C" int glt_block_step(GltModel* m, const uint16_t* x, const float* y, float lr, int step,
                              float* loss, uint16_t* out, float* dx, void* stream) {
  if (!m || !x || !y) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->block_step(x, y, lr, step, loss, out, dx,
                                                 static_cast<cudaStream_t>(stream));
}

extern "C" int glt_model_profile(GltModel* m, int enable) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  reinterpret_cast<Model*>(m)->prof_on = enable != 0;
  return GLT_OK;
}

extern "C" int glt_model_profile_read(GltModel* m, double* ms, int64_t* launches, int reset) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  Model* mm = reinterpret_cast<Model*>(m);
  GLT_TRY(mm->prof_collect());
  for (int k = 0; k < GLT_PROF_KINDS; ++k) {
    if (ms) ms[k] = mm->prof_ms[k];
    if (launches) launches[k] = mm->prof_n[k];
    if (reset) {
      mm->prof_ms[k] = 0.0;
      mm->prof_n[k] = 0;
    }
  }
  return GLT_OK;
}

extern "C" int glt_model_activation(GltModel* m, int which, int layer, void** ptr, int64_t* numel) {
  if (!m || !ptr || !numel) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<Model*>(m)->activation(which, layer, ptr, numel);
}
