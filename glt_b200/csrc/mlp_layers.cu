// Layer-level entry points of the grafted MLP for callers that keep their
// own layer loop, and stand-alone graft weights.
//
// Reference mapping (Hinedes/GLT):
//   allocate_graft_weights / free_graft_weights_noexcept
//       src/graft_weights_impl.inc:6-62      -> glt_graft_weights_alloc / _free
//   refresh of the bf16 graft copy the GEMMs read (delta_bf16_mirror)
//                                            -> glt_mlp_set_graft
//   forward_layer, MLP half (post-attention RMSNorm, gate/up + deltas,
//       SiLU*mul, down + delta, residual)   src/layer_forward_impl.inc:53-285
//                                            -> glt_mlp_fwd
//   recompute_ffn                            src/layer_recompute_impl.inc:8-91
//                                            -> glt_mlp_recompute
//   backward_layer, MLP half + post-attention RMSNorm backward
//                                            src/layer_backward_impl.inc:36-367
//                                            -> glt_mlp_bwd
// The MLP runs in the same fused tcgen05 GEMMs as the whole-model step
// (Model::ffn_forward / ffn_backward); the handle is a Model that holds only
// the fused layer weights and one layer's scratch, with the caller's saved
// activations, gradients and OOD mask bound for the duration of each call.
#include <string.h>

#include "common.cuh"
#include "kernels_mem.cuh"
#include "model.cuh"

namespace glt {
namespace {

Model* as_model(GltMlp* m) { return reinterpret_cast<Model*>(m); }

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_layer(const Model* m, int layer) {
  if (layer < 0 || layer >= m->L) return fail(GLT_EINVAL, "layer %d out of range [0, %d)", layer, m->L);
  return GLT_OK;
}

// Binds the caller's saved activations of `layer` (and its gate_pre/up store).
int bind_saved(Model* m, int layer, const GltMlpSaved* sv, const void* gate_up, bool need_energy) {
  if (!sv || !sv->x_ffn || !sv->variance) return fail(GLT_EINVAL, "saved activations: null x_ffn or variance");
  if (!al16(sv->x_ffn)) return fail(GLT_EINVAL, "saved x_ffn must be 16-byte aligned");
  const bool down = m->enabled[3 * layer + 2] != 0;
  if (need_energy && !sv->energy_sq) return fail(GLT_EINVAL, "saved activations: null energy_sq");
  if (down && need_energy && (!sv->delta_down || !al16(sv->delta_down)))
    return fail(GLT_EINVAL, "saved delta_down (16-byte aligned) is needed: layer %d grafts the down projection", layer);
  if (gate_up && !al16(gate_up)) return fail(GLT_EINVAL, "gate_up store must be 16-byte aligned");
  Layer& y = m->layers[layer];
  y.x_ffn = sv->x_ffn;
  y.var2 = sv->variance;
  y.esq = sv->energy_sq;
  y.dd = sv->delta_down;
  y.gu = static_cast<uint16_t*>(const_cast<void*>(gate_up));
  return GLT_OK;
}

void unbind(Model* m, int layer) {
  Layer& y = m->layers[layer];
  y.x_ffn = nullptr;
  y.var2 = nullptr;
  y.esq = nullptr;
  y.dd = nullptr;
  y.gu = nullptr;
  m->dx = nullptr;
  m->grad = nullptr;
  m->ood = nullptr;
}

}  // namespace
}  // namespace glt

using glt::Model;

extern "C" int glt_graft_weights_alloc(const GltModelConfig* cfg, int domain_id, int with_bf16_mirror,
                                       GltGraftWeights* g) {
  if (!cfg || !g) return glt::fail(GLT_EINVAL, "null argument");
  if (g->allocated) GLT_TRY(glt_graft_weights_free(g));   // as the reference: re-allocation frees first
  memset(g, 0, sizeof(*g));
  if (cfg->num_layers <= 0 || cfg->slice_dim <= 0 || cfg->hidden_dim <= 0 || cfg->max_domains <= 0)
    return glt::fail(GLT_EINVAL, "graft weights: non-positive dimensions");
  const int64_t H = cfg->layout == GLT_LAYOUT_CONCAT ? cfg->hidden_dim : cfg->hidden_dim / cfg->max_domains;
  const int64_t n = static_cast<int64_t>(3) * cfg->num_layers * cfg->slice_dim * H;
  float* w = nullptr;
  if (cudaMalloc(&w, static_cast<size_t>(n) * 4) != cudaSuccess) {
    (void)cudaGetLastError();
    return glt::fail(GLT_ENOMEM, "graft weights: cudaMalloc(%lld fp32) failed", (long long)n);
  }
  uint16_t* wb = nullptr;
  if (with_bf16_mirror && cudaMalloc(&wb, static_cast<size_t>(n) * 2) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(w);
    return glt::fail(GLT_ENOMEM, "graft weights: cudaMalloc(%lld bf16 mirror) failed", (long long)n);
  }
  cudaError_t e = cudaMemset(w, 0, static_cast<size_t>(n) * 4);
  if (e == cudaSuccess && wb) e = cudaMemset(wb, 0, static_cast<size_t>(n) * 2);
  if (e != cudaSuccess) {
    cudaFree(w);
    if (wb) cudaFree(wb);
    return glt::fail(GLT_ECUDA, "graft weights: zero-init failed: %s", cudaGetErrorString(e));
  }
  g->weight = w;
  g->weight_bf16 = wb;
  g->weight_elems = n;
  g->domain_id = domain_id;
  g->allocated = 1;
  g->active = 0;
  return GLT_OK;
}

extern "C" int glt_graft_weights_free(GltGraftWeights* g) {
  if (!g) return glt::fail(GLT_EINVAL, "null argument");
  int rc = GLT_OK;
  if (g->weight && cudaFree(g->weight) != cudaSuccess) rc = glt::fail(GLT_ECUDA, "graft weights: cudaFree failed");
  if (g->weight_bf16 && cudaFree(g->weight_bf16) != cudaSuccess)
    rc = glt::fail(GLT_ECUDA, "graft weights: cudaFree (mirror) failed");
  memset(g, 0, sizeof(*g));   // every field reset, even when a free reported an error
  return rc;
}

extern "C" int glt_mlp_create(const GltModelConfig* cfg, int tokens, GltMlp** out) {
  if (!cfg || !out) return glt::fail(GLT_EINVAL, "null argument");
  if (tokens <= 0) return glt::fail(GLT_EINVAL, "tokens must be positive");
  Model* m = new (std::nothrow) Model();
  if (!m) return glt::fail(GLT_ENOMEM, "host allocation failed");
  m->external_acts = true;
  const int s = m->setup(*cfg, 1, tokens, GLT_MODEL_MLP_BLOCK);
  if (s != GLT_OK) {
    delete m;
    return s;
  }
  *out = reinterpret_cast<GltMlp*>(m);
  return GLT_OK;
}

extern "C" int glt_mlp_destroy(GltMlp* m) {
  delete glt::as_model(m);
  return GLT_OK;
}

extern "C" int glt_mlp_set_weight(GltMlp* m, int layer, int which, const void* src_bf16, int64_t numel,
                                  int src_is_host, void* stream) {
  if (!m || !src_bf16) return glt::fail(GLT_EINVAL, "null argument");
  if (which != GLT_W_POST_NORM && which != GLT_W_GATE && which != GLT_W_UP && which != GLT_W_DOWN)
    return glt::fail(GLT_EINVAL, "MLP weights are POST_NORM, GATE, UP and DOWN (got %d)", which);
  Model* mm = glt::as_model(m);
  GLT_TRY(glt::check_layer(mm, layer));
  return mm->set_weight(layer, which, src_bf16, numel, src_is_host, static_cast<cudaStream_t>(stream));
}

extern "C" int glt_mlp_set_graft(GltMlp* m, const GltGraftWeights* g, void* stream) {
  if (!m || !g) return glt::fail(GLT_EINVAL, "null argument");
  Model* mm = glt::as_model(m);
  if (!g->allocated || !g->weight) return glt::fail(GLT_ESTATE, "graft weights are not allocated");
  if (g->weight_elems != mm->graft_numel)
    return glt::fail(GLT_EINVAL, "graft weights hold %lld elements, the MLP needs %lld",
                     (long long)g->weight_elems, (long long)mm->graft_numel);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GLT_TRY(glt::refresh_mirror(g->weight, mm->L, mm->S, mm->H, mm->mirror(), st));
  if (g->weight_bf16) GLT_TRY(glt::cast_f32_to_bf16(g->weight, g->weight_bf16, g->weight_elems, st));
  return GLT_OK;
}

extern "C" int glt_mlp_recompute_bytes(const GltMlp* m, int64_t* bytes) {
  if (!m || !bytes) return glt::fail(GLT_EINVAL, "null argument");
  const Model* mm = reinterpret_cast<const Model*>(m);
  // blocked layout of 32-row bands of the interleaved [M, 2F'] gate_pre/up
  const int64_t rows = (static_cast<int64_t>(mm->M) + 31) / 32 * 32;
  *bytes = (rows * 2 * mm->FF * 2 + 255) / 256 * 256;
  return GLT_OK;
}

extern "C" int glt_mlp_fwd(GltMlp* m, int layer, const uint16_t* x_post, uint16_t* x_out,
                           const GltMlpSaved* saved, int use_graft, void* stream) {
  if (!m || !x_post || !x_out) return glt::fail(GLT_EINVAL, "null argument");
  Model* mm = glt::as_model(m);
  GLT_TRY(glt::check_layer(mm, layer));
  if (!glt::al16(x_post) || !glt::al16(x_out)) return glt::fail(GLT_EINVAL, "x_post / x_out must be 16-byte aligned");
  if (x_post == x_out) return glt::fail(GLT_EINVAL, "x_out must not alias x_post");
  GLT_TRY(glt::bind_saved(mm, layer, saved, nullptr, true));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = GLT_OK;
  if (cudaMemsetAsync(saved->energy_sq, 0, sizeof(float) * 3 * static_cast<size_t>(mm->M), st) != cudaSuccess)
    rc = glt::fail(GLT_ECUDA, "glt_mlp_fwd: energy reset failed");
  if (rc == GLT_OK) rc = mm->ffn_forward(layer, x_post, x_out, saved->variance, use_graft != 0, st);
  glt::unbind(mm, layer);
  return rc;
}

extern "C" int glt_mlp_recompute(GltMlp* m, int layer, const GltMlpSaved* saved, void* gate_up, void* stream) {
  if (!m || !gate_up) return glt::fail(GLT_EINVAL, "null argument");
  Model* mm = glt::as_model(m);
  GLT_TRY(glt::check_layer(mm, layer));
  GLT_TRY(glt::bind_saved(mm, layer, saved, gate_up, false));
  const int rc = mm->ffn_recompute(layer, static_cast<cudaStream_t>(stream));
  glt::unbind(mm, layer);
  return rc;
}

extern "C" int glt_mlp_bwd(GltMlp* m, int layer, float* dx, const uint16_t* x_post, const GltMlpSaved* saved,
                           const void* gate_up, const int32_t* ood_mask, float lambda_effective, float* grad,
                           void* stream) {
  if (!m || !dx || !x_post || !ood_mask || !grad) return glt::fail(GLT_EINVAL, "null argument");
  Model* mm = glt::as_model(m);
  GLT_TRY(glt::check_layer(mm, layer));
  if (!glt::al16(dx) || !glt::al16(x_post)) return glt::fail(GLT_EINVAL, "dx / x_post must be 16-byte aligned");
  GLT_TRY(glt::bind_saved(mm, layer, saved, gate_up, true));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  mm->dx = dx;
  mm->grad = grad;
  mm->ood = const_cast<int32_t*>(ood_mask);
  int rc = glt::set_lambda_eff(mm->stats, lambda_effective, st);
  // this layer's three [S, H] gradient slices start at zero (the split-K
  // weight-gradient GEMMs accumulate into them): beta = 0 as the reference
  const int64_t SH = static_cast<int64_t>(mm->S) * mm->H;
  if (rc == GLT_OK && cudaMemsetAsync(grad + 3 * layer * SH, 0, sizeof(float) * 3 * static_cast<size_t>(SH), st) != cudaSuccess)
    rc = glt::fail(GLT_ECUDA, "glt_mlp_bwd: gradient reset failed");
  if (rc == GLT_OK) rc = mm->ffn_backward(layer, st);
  // post-attention RMSNorm backward with the residual: dx += RMSNorm^T(d x_ffn)
  if (rc == GLT_OK)
    rc = glt::rmsnorm_bwd(mm->dtmp, x_post, mm->layers[layer].post_norm, saved->variance, dx, dx, nullptr, mm->M,
                          mm->D, mm->cfg.rms_norm_eps, st);
  glt::unbind(mm, layer);
  return rc;
}
