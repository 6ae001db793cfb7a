// Eval-only and shadow-eval: the deterministic forward over an eval token set
// with the reference's metrics (grafting.hip:446-713):
//   mean_ce      mean next-token cross entropy over all B*(T-1) positions of
//                every sequence (no OOD mask), ppl = exp(mean_ce)
//   logits_sum   sum of all logits as fp32 values (bf16 logits widened)
//   logits_l2    sqrt(sum of squares)
//   logits_hash  FNV-1a 64 over the little-endian fp32 bytes of the logits,
//                [sequence, position, vocab] row-major, chained over batches
// The reference copies every batch's [B, T, V] logits to the host and walks
// them there.  Here the logits never leave the GPU:
//   * eval_rows_kernel   one CTA per row: online log-sum-exp (fp32), the
//                        target logit, row sum and sum of squares (fp64);
//   * eval_fnv_kernel    one CTA per row, one thread per value s of the low
//                        byte of the incoming hash state: F_row(s).  FNV-1a's
//                        XOR touches only the low byte and the multiply keeps
//                        the low byte a function of the low byte, so
//                        F_row(h) = F_row(h & 255) + (h - (h & 255)) * P^n;
//   * eval_fold_kernel   one CTA: the sequential fold of the row tables into
//                        the running hash, and fixed-order sums of the row
//                        partials, so repeated evals are bit-identical.
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "gemm.cuh"
#include "model.cuh"

namespace glt {

namespace {

constexpr uint64_t kFnvPrime = 1099511628211ull;
constexpr uint64_t kFnvBasis = 1469598103934665603ull;
constexpr int kEvalThreads = 256;

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;  // both empty
  s = s * expf(m - mx) + s2 * expf(m2 - mx);
  m = mx;
}

__global__ void __launch_bounds__(kEvalThreads) eval_rows_kernel(
    const uint16_t* __restrict__ logits, int V, int r0, const int32_t* __restrict__ ids, int T,
    double* __restrict__ out) {
  __shared__ float sm_m[kEvalThreads / 32], sm_s[kEvalThreads / 32];
  __shared__ double sm_a[kEvalThreads / 32], sm_b[kEvalThreads / 32];
  const int row = blockIdx.x;
  const uint16_t* x = logits + static_cast<int64_t>(row) * V;
  float m = -INFINITY, s = 0.f;
  double sum = 0.0, sq = 0.0;
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  for (int i = threadIdx.x; i < (V >> 3); i += kEvalThreads) {
    const uint4 w = x4[i];
    const float f[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                        bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
    float cm = f[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) cm = fmaxf(cm, f[k]);
    if (cm > m) {
      s = (m == -INFINITY) ? 0.f : s * expf(m - cm);
      m = cm;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s += expf(f[k] - m);
      sum += static_cast<double>(f[k]);
      sq += static_cast<double>(f[k]) * static_cast<double>(f[k]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
    sm_a[warp] = sum;
    sm_b[warp] = sq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm_m[0], Sx = sm_s[0];
    double a = sm_a[0], b = sm_b[0];
    for (int w = 1; w < kEvalThreads / 32; ++w) {
      lse_merge(M, Sx, sm_m[w], sm_s[w]);
      a += sm_a[w];
      b += sm_b[w];
    }
    const int g = r0 + row;
    double nll = 0.0;
    if (g % T != T - 1) {  // position t predicts token t+1 of the same sequence
      const int tgt = ids[g + 1];
      const float xt = (tgt >= 0 && tgt < V) ? bf16_bits_to_f32(x[tgt]) : 0.f;
      nll = static_cast<double>(M + logf(Sx)) - static_cast<double>(xt);
    }
    out[3 * static_cast<int64_t>(row) + 0] = nll;
    out[3 * static_cast<int64_t>(row) + 1] = a;
    out[3 * static_cast<int64_t>(row) + 2] = b;
  }
}

// F_row(s) for s = threadIdx.x.  A bf16 logit e widened to fp32 has the
// little-endian bytes {0, 0, e & 255, e >> 8}; the two zero bytes are a plain
// multiply by P^2.
constexpr int kFnvStage = 4096;  // bf16 values staged in shared memory per pass
__global__ void __launch_bounds__(kEvalThreads) eval_fnv_kernel(const uint16_t* __restrict__ logits,
                                                                int V, uint64_t* __restrict__ tables) {
  __shared__ __align__(16) uint32_t buf[kFnvStage / 2];
  const int row = blockIdx.x;
  const uint16_t* x = logits + static_cast<int64_t>(row) * V;
  const uint64_t P = kFnvPrime, P2 = kFnvPrime * kFnvPrime;
  uint64_t h = threadIdx.x;
  for (int base = 0; base < V; base += kFnvStage) {
    const int n = min(kFnvStage, V - base);  // a multiple of 8
    const uint4* src = reinterpret_cast<const uint4*>(x + base);
    for (int i = threadIdx.x; i < (n >> 3); i += kEvalThreads) reinterpret_cast<uint4*>(buf)[i] = src[i];
    __syncthreads();
#pragma unroll 4
    for (int i = 0; i < (n >> 1); ++i) {
      const uint32_t w = buf[i];  // same address in every thread: a broadcast
      h *= P2;
      h = (h ^ (w & 0xFFu)) * P;
      h = (h ^ ((w >> 8) & 0xFFu)) * P;
      h *= P2;
      h = (h ^ ((w >> 16) & 0xFFu)) * P;
      h = (h ^ (w >> 24)) * P;
    }
    __syncthreads();
  }
  tables[static_cast<int64_t>(row) * 256 + threadIdx.x] = h;
}

__global__ void __launch_bounds__(kEvalThreads) eval_fold_kernel(const uint64_t* __restrict__ tables,
                                                                 const double* __restrict__ rows_out,
                                                                 int rows, uint64_t pn,
                                                                 EvalAccum* __restrict__ acc) {
  __shared__ double red[3][kEvalThreads];
  double a = 0.0, b = 0.0, c = 0.0;
  for (int r = threadIdx.x; r < rows; r += kEvalThreads) {
    a += rows_out[3 * static_cast<int64_t>(r)];
    b += rows_out[3 * static_cast<int64_t>(r) + 1];
    c += rows_out[3 * static_cast<int64_t>(r) + 2];
  }
  red[0][threadIdx.x] = a;
  red[1][threadIdx.x] = b;
  red[2][threadIdx.x] = c;
  __syncthreads();
  for (int w = kEvalThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      red[0][threadIdx.x] += red[0][threadIdx.x + w];
      red[1][threadIdx.x] += red[1][threadIdx.x + w];
      red[2][threadIdx.x] += red[2][threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    uint64_t h = acc->hash;
    for (int r = 0; r < rows; ++r) {
      const uint64_t s = h & 255u;
      h = tables[static_cast<int64_t>(r) * 256 + s] + (h - s) * pn;
    }
    acc->hash = h;
    acc->nll += red[0][0];
    acc->sum += red[1][0];
    acc->sumsq += red[2][0];
  }
}

uint64_t pow_mod64(uint64_t b, uint64_t e) {
  uint64_t r = 1;
  while (e) {
    if (e & 1) r *= b;
    b *= b;
    e >>= 1;
  }
  return r;
}

}  // namespace

// Restores the model's batch geometry after a partial last batch.
struct BatchGuard {
  Model& m;
  int B, M;
  explicit BatchGuard(Model& mm) : m(mm), B(mm.B), M(mm.M) {}
  ~BatchGuard() { m.B = B; m.M = M; }
};

int Model::eval_alloc() {
  if (eval_mem) return GLT_OK;
  const size_t tables = sizeof(uint64_t) * 256 * static_cast<size_t>(ce_rows);
  const size_t rows = sizeof(double) * 3 * static_cast<size_t>(ce_rows);
  GLT_CUDA_TRY(cudaMalloc(&eval_mem, tables + rows + 256));
  ev_tables = static_cast<uint64_t*>(eval_mem);
  ev_rows = reinterpret_cast<double*>(static_cast<uint8_t*>(eval_mem) + tables);
  ev_acc = reinterpret_cast<EvalAccum*>(static_cast<uint8_t*>(eval_mem) + tables + rows);
  GLT_CUDA_TRY(cudaMallocHost(&ev_pinned, sizeof(EvalAccum)));
  return GLT_OK;
}

int Model::eval(const int32_t* ids_in, int64_t n_seq, int host, int use_graft, GltEvalStats* out,
                cudaStream_t st) {
  ScopedTileCounter tile_claims(gemm_counter());
  if (kind != GLT_MODEL_DECODER) return fail(GLT_ESTATE, "eval needs the decoder model");
  if (!ids_in || !out) return fail(GLT_EINVAL, "null argument");
  if (n_seq <= 0) return fail(GLT_EINVAL, "eval needs at least one sequence");
  if (T < 2) return fail(GLT_EINVAL, "eval needs seq_len >= 2");
  if (use_graft && !gw) return fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_TRY(eval_alloc());
  EvalAccum init{};
  init.hash = kFnvBasis;
  GLT_CUDA_TRY(cudaMemcpyAsync(ev_acc, &init, sizeof(init), cudaMemcpyHostToDevice, st));
  const uint64_t pn = pow_mod64(kFnvPrime, 4ull * static_cast<uint64_t>(V));
  const cudaMemcpyKind k = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  int64_t tokens = 0, graft_calls = 0;
  {
    BatchGuard guard(*this);
    const int Bmax = B;
    for (int64_t s0 = 0; s0 < n_seq; s0 += Bmax) {
      const int cur = static_cast<int>(std::min<int64_t>(Bmax, n_seq - s0));
      B = cur;
      M = cur * T;
      GLT_CUDA_TRY(cudaMemcpyAsync(ids, ids_in + s0 * T, sizeof(int32_t) * M, k, st));
      GLT_CUDA_TRY(cudaMemsetAsync(esq_all, 0, sizeof(float) * 3 * static_cast<size_t>(L) * M, st));
      GLT_TRY(forward_all(use_graft != 0, st));
      for (int r0 = 0; r0 < M; r0 += ce_rows) {
        const int rows = std::min(ce_rows, M - r0);
        GLT_TRY(lm_head_chunk(r0, rows, st));
        eval_rows_kernel<<<rows, kEvalThreads, 0, st>>>(logits, V, r0, ids, T, ev_rows);
        GLT_LAUNCH_CHECK();
        eval_fnv_kernel<<<rows, kEvalThreads, 0, st>>>(logits, V, ev_tables);
        GLT_LAUNCH_CHECK();
        eval_fold_kernel<<<1, kEvalThreads, 0, st>>>(ev_tables, ev_rows, rows, pn, ev_acc);
        GLT_LAUNCH_CHECK();
      }
      tokens += static_cast<int64_t>(cur) * (T - 1);
      // forward_layer dispatches graft GEMMs when the graft is active (the
      // reference's g_graft_fwd_calls, layer_forward_impl.inc:13,83)
      if (use_graft) graft_calls += L;
    }
  }
  GLT_TRY(collect_device_error(device_error_word(), d_err, &ev_acc->dev_err, st));
  GLT_CUDA_TRY(cudaMemcpyAsync(ev_pinned, ev_acc, sizeof(EvalAccum), cudaMemcpyDeviceToHost, st));
  GLT_CUDA_TRY(cudaStreamSynchronize(st));
  const EvalAccum& a = *ev_pinned;
  GLT_TRY(status_from_device_error(a.dev_err, "glt_model_eval"));
  out->tokens = tokens;
  out->total_nll = a.nll;
  out->mean_ce = a.nll / static_cast<double>(tokens);
  out->ppl = exp(out->mean_ce);
  out->logits_sum = a.sum;
  out->logits_l2 = sqrt(a.sumsq);
  out->logits_hash = a.hash;
  out->graft_forward_calls = graft_calls;
  return GLT_OK;
}

// apply_graft_to_shadow for the model's own graft (shadow_bake_impl.inc:58-128),
// then the graft storage is freed as the reference's shadow-eval does before
// its first forward (grafting.hip:483-490).  Overlay geometry bakes into the
// fused base weights (shadow_bake_fused).  In concat geometry the base has
// no rows in the graft's columns (they are zero padding), so the baked weight
// bf16(0 + delta) is exactly the bf16 copy the fused weights already hold;
// the layer keeps those columns in its GEMMs from now on.
int Model::shadow_bake_self(cudaStream_t st) {
  if (shadow_baked) return fail(GLT_ESTATE, "apply_graft_to_shadow called twice on the same model instance");
  if (!gw) return fail(GLT_ESTATE, "no graft to bake");
  shadow_baked = true;  // set before the work, like g_shadow_baked (shadow_bake_impl.inc:59-62)
  if (overlay)
    GLT_TRY(shadow_bake_fused(gw, L, S, H, i0, h0, mirror(), st));
  else
    GLT_TRY(refresh_graft(st));
  GLT_CUDA_TRY(cudaStreamSynchronize(st));
  GLT_CUDA_TRY(cudaFree(graft_mem));
  graft_mem = nullptr;
  graft_bytes = 0;
  gw = grad = adam_m = adam_v = nullptr;
  return GLT_OK;
}

}  // namespace glt

using glt::Model;

extern "C" int glt_model_eval(GltModel* m, const int32_t* ids, int64_t num_sequences,
                              int host_ids, int use_graft, GltEvalStats* out, void* stream) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<Model*>(m)->eval(ids, num_sequences, host_ids, use_graft, out,
                                           static_cast<cudaStream_t>(stream));
}

extern "C" int glt_model_shadow_bake(GltModel* m, void* stream) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<Model*>(m)->shadow_bake_self(static_cast<cudaStream_t>(stream));
}
