// The six stand-alone graft GEMMs of the reference (src/graft_ops_impl.inc,
// src/gemm_impl.inc:388-584) in general overlay geometry, on the tcgen05
// GEMM.  Operands whose layout TMA cannot address directly (f32 data, rows
// not 16-byte aligned, tiny slices such as the reference's S=3, H=2 golden
// vectors) are first packed to bf16 with 16-byte-aligned rows in a
// caller-provided workspace -- the counterpart of arena.d_bf16_temp, into
// which the reference converts f32 operands before every rocBLAS call.
#include <string.h>

#include <new>

#include "common.cuh"
#include "gemm.cuh"
#include "graft_ops.cuh"
#include "kernels_mem.cuh"

namespace glt {

namespace {

inline int64_t rup8(int64_t x) { return (x + 7) / 8 * 8; }

struct Scratch {
  uint8_t* base;
  size_t cap, used;
  uint16_t* take(size_t elems) {
    const size_t bytes = (elems * 2 + 255) / 256 * 256;
    if (used + bytes > cap) return nullptr;
    uint16_t* p = reinterpret_cast<uint16_t*>(base + used);
    used += bytes;
    return p;
  }
};

// Makes a bf16 view of a [rows, cols] matrix (row stride ld) usable by TMA,
// packing into scratch when the source is f32 or not aligned.
int stage(const void* src, int is_f32, int64_t ld, int rows, int cols, Scratch& sc,
          cudaStream_t st, const uint16_t** out, int64_t* out_ld, size_t* need) {
  const bool ok = !is_f32 && aligned16(src) && ld % 8 == 0 && ld >= cols;
  if (ok) {
    *out = static_cast<const uint16_t*>(src);
    *out_ld = ld;
    return GLT_OK;
  }
  const int64_t l2 = rup8(cols < 8 ? 8 : cols);
  *need += ((static_cast<size_t>(rows) * l2 * 2) + 255) / 256 * 256;
  uint16_t* dst = sc.take(static_cast<size_t>(rows) * l2);
  if (!dst) return GLT_ENOMEM;  // reported by the caller with the total need
  GLT_TRY(pack_bf16(src, is_f32, ld, rows, cols, dst, l2, st));
  *out = dst;
  *out_ld = l2;
  return GLT_OK;
}

template <bool AMN, bool BMN>
int run_f32(const Operand& a, const Operand& b, int M, int N, int K, float* C, int64_t ldc,
            float alpha, float beta, cudaStream_t st) {
  const bool vec = aligned16(C) && ldc % 4 == 0 && N % 4 == 0;
  EpiF32<128> e{C, ldc, M, N, alpha, beta, 0, vec ? 1 : 0};
  return launch_gemm<128, 6, AMN, BMN>(a, b, M, N, K, e, st);
}

}  // namespace

int graft_op(int op, int M, int S, int H, const float* w_f32, const uint16_t* w_bf16,
             const void* x, int x_is_f32, int64_t x_stride, const void* dy, int dy_is_f32,
             int64_t dy_stride, float* out, int64_t out_stride, float alpha, float beta,
             void* scratch, size_t scratch_bytes, cudaStream_t st) {
  if (M < 0 || S <= 0 || H <= 0) return fail(GLT_EINVAL, "graft op: bad sizes M=%d S=%d H=%d", M, S, H);
  if (!out) return fail(GLT_EINVAL, "graft op: null output");
  if (M == 0) return GLT_OK;
  Scratch sc{static_cast<uint8_t*>(scratch), scratch ? scratch_bytes : 0, 0};
  size_t need = 0;
  int s = GLT_OK;
  // weight [S, H] as bf16
  const uint16_t* W = nullptr;
  int64_t ldw = 0;
  if (op != GLT_GRAFT_EXPAND_WGRAD && op != GLT_GRAFT_CONTRACT_WGRAD) {
    if (w_bf16) {
      s = stage(w_bf16, 0, H, S, H, sc, st, &W, &ldw, &need);
    } else {
      if (!w_f32) return fail(GLT_EINVAL, "graft op: no weight");
      s = stage(w_f32, 1, H, S, H, sc, st, &W, &ldw, &need);
    }
  }
  const uint16_t* X = nullptr;
  const uint16_t* Y = nullptr;
  int64_t ldx = 0, ldy = 0;
  switch (op) {
    case GLT_GRAFT_EXPAND_FWD:       // out[M,S] = x_h[M,H] . W[S,H]^T
      if (s == GLT_OK) s = stage(x, x_is_f32, x_stride, M, H, sc, st, &X, &ldx, &need);
      break;
    case GLT_GRAFT_CONTRACT_FWD:     // out[M,H] = x_i[M,S] . W[S,H]
      if (s == GLT_OK) s = stage(x, x_is_f32, x_stride, M, S, sc, st, &X, &ldx, &need);
      break;
    case GLT_GRAFT_EXPAND_WGRAD:     // dW[S,H] = dy[M,S]^T . x_h[M,H]
      s = stage(dy, dy_is_f32, dy_stride, M, S, sc, st, &Y, &ldy, &need);
      if (s == GLT_OK) s = stage(x, x_is_f32, x_stride, M, H, sc, st, &X, &ldx, &need);
      break;
    case GLT_GRAFT_CONTRACT_WGRAD:   // dW[S,H] = x_i[M,S]^T . dy[M,H]
      s = stage(x, x_is_f32, x_stride, M, S, sc, st, &X, &ldx, &need);
      if (s == GLT_OK) s = stage(dy, dy_is_f32, dy_stride, M, H, sc, st, &Y, &ldy, &need);
      break;
    case GLT_GRAFT_EXPAND_DGRAD:     // dx_h[M,H] = dy[M,S] . W[S,H]
      if (s == GLT_OK) s = stage(dy, dy_is_f32, dy_stride, M, S, sc, st, &Y, &ldy, &need);
      break;
    case GLT_GRAFT_CONTRACT_DGRAD:   // gi[M,S] = dy_h[M,H] . W[S,H]^T
      if (s == GLT_OK) s = stage(dy, dy_is_f32, dy_stride, M, H, sc, st, &Y, &ldy, &need);
      break;
    default:
      return fail(GLT_EINVAL, "unknown graft op %d", op);
  }
  if (s == GLT_ENOMEM)
    return fail(GLT_ENOMEM, "graft op: workspace of %zu bytes too small (needs at least %zu)",
                scratch_bytes, need + 4096);
  if (s != GLT_OK) return s;
  switch (op) {
    case GLT_GRAFT_EXPAND_FWD:
      return run_f32<false, false>(Operand{X, ldx, false}, Operand{W, ldw, false}, M, S, H, out,
                                   out_stride, alpha, beta, st);
    case GLT_GRAFT_CONTRACT_FWD:
      return run_f32<false, true>(Operand{X, ldx, false}, Operand{W, ldw, true}, M, H, S, out,
                                  out_stride, alpha, beta, st);
    case GLT_GRAFT_EXPAND_WGRAD:
      return run_f32<true, true>(Operand{Y, ldy, true}, Operand{X, ldx, true}, S, H, M, out,
                                 out_stride, alpha, beta, st);
    case GLT_GRAFT_CONTRACT_WGRAD:
      return run_f32<true, true>(Operand{X, ldx, true}, Operand{Y, ldy, true}, S, H, M, out,
                                 out_stride, alpha, beta, st);
    case GLT_GRAFT_EXPAND_DGRAD:
      return run_f32<false, true>(Operand{Y, ldy, false}, Operand{W, ldw, true}, M, H, S, out,
                                  out_stride, alpha, beta, st);
    case GLT_GRAFT_CONTRACT_DGRAD:
      return run_f32<false, false>(Operand{Y, ldy, false}, Operand{W, ldw, false}, M, S, H, out,
                                   out_stride, alpha, beta, st);
  }
  return GLT_OK;
}

}  // namespace glt

// ------------------------------- C ABI -------------------------------------
struct GltArena {
  void* ptr = nullptr;
  size_t bytes = 0;
};

extern "C" int glt_arena_create(int64_t scratch_bytes, GltArena** out) {
  if (!out || scratch_bytes < 0) return glt::fail(GLT_EINVAL, "bad arguments");
  GltArena* a = new (std::nothrow) GltArena();
  if (!a) return glt::fail(GLT_ENOMEM, "host allocation failed");
  if (scratch_bytes > 0) {
    cudaError_t e = cudaMalloc(&a->ptr, static_cast<size_t>(scratch_bytes));
    if (e != cudaSuccess) {
      delete a;
      return glt::fail(GLT_ENOMEM, "cudaMalloc(%lld): %s", (long long)scratch_bytes,
                       cudaGetErrorString(e));
    }
  }
  a->bytes = static_cast<size_t>(scratch_bytes);
  *out = a;
  return GLT_OK;
}

extern "C" int glt_arena_destroy(GltArena* a) {
  if (a) {
    if (a->ptr) cudaFree(a->ptr);
    delete a;
  }
  return GLT_OK;
}

extern "C" int glt_graft_op(int op, int M, int S, int H, const float* w_f32,
                            const uint16_t* w_bf16, const void* x, int x_is_f32, int64_t x_stride,
                            const void* dy, int dy_is_f32, int64_t dy_stride, float* out,
                            int64_t out_stride, float alpha, float beta, GltArena* arena,
                            void* stream) {
  return glt::graft_op(op, M, S, H, w_f32, w_bf16, x, x_is_f32, x_stride, dy, dy_is_f32,
                       dy_stride, out, out_stride, alpha, beta, arena ? arena->ptr : nullptr,
                       arena ? arena->bytes : 0, static_cast<cudaStream_t>(stream));
}

extern "C" int glt_shadow_bake(uint16_t* base, int64_t base_stride, const float* graft, int S,
                               int H, int i0, int h0, int mode, void* stream) {
  if (!base || !graft) return glt::fail(GLT_EINVAL, "null argument");
  if (mode != 0 && mode != 1) return glt::fail(GLT_EINVAL, "bake mode must be 0 (expand) or 1 (contract)");
  if (i0 < 0 || h0 < 0 || S < 0 || H < 0) return glt::fail(GLT_EINVAL, "negative offset or size");
  return glt::shadow_bake(base, base_stride, graft, S, H, i0, h0, mode,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int glt_apply_graft_to_shadow(const GltModelConfig* cfg, uint16_t* const* gate,
                                         uint16_t* const* up, uint16_t* const* down,
                                         int64_t gate_up_stride, int64_t down_stride,
                                         const float* graft, int* baked_flag, void* stream) {
  if (!cfg || !baked_flag) return glt::fail(GLT_EINVAL, "null argument");
  if (*baked_flag)
    return glt::fail(GLT_ESTATE, "apply_graft_to_shadow called twice on the same model instance");
  *baked_flag = 1;  // set before the work, like g_shadow_baked (shadow_bake_impl.inc:62-64)
  if (!graft) return GLT_OK;  // empty graft: nothing to bake
  const int S = cfg->slice_dim;
  const int H = cfg->layout == GLT_LAYOUT_CONCAT ? cfg->hidden_dim : cfg->hidden_dim / cfg->max_domains;
  const int i0 = cfg->layout == GLT_LAYOUT_CONCAT ? cfg->intermediate_dim : cfg->domain_id * S;
  const int h0 = cfg->layout == GLT_LAYOUT_CONCAT ? 0 : cfg->domain_id * H;
  const int64_t SH = static_cast<int64_t>(S) * H;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int l = 0; l < cfg->num_layers; ++l) {
    if (l < cfg->graft_layer_start || l > cfg->graft_layer_end) continue;
    if (cfg->graft_proj_gate && gate)
      GLT_TRY(glt::shadow_bake(gate[l], gate_up_stride, graft + (3 * l + 0) * SH, S, H, i0, h0, 0, st));
    if (cfg->graft_proj_up && up)
      GLT_TRY(glt::shadow_bake(up[l], gate_up_stride, graft + (3 * l + 1) * SH, S, H, i0, h0, 0, st));
    if (cfg->graft_proj_down && down)
      GLT_TRY(glt::shadow_bake(down[l], down_stride, graft + (3 * l + 2) * SH, S, H, i0, h0, 1, st));
  }
  GLT_CUDA_TRY(cudaStreamSynchronize(st));
  return GLT_OK;
}
