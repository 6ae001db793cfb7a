// Grafted MLP in the reference's own overlay geometry: the graft adds
//   delta_gate = x[:, h0:h0+H] . Delta_gate^T   into gate_pre[:, i0:i0+S]
//   delta_up   = x[:, h0:h0+H] . Delta_up^T     into up[:, i0:i0+S]
//   delta_down = h[:, i0:i0+S] . Delta_down     into ffn_out[:, h0:h0+H]
// with i0 = domain_id * S, h0 = domain_id * H and Delta stored [S, H]
// (layer_forward_impl.inc:21-218, graft_ops_impl.inc:5-114).
//
// Forward per layer:
//   expand delta GEMM (both projections in one GEMM: gate and up are adjacent
//   in the [3L, S, H] layout) -> fp32 deltas + energies;
//   base gate/up GEMM with the deltas injected before SwiGLU;
//   contract delta GEMM -> fp32 delta_down + energy (bf16 copy saved);
//   base down GEMM with delta_down injected and the residual added.
// Backward per layer (layer_backward_impl.inc:36-361):
//   dy = bf16(dx), dyh = bf16(dx_h + silence) on the hidden window;
//   ContractInputGrad dyh . Delta_down^T injected into the dh GEMM;
//   expand deltas recomputed; recompute GEMM with SwiGLU backward, silence
//   blend of the expand grads and the h slice;
//   ContractWeightGrad, ExpandWeightGrad (split-K, K = tokens);
//   base dx GEMM, then ExpandInputGrad accumulated into its hidden window.
#include "common.cuh"
#include "gemm.cuh"
#include "kernels_mem.cuh"
#include "mlp_epilogues.cuh"
#include "model.cuh"

namespace glt {

namespace {
inline Operand kmaj(const void* p, int64_t ld) { return Operand{p, ld, false}; }
inline Operand mnmaj(const void* p, int64_t ld) { return Operand{p, ld, true}; }

template <typename Epi128, typename Epi256, bool A_MN, bool B_MN>
int launch_by_n(const Operand& A, const Operand& B, int M, int N, int K, const Epi128& e128,
                const Epi256& e256, cudaStream_t st, int splits = 1) {
  if (N >= 1024 && splits == 1) return launch_gemm<256, 4, A_MN, B_MN>(A, B, M, N, K, e256, st);
  return launch_gemm<128, 6, A_MN, B_MN>(A, B, M, N, K, e128, st, splits);
}
}  // namespace

// delta[:, 0:S] (gate) and delta[:, S:2S] (up) = x_h . Delta^T, fp32 in dlt;
// per-token sums of squares into esq_gate / esq_up when non-null.
int Model::expand_deltas(int l, bool gate, bool up, float* esq_gate, float* esq_up, cudaStream_t st) {
  const Layer& y = layers[l];
  const int64_t SH = static_cast<int64_t>(S) * H;
  const int p0 = gate ? 0 : 1;
  const int N = (gate && up) ? 2 * S : S;
  float* C = dlt + p0 * S;
  float* lo = gate ? esq_gate : esq_up;
  float* hi = (gate && up) ? esq_up : nullptr;
  EpiDeltaF32<128> e1{C, 2 * static_cast<int64_t>(S), nullptr, 0, M, N, S, lo, hi};
  EpiDeltaF32<256> e2{C, 2 * static_cast<int64_t>(S), nullptr, 0, M, N, S, lo, hi};
  // ExpandForward (graft_ops_impl.inc:14-24): A = x[:, h0:h0+H] (ld D), B = Delta [S, H]
  return launch_by_n<EpiDeltaF32<128>, EpiDeltaF32<256>, false, false>(
      kmaj(y.x_ffn + h0, D), kmaj(gwb + (3 * l + p0) * SH, H), M, N, H, e1, e2, st);
}

int Model::ffn_forward_overlay(int l, const uint16_t* x_in, uint16_t* x_out, float* var_out,
                               bool use_graft, cudaStream_t st) {
  Layer& y = layers[l];
  const bool g = use_graft && enabled[3 * l], u = use_graft && enabled[3 * l + 1];
  const bool d = use_graft && enabled[3 * l + 2];
  const int64_t SH = static_cast<int64_t>(S) * H;
  GLT_PROF(GLT_PROF_RMSNORM, rmsnorm_fwd(x_in, y.post_norm, y.x_ffn, var_out, M, D, cfg.rms_norm_eps, st));
  if (g || u) GLT_PROF(GLT_PROF_DELTA_EXPAND, expand_deltas(l, g, u, y.esq, y.esq + M, st));
  {
    EpiSwiGLUFwdOv e{h, FF, M, g ? dlt : nullptr, u ? dlt + S : nullptr, 2 * static_cast<int64_t>(S),
                     i0, i0 + S, saving ? y.gu : nullptr, 2 * static_cast<int64_t>(FF) / 8};
    GLT_PROF(GLT_PROF_GATE_UP_FWD,
             (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * FF, D, e, st)));
  }
  float* dd32 = dtmp;  // [M, H] fp32; dtmp is free during the forward
  if (d) {
    // ContractForward (graft_ops_impl.inc:33-114): A = h[:, i0:i0+S], B[n=h][k=s] = Delta_down[s, h]
    EpiDeltaF32<128> e1{dd32, H, y.dd, H, M, H, H, y.esq + 2 * static_cast<int64_t>(M), nullptr};
    EpiDeltaF32<256> e2{dd32, H, y.dd, H, M, H, H, y.esq + 2 * static_cast<int64_t>(M), nullptr};
    GLT_PROF(GLT_PROF_DELTA_DOWN, (launch_by_n<EpiDeltaF32<128>, EpiDeltaF32<256>, false, true>(
                                      kmaj(h + i0, FF), mnmaj(gwb + (3 * l + 2) * SH, H), M, H, S,
                                      e1, e2, st)));
  }
  {
    EpiBF16Inj<128> e1{x_out, D, x_in, D, M, D, d ? dd32 : nullptr, H, h0, h0 + H};
    EpiBF16Inj<256> e2{x_out, D, x_in, D, M, D, d ? dd32 : nullptr, H, h0, h0 + H};
    GLT_PROF(GLT_PROF_DOWN_FWD, (launch_by_n<EpiBF16Inj<128>, EpiBF16Inj<256>, false, false>(
                                    kmaj(h, FF), kmaj(y.w_d, FF), M, D, FF, e1, e2, st)));
  }
  return GLT_OK;
}

int Model::ffn_backward_overlay(int l, cudaStream_t st) {
  Layer& y = layers[l];
  const bool g = enabled[3 * l], u = enabled[3 * l + 1], d = enabled[3 * l + 2];
  const int64_t SH = static_cast<int64_t>(S) * H;
  const int64_t S2 = 2 * static_cast<int64_t>(S);
  // dy = bf16(dx);  dyh = bf16(dx[:, h0:h0+H] + silence_down)  [M, H]
  GLT_TRY(silence_down_prep(dx, d ? y.dd : nullptr, H, y.esq + 2 * static_cast<int64_t>(M), ood,
                            stats, dy_b, dyg_b, H, M, D, h0, H, st));
  if (y.gu) {
    // gate_pre/up (with the deltas) were stored by the forward: no recompute.
    // ContractInputGrad (layer_backward_impl.inc:311-342): gi_slice =
    // dyh . Delta_down^T -> dtmp [M, S] (free until the dx GEMM below); the
    // expand deltas -> dlt for the silence term; then dh = dy . W_d with
    // SwiGLU's backward in its epilogue.
    float* gi = d ? dtmp : nullptr;
    if (d) {
      EpiF32<128> e1{gi, S, M, S, 1.f, 0.f, 0, 1};
      EpiF32<256> e2{gi, S, M, S, 1.f, 0.f, 0, 1};
      GLT_PROF(GLT_PROF_GRAFT_DGRAD, (launch_by_n<EpiF32<128>, EpiF32<256>, false, false>(
                                kmaj(dyg_b, H), kmaj(gwb + (3 * l + 2) * SH, H), M, S, H, e1, e2, st)));
    }
    if (g || u) GLT_PROF(GLT_PROF_DELTA_EXPAND, expand_deltas(l, g, u, nullptr, nullptr, st));
    const int64_t ld2 = 2 * static_cast<int64_t>(FF);
    if (FF >= 1024) {
      EpiSwiGLUBwdStoredOv<256> e{y.gu, ld2 / 8, dgu, ld2, gi, S, g ? dlt : nullptr, u ? dlt + S : nullptr, S2,
                                  (g || u) ? dys : nullptr, S2, d ? hg : nullptr, S_pad, M, FF, i0, i0 + S, S,
                                  y.esq, y.esq + M, ood, stats};
      GLT_PROF(GLT_PROF_DH, (launch_gemm<256, 4, false, true>(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, FF, D, e, st)));
    } else {
      EpiSwiGLUBwdStoredOv<128> e{y.gu, ld2 / 8, dgu, ld2, gi, S, g ? dlt : nullptr, u ? dlt + S : nullptr, S2,
                                  (g || u) ? dys : nullptr, S2, d ? hg : nullptr, S_pad, M, FF, i0, i0 + S, S,
                                  y.esq, y.esq + M, ood, stats};
      GLT_PROF(GLT_PROF_DH, (launch_gemm<128, 6, false, true>(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, FF, D, e, st)));
    }
  } else {
  // ContractInputGrad (layer_backward_impl.inc:311-342): gi_slice = dyh . Delta_down^T -> dlt [M, S]
  if (d) {
    EpiF32<128> e1{dlt, S, M, S, 1.f, 0.f, 0, 1};
    EpiF32<256> e2{dlt, S, M, S, 1.f, 0.f, 0, 1};
    GLT_PROF(GLT_PROF_GRAFT_DGRAD, (launch_by_n<EpiF32<128>, EpiF32<256>, false, false>(
                              kmaj(dyg_b, H), kmaj(gwb + (3 * l + 2) * SH, H), M, S, H, e1, e2, st)));
  }
  // dh = dy . W_d (+ gi_slice on [i0, i0+S))
  {
    EpiBF16Inj<256> e{dh, FF, nullptr, 0, M, FF, d ? dlt : nullptr, S, i0, i0 + S};
    GLT_PROF(GLT_PROF_DH,
             (launch_gemm<256, 4, false, true>(kmaj(dy_b, D), mnmaj(y.w_d, FF), M, FF, D, e, st)));
  }
  // expand deltas again (overwrites gi_slice, consumed above)
  if (g || u) GLT_PROF(GLT_PROF_DELTA_EXPAND, expand_deltas(l, g, u, nullptr, nullptr, st));
  // recompute gate/up + SwiGLU backward + silence blend + h slice
  {
    EpiSwiGLUBwdOv e{dh, FF, dgu, 2 * static_cast<int64_t>(FF), g ? dlt : nullptr,
                     u ? dlt + S : nullptr, S2, (g || u) ? dys : nullptr, S2, d ? hg : nullptr,
                     S_pad, M, i0, i0 + S, S, y.esq, y.esq + M, ood, stats};
    GLT_PROF(GLT_PROF_RECOMPUTE,
             (launch_gemm<256, 4, false, false>(kmaj(y.x_ffn, D), kmaj(y.w_gu, D), M, 2 * FF, D, e, st)));
  }
  }
  // ContractWeightGrad (graft_ops_impl.inc:214-228): dDelta_down = h_sliceᵀ . dyh
  // ExpandWeightGrad (graft_ops_impl.inc:120-156): dDelta_{gate,up} = dysᵀ . x_h
  // 128x256 tiles when the H slice is wide (half the L2 operand traffic per
  // FLOP of 128x128), splits for ~1.5 waves.
  const bool wide = H >= 512;
  if (d) {
    if (wide) {
      EpiF32<256> e{grad + (3 * l + 2) * SH, H, S, H, 1.f, 0.f, 1, 1};
      GLT_PROF(GLT_PROF_WGRAD_DOWN, (launch_gemm<256, 4, true, true>(mnmaj(hg, S_pad), mnmaj(dyg_b, H), S, H, M,
                                                                     e, st, pick_k_splits(S, H, M, 256, 3))));
    } else {
      EpiF32<128> e{grad + (3 * l + 2) * SH, H, S, H, 1.f, 0.f, 1, 1};
      GLT_PROF(GLT_PROF_WGRAD_DOWN, (launch_gemm<128, 6, true, true>(mnmaj(hg, S_pad), mnmaj(dyg_b, H), S, H, M,
                                                                     e, st, pick_k_splits(S, H, M, 128))));
    }
  }
  if (g || u) {
    const int p0 = g ? 0 : 1;
    const int rows = (g && u) ? 2 * S : S;
    const Operand a = mnmaj(dys + p0 * S, S2), b = mnmaj(y.x_ffn + h0, D);
    if (wide) {
      EpiF32<256> e{grad + (3 * l + p0) * SH, H, rows, H, 1.f, 0.f, 1, 1};
      GLT_PROF(GLT_PROF_WGRAD_GATE_UP,
               (launch_gemm<256, 4, true, true>(a, b, rows, H, M, e, st, pick_k_splits(rows, H, M, 256, 3))));
    } else {
      EpiF32<128> e{grad + (3 * l + p0) * SH, H, rows, H, 1.f, 0.f, 1, 1};
      GLT_PROF(GLT_PROF_WGRAD_GATE_UP,
               (launch_gemm<128, 6, true, true>(a, b, rows, H, M, e, st, pick_k_splits(rows, H, M, 128))));
    }
  }
  // base input grad through gate/up
  {
    EpiF32<256> e{dtmp, D, M, D, 1.f, 0.f, 0, 1};
    GLT_PROF(GLT_PROF_DX_GATE_UP,
             (launch_gemm<256, 4, false, true>(kmaj(dgu, 2 * static_cast<int64_t>(FF)), mnmaj(y.w_gu, D),
                                               M, D, 2 * FF, e, st)));
  }
  // ExpandInputGrad (layer_backward_impl.inc:148-155): dx[:, h0:h0+H] += dys . Delta
  if (g || u) {
    const int p0 = g ? 0 : 1;
    const int K = (g && u) ? 2 * S : S;
    EpiF32<128> e{dtmp + h0, D, M, H, 1.f, 1.f, 0, 1};
    GLT_PROF(GLT_PROF_GRAFT_DGRAD,
             (launch_gemm<128, 6, false, true>(kmaj(dys + p0 * S, S2), mnmaj(gwb + (3 * l + p0) * SH, H),
                                               M, H, K, e, st)));
  }
  return GLT_OK;
}

}  // namespace glt
