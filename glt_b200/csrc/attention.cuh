// Causal GQA attention of the decoder layer (reference: layer_forward_impl.inc:25-59
// forward with at::scaled_dot_product_attention, attention_autograd_impl.inc:1-39
// backward by autograd re-run).  Flash-style: the [T, T] score matrix is never
// materialised; GQA is handled by indexing (no repeat_interleave copies).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace glt {

struct AttnShape {
  int B, T, nh, nkv, hd;
  int64_t ld_qkv;   // row stride of the packed [q | k | v] activation (elements)
  int64_t ld_o;     // row stride of O / dO (elements)
  float scale;      // 1/sqrt(hd)
};

// In-place half-split RoPE on the q and k parts of the packed qkv rows
// (rope_impl.inc:8-39).  cos/sin tables are [T, hd/2] fp32.  inverse = 1
// applies the transpose rotation (used on dq/dk in the backward pass).
int rope_apply(uint16_t* qkv, const AttnShape& s, const float* cos_t, const float* sin_t,
               int inverse, int apply_q, int apply_k, cudaStream_t st);

// O = softmax(Q K^T * scale, causal) V, lse = logsumexp per (b, h, t).
// flash_fwd: mma.sync kernel (seq_len % 64 == 0); flash_fwd_tc: tcgen05/TMEM
// kernel (attention_tc.cu, seq_len % 128 == 0).  Same outputs.
int flash_fwd(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s, cudaStream_t st);
int flash_fwd_tc(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s, cudaStream_t st);

// Backward: dqkv (bf16, same packing as qkv) from dO, O, lse.  Needs fp32
// workspaces dq_acc [B*T, nh*hd] and dsum [B*nh*T].
int flash_bwd(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
              uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st);
// tcgen05/TMEM backward (attention_tc.cu; hd 128, seq_len % 128 == 0); same
// contract as flash_bwd.  dsum_ready: dsum was computed by the caller (the
// dO GEMM's epilogue, EpiBF16Dsum).  rope_cos/sin (nullable, [T, hd/2]):
// the inverse RoPE of the q columns is applied to dq before its bf16
// rounding (the k columns are left to rope_apply).
int flash_bwd_tc(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
                 uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st,
                 bool dsum_ready = false, const float* rope_cos = nullptr, const float* rope_sin = nullptr);
// tcgen05/TMEM backward for head_dim 64 (attention_tc.cu; seq_len % 128 == 0):
// same outputs as flash_bwd.  acc is an fp32 workspace of
// B*T*(nh + 2*nkv)*hd floats (dQ, then dK and dV accumulated over the GQA
// heads).  rope_cos/sin (nullable, [T, hd/2]): the inverse RoPE of the q and
// k columns is applied before their bf16 rounding (no separate RoPE pass).
int flash_bwd_tc64(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
                   uint16_t* dqkv, float* acc, float* dsum, const AttnShape& s, cudaStream_t st,
                   bool dsum_ready = false, const float* rope_cos = nullptr, const float* rope_sin = nullptr);
// Shared pre/post steps of both backward kernels: zero dq_acc and compute
// dsum = rowsum(dO * O) (unless dsum_ready); convert dq_acc (fp32) into the
// q columns of dqkv, with the inverse RoPE when tables are given.
int attn_bwd_prep(const uint16_t* o, const uint16_t* dout, float* dq_acc, float* dsum,
                  const AttnShape& s, cudaStream_t st, bool dsum_ready = false);
int attn_bwd_finish(const float* dq_acc, uint16_t* dqkv, const AttnShape& s, cudaStream_t st,
                    const float* rope_cos = nullptr, const float* rope_sin = nullptr);

}  // namespace glt
