// Shared device/host helpers for the B200 graft-train library.
//
// Conventions kept from the reference (Hinedes/GLT):
//  * bf16 rounding is the bias trick `bits += ((bits>>16)&1) + 0x7FFF`
//    (src/kernels_elementwise_impl.inc:575-580, src/gemm_impl.inc:69-80,
//    src/checkpoint_impl.inc:49-57).  It equals IEEE RNE for every finite
//    value and differs only in NaN payload handling, so the bf16 stores that
//    reach files or the reference's element-wise entry points use it to stay
//    bit-identical with the reference.  The GEMM and attention epilogues,
//    whose outputs are intermediate activations, round with the hardware
//    RNE conversion (pack_bf16x2_rn): one instruction per two values, the
//    same bits for every finite value.
//  * Errors never throw across the C ABI: every entry point returns a
//    GltStatus and records a message readable through glt_last_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/glt_graft.h"

namespace glt {

// Records a formatted error message for glt_last_error() (thread local).
void set_error(const char* fmt, ...);
// Convenience: record message, return status.
int fail(int status, const char* fmt, ...);

}  // namespace glt

#define GLT_CUDA_TRY(expr)                                                        \
  do {                                                                            \
    cudaError_t _e = (expr);                                                      \
    if (_e != cudaSuccess) {                                                      \
      return ::glt::fail(GLT_ECUDA, "%s:%d: %s -> %s", __FILE__, __LINE__, #expr, \
                         cudaGetErrorString(_e));                                 \
    }                                                                             \
  } while (0)

#define GLT_TRY(expr)          \
  do {                         \
    int _s = (expr);           \
    if (_s != GLT_OK) return _s; \
  } while (0)

namespace glt {
// Counts this library's kernel launches (glt_launch_count).
void count_launch();
}  // namespace glt

#define GLT_LAUNCH_CHECK()           \
  do {                               \
    ::glt::count_launch();           \
    GLT_CUDA_TRY(cudaGetLastError()); \
  } while (0)

// ----------------------------------------------------------------------------
// bf16 <-> f32 (bit-level, reference rounding)
// ----------------------------------------------------------------------------
__host__ __device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
  uint32_t bits = static_cast<uint32_t>(v) << 16;
  float f;
#ifdef __CUDA_ARCH__
  f = __uint_as_float(bits);
#else
  __builtin_memcpy(&f, &bits, 4);
#endif
  return f;
}

__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t bits;
#ifdef __CUDA_ARCH__
  bits = __float_as_uint(f);
#else
  __builtin_memcpy(&bits, &f, 4);
#endif
  bits += ((bits >> 16) & 1u) + 0x7FFFu;
  return static_cast<uint16_t>(bits >> 16);
}

// Packs two floats into one 32-bit word of two bf16 (lo = a, hi = b).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  return static_cast<uint32_t>(f32_to_bf16_bits(a)) |
         (static_cast<uint32_t>(f32_to_bf16_bits(b)) << 16);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// Packs two floats into two bf16 (lo = a, hi = b) with the hardware
// round-to-nearest-even conversion: one instruction where pack_bf16x2 takes
// several.  Same result for finite values; for kernel-internal operands
// (attention probabilities) that no reference pins bit for bit.
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Eight bf16 values in one 16-byte word <-> eight floats.
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]); u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]); u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// Round-trip an fp32 value through bf16 (reference rounding).
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_f32(f32_to_bf16_bits(f));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Device-side error word: kernels that give up a bounded wait write a code
// into this per-device word (they never trap); the host reads it back with
// glt_device_error().  Allocated lazily once per device.
namespace glt {
unsigned int* device_error_word();
// GLT_OK for code 0, else GLT_ETIMEOUT (a bounded wait ran out) or
// GLT_EINVAL (a kernel rejected its shape), with a message naming `where`.
int status_from_device_error(unsigned int code, const char* where);
// Reads and clears the error word of the allocation-free graft op on the
// current device (graft_ops_noalloc.cu); noalloc_error_word gives its device
// address (for the failure-path self-test).
int noalloc_error_take(unsigned int* code);
int noalloc_error_word(unsigned int** word);
}
#define GLT_DEVERR_MBAR_TIMEOUT 1u
#define GLT_DEVERR_BAD_SHAPE 2u
