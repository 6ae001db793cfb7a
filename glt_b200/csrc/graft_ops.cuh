// Stand-alone graft GEMMs (see graft_ops.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/glt_graft.h"

namespace glt {

int graft_op(int op, int M, int S, int H, const float* w_f32, const uint16_t* w_bf16,
             const void* x, int x_is_f32, int64_t x_stride, const void* dy, int dy_is_f32,
             int64_t dy_stride, float* out, int64_t out_stride, float alpha, float beta,
             void* scratch, size_t scratch_bytes, cudaStream_t st);

}  // namespace glt
