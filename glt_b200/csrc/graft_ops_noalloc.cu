// Allocation-free variant of glt_graft_op.
//
// Some callers cannot call cudaMalloc: code embedded in a framework whose
// own caching allocator owns the device memory budget, and latency-critical
// paths where cudaMalloc's implicit device synchronisation would stall other
// streams.  For them this entry point stages operands in a fixed workspace
// compiled into the library -- a file-scope __device__ array of
// kNoAllocScratchBytes that every GPU loading the library holds until the
// process exits -- instead of a caller-provided GltArena, and it never calls
// cudaMalloc, cudaFree or any allocating routine.
//
// In host code the array's name is only a host-side stand-in, not a device
// address, so its device address is fetched with cudaGetSymbolAddress once
// per device (with that device current) on the first call there; make that
// first call before any stream capture.  All calls on a device share the one
// array and leave their data in it: every byte a call reads is written by the
// same call first (packing also writes the zero padding), and calls that can
// overlap on the GPU (different streams, or different host threads) race on
// it and must be serialised by the caller.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels_mem.cuh"

namespace glt {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ unsigned int g_noalloc_err;  // device error word of this entry point

struct Slots {
  uint8_t* scratch;
  unsigned int* err;
};

std::mutex g_slots_mu;
std::unordered_map<int, Slots> g_slots;  // host-side map: device -> symbol addresses

int device_slots(Slots* out) {
  int dev = 0;
  GLT_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_slots_mu);
  auto it = g_slots.find(dev);
  if (it != g_slots.end()) {
    *out = it->second;
    return GLT_OK;
  }
  Slots s{nullptr, nullptr};
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.scratch), g_noalloc_scratch);
  if (e != cudaSuccess)
    return fail(GLT_ECUDA, "cudaGetSymbolAddress(workspace) failed: %s", cudaGetErrorString(e));
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err), g_noalloc_err);
  if (e != cudaSuccess)
    return fail(GLT_ECUDA, "cudaGetSymbolAddress(error word) failed: %s", cudaGetErrorString(e));
  g_slots[dev] = s;
  *out = s;
  return GLT_OK;
}

inline int64_t rup8(int64_t x) { return (x + 7) / 8 * 8; }

// Places a bf16 view of a [rows, cols] matrix at scratch offset *used when the
// source cannot be read by TMA in place (fp32, or rows not 16-byte aligned).
int stage(const void* src, int is_f32, int64_t ld, int rows, int cols, uint8_t* scratch,
          size_t* used, cudaStream_t st, const uint16_t** out, int64_t* out_ld) {
  if (!is_f32 && aligned16(src) && ld % 8 == 0 && ld >= cols) {
    *out = static_cast<const uint16_t*>(src);
    *out_ld = ld;
    return GLT_OK;
  }
  const int64_t l2 = rup8(cols < 8 ? 8 : cols);
  const size_t bytes = (static_cast<size_t>(rows) * l2 * 2 + 255) / 256 * 256;
  if (*used + bytes > kNoAllocScratchBytes)
    return fail(GLT_EINVAL,
                "glt_graft_op_noalloc: staged operands need more than the fixed %zu-byte "
                "workspace; use glt_graft_op with a GltArena for this size",
                kNoAllocScratchBytes);
  uint16_t* dst = reinterpret_cast<uint16_t*>(scratch + *used);
  *used += bytes;
  GLT_TRY(pack_bf16(src, is_f32, ld, rows, cols, dst, l2, st));
  *out = dst;
  *out_ld = l2;
  return GLT_OK;
}

template <bool AMN, bool BMN>
int gemm_f32(const Operand& a, const Operand& b, int M, int N, int K, float* C, int64_t ldc,
             float alpha, float beta, unsigned int* err, cudaStream_t st) {
  // the launcher shared with every other GEMM, with this entry point's own
  // error word (launch_gemm allocates nothing when it is given one)
  const bool vec = aligned16(C) && ldc % 4 == 0 && N % 4 == 0;
  EpiF32<128> epi{C, ldc, M, N, alpha, beta, 0, vec ? 1 : 0};
  return launch_gemm<128, 6, AMN, BMN>(a, b, M, N, K, epi, st, 1, nullptr, INT_MAX, 32, nullptr, 0, err);
}

}  // namespace

int noalloc_error_word(unsigned int** word) {
  Slots slots;
  GLT_TRY(device_slots(&slots));
  *word = slots.err;
  return GLT_OK;
}

int noalloc_error_take(unsigned int* code) {
  // a symbol copy allocates nothing; the word is this file's, per device
  unsigned int v = 0;
  GLT_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(v)));
  if (v) {
    const unsigned int zero = 0;
    GLT_CUDA_TRY(cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(zero)));
  }
  *code = v;
  return GLT_OK;
}

}  // namespace glt

extern "C" int glt_graft_op_noalloc(int op, int M, int S, int H, const float* w_f32,
                                    const uint16_t* w_bf16, const void* x, int x_is_f32,
                                    int64_t x_stride, const void* dy, int dy_is_f32,
                                    int64_t dy_stride, float* out, int64_t out_stride,
                                    float alpha, float beta, void* stream) {
  using namespace glt;
  if (M < 0 || S <= 0 || H <= 0) return fail(GLT_EINVAL, "graft op: bad sizes M=%d S=%d H=%d", M, S, H);
  if (!out) return fail(GLT_EINVAL, "graft op: null output");
  if (op < GLT_GRAFT_EXPAND_FWD || op > GLT_GRAFT_CONTRACT_DGRAD)
    return fail(GLT_EINVAL, "unknown graft op %d", op);
  Slots slots;
  GLT_TRY(device_slots(&slots));
  if (M == 0) return GLT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  size_t used = 0;
  const uint16_t *W = nullptr, *X = nullptr, *Y = nullptr;
  int64_t ldw = 0, ldx = 0, ldy = 0;
  const bool wgrad = op == GLT_GRAFT_EXPAND_WGRAD || op == GLT_GRAFT_CONTRACT_WGRAD;
  if (!wgrad) {
    if (w_bf16) {
      GLT_TRY(stage(w_bf16, 0, H, S, H, slots.scratch, &used, st, &W, &ldw));
    } else {
      if (!w_f32) return fail(GLT_EINVAL, "graft op: no weight");
      GLT_TRY(stage(w_f32, 1, H, S, H, slots.scratch, &used, st, &W, &ldw));
    }
  }
  switch (op) {
    case GLT_GRAFT_EXPAND_FWD:
      GLT_TRY(stage(x, x_is_f32, x_stride, M, H, slots.scratch, &used, st, &X, &ldx));
      return gemm_f32<false, false>(Operand{X, ldx, false}, Operand{W, ldw, false}, M, S, H, out,
                                    out_stride, alpha, beta, slots.err, st);
    case GLT_GRAFT_CONTRACT_FWD:
      GLT_TRY(stage(x, x_is_f32, x_stride, M, S, slots.scratch, &used, st, &X, &ldx));
      return gemm_f32<false, true>(Operand{X, ldx, false}, Operand{W, ldw, true}, M, H, S, out,
                                   out_stride, alpha, beta, slots.err, st);
    case GLT_GRAFT_EXPAND_WGRAD:
      GLT_TRY(stage(dy, dy_is_f32, dy_stride, M, S, slots.scratch, &used, st, &Y, &ldy));
      GLT_TRY(stage(x, x_is_f32, x_stride, M, H, slots.scratch, &used, st, &X, &ldx));
      return gemm_f32<true, true>(Operand{Y, ldy, true}, Operand{X, ldx, true}, S, H, M, out,
                                  out_stride, alpha, beta, slots.err, st);
    case GLT_GRAFT_CONTRACT_WGRAD:
      GLT_TRY(stage(x, x_is_f32, x_stride, M, S, slots.scratch, &used, st, &X, &ldx));
      GLT_TRY(stage(dy, dy_is_f32, dy_stride, M, H, slots.scratch, &used, st, &Y, &ldy));
      return gemm_f32<true, true>(Operand{X, ldx, true}, Operand{Y, ldy, true}, S, H, M, out,
                                  out_stride, alpha, beta, slots.err, st);
    case GLT_GRAFT_EXPAND_DGRAD:
      GLT_TRY(stage(dy, dy_is_f32, dy_stride, M, S, slots.scratch, &used, st, &Y, &ldy));
      return gemm_f32<false, true>(Operand{Y, ldy, false}, Operand{W, ldw, true}, M, H, S, out,
                                   out_stride, alpha, beta, slots.err, st);
    default:  // GLT_GRAFT_CONTRACT_DGRAD
      GLT_TRY(stage(dy, dy_is_f32, dy_stride, M, H, slots.scratch, &used, st, &Y, &ldy));
      return gemm_f32<false, false>(Operand{Y, ldy, false}, Operand{W, ldw, false}, M, S, H, out,
                                    out_stride, alpha, beta, slots.err, st);
  }
}
