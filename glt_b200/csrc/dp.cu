// Data parallelism: each rank runs its own microbatch; the only exchange is a
// sum all-reduce of the graft gradients (base weights are frozen), issued per
// bucket of layers on a dedicated stream as soon as the bucket's weight-grad
// GEMMs have finished, so it overlaps the backward of the layers below.  Clip and AdamW
// then run replicated on identical (mean) gradients.  The reference is
// single-GPU; this is the new exchange step of the multi-GPU path.
//
// NCCL is resolved with dlopen at dp_init, so the library loads (and its
// single-GPU paths run) without NCCL present.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "model.cuh"

namespace glt {
namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;

int load_nccl() {
  if (g_nccl.handle) return GLT_OK;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* n : names) {
    h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) return fail(GLT_ENCCL, "cannot dlopen libnccl.so.2: %s", dlerror());
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
  g_nccl.CommInitRank = reinterpret_cast<decltype(g_nccl.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
  g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(dlsym(h, "ncclAllReduce"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
  g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(dlsym(h, "ncclCommAbort"));
  g_nccl.CommGetAsyncError =
      reinterpret_cast<decltype(g_nccl.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
  g_nccl.GetErrorString =
      reinterpret_cast<decltype(g_nccl.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRank || !g_nccl.AllReduce || !g_nccl.CommDestroy)
    return fail(GLT_ENCCL, "libnccl is missing required symbols");
  g_nccl.handle = h;
  return GLT_OK;
}

const char* nccl_err(ncclResult_t r) {
  return g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "nccl error";
}

}  // namespace

int Model::dp_init(const void* unique_id, int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) return fail(GLT_EINVAL, "bad rank/world");
  if (nccl_comm) return fail(GLT_ESTATE, "data parallelism already initialised");
  if (world == 1) {
    dp_rank = 0;
    dp_world = 1;
    return GLT_OK;
  }
  GLT_TRY(load_nccl());
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = g_nccl.CommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) return fail(GLT_ENCCL, "ncclCommInitRank: %s", nccl_err(r));
  nccl_comm = comm;
  dp_rank = rank;
  dp_world = world;
  // Layers per all-reduce (GLT_DP_BUCKET_LAYERS overrides the default 4).
  // Every all-reduce that NCCL starts while the persistent GEMMs run takes
  // SMs from the next GEMM, whose static tile schedule then waits for the
  // collective; four layers per call (200 MB at the Llama shape) cut those
  // collisions 4x while the call still overlaps the next four layers'
  // backward (2-GPU step 1271 -> 1256 ms, the same as one GPU).
  if (L > 0 && dp_bucket > L) dp_bucket = L;
  if (const char* e = getenv("GLT_DP_BUCKET_LAYERS")) {
    const int v = atoi(e);
    dp_bucket = v < 1 ? 1 : (v > L ? L : v);
  }
  // SMs left to NCCL by the GEMM that follows each all-reduce
  // (GLT_DP_RESERVE_SMS; NCCL's ring runs 32 CTAs at 2 and 4 ranks, NVLS 24
  // at 8) and how many GEMMs do so (GLT_DP_RESERVE_GEMMS, default 1: the dO
  // GEMM, which starts right after the all-reduce).
  if (const char* e = getenv("GLT_DP_RESERVE_SMS")) {
    const int v = atoi(e);
    dp_reserve_sms = v < 0 ? 0 : (v > 96 ? 96 : v);
  }
  if (const char* e = getenv("GLT_DP_RESERVE_GEMMS")) {
    const int v = atoi(e);
    dp_reserve_gemms = v < 0 ? 0 : (v > 8 ? 8 : v);
  }
  // GLT_DP_COMM_PRIORITY=high puts the all-reduce stream at the device's
  // highest stream priority, so that at each kernel boundary of the backward
  // the block scheduler starts the collective's CTAs before the next GEMM's.
  if (const char* e = getenv("GLT_DP_COMM_PRIORITY")) {
    if (strcmp(e, "high") == 0) {
      int least = 0, greatest = 0;
      GLT_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
      cudaStream_t hp = nullptr;
      GLT_CUDA_TRY(cudaStreamCreateWithPriority(&hp, cudaStreamNonBlocking, greatest));
      cudaStreamSynchronize(comm_stream);
      cudaStreamDestroy(comm_stream);
      comm_stream = hp;
    } else if (strcmp(e, "default") != 0) {
      return fail(GLT_EINVAL, "GLT_DP_COMM_PRIORITY=%s (high or default)", e);
    }
  }
  return GLT_OK;
}

int Model::dp_allreduce_layers(int l0, int l1) {
  if (dp_world <= 1 || l1 <= l0) return GLT_OK;
  const size_t n = static_cast<size_t>(3) * (l1 - l0) * S * H;   // layer-major: contiguous
  float* buf = grad + static_cast<int64_t>(3) * l0 * S * H;
  GLT_CUDA_TRY(cudaStreamWaitEvent(comm_stream, layer_done[l0], 0));
  ncclResult_t r = g_nccl.AllReduce(buf, buf, n, ncclFloat32, ncclSum,
                                    static_cast<ncclComm_t>(nccl_comm), comm_stream);
  if (r != ncclSuccess) return fail(GLT_ENCCL, "ncclAllReduce: %s", nccl_err(r));
  return GLT_OK;
}

// Asynchronous communicator state (ncclCommGetAsyncError): ncclSuccess, or
// the error a collective of this communicator ran into.
int Model::dp_async_error(int* nccl_result) {
  *nccl_result = 0;
  if (!nccl_comm || !g_nccl.CommGetAsyncError) return GLT_OK;
  ncclResult_t r = ncclSuccess;
  ncclResult_t q = g_nccl.CommGetAsyncError(static_cast<ncclComm_t>(nccl_comm), &r);
  if (q != ncclSuccess) return fail(GLT_ENCCL, "ncclCommGetAsyncError: %s", nccl_err(q));
  *nccl_result = static_cast<int>(r);
  if (r != ncclSuccess) return fail(GLT_ENCCL, "data-parallel communicator error: %s", nccl_err(r));
  return GLT_OK;
}

// Tears the communicator down without waiting for the other ranks
// (ncclCommAbort): for a rank that learned on the host that a peer has left,
// so that it neither waits in ncclCommDestroy nor starts another collective.
// The model stays usable for one-GPU training.
int Model::dp_abort() {
  if (!nccl_comm) {
    dp_world = 1;
    return GLT_OK;
  }
  ncclResult_t r = ncclSuccess;
  if (g_nccl.CommAbort) r = g_nccl.CommAbort(static_cast<ncclComm_t>(nccl_comm));
  nccl_comm = nullptr;
  dp_rank = 0;
  dp_world = 1;
  if (r != ncclSuccess) return fail(GLT_ENCCL, "ncclCommAbort: %s", nccl_err(r));
  return GLT_OK;
}

void Model::dp_shutdown() {
  if (nccl_comm) {
    cudaStreamSynchronize(comm_stream);
    g_nccl.CommDestroy(static_cast<ncclComm_t>(nccl_comm));
    nccl_comm = nullptr;
  }
  dp_world = 1;
}

}  // namespace glt

extern "C" int glt_dp_unique_id(void* out, int out_bytes) {
  if (!out || out_bytes < static_cast<int>(sizeof(ncclUniqueId)))
    return glt::fail(GLT_EINVAL, "unique id buffer must hold %d bytes", (int)sizeof(ncclUniqueId));
  GLT_TRY(glt::load_nccl());
  ncclUniqueId id;
  ncclResult_t r = glt::g_nccl.GetUniqueId(&id);
  if (r != ncclSuccess) return glt::fail(GLT_ENCCL, "ncclGetUniqueId: %s", glt::nccl_err(r));
  memcpy(out, &id, sizeof(id));
  return GLT_OK;
}

extern "C" int glt_dp_init(GltModel* m, const void* unique_id, int rank, int world) {
  if (!m || (!unique_id && world > 1)) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<glt::Model*>(m)->dp_init(unique_id, rank, world);
}

extern "C" int glt_dp_async_error(GltModel* m, int* nccl_result) {
  if (!m || !nccl_result) return glt::fail(GLT_EINVAL, "null argument");
  return reinterpret_cast<glt::Model*>(m)->dp_async_error(nccl_result);
}

extern "C" int glt_dp_abort(GltModel* m) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<glt::Model*>(m)->dp_abort();
}

extern "C" int glt_dp_finalize(GltModel* m) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  reinterpret_cast<glt::Model*>(m)->dp_shutdown();
  return GLT_OK;
}
