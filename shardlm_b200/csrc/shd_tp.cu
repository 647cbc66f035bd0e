// Tensor parallelism over NVLink: NCCL, loaded at run time (dlopen of libnccl.so.2 -- inside a
// PyTorch process this resolves to the NCCL torch already loaded). All-reduce is linear over
// additive shares, so the client and server partial shares of a row-parallel projection are summed
// by ONE all-reduce of the packed [2][M][h] buffer. Vocabulary-parallel lm_head: the greedy token is
// an all-reduce MAX of (orderable logit, global index) keys.
//
// The reference has no NCCL at all (crates/v2/core/src/comm.rs:95-136 sums on the host, TODO at
// :105); its only TP is the plaintext DistributedEngine (crates/v2/model/src/distributed.rs:312-624).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "shd_model.cuh"

namespace {

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  std::string error;
};

NcclApi* nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.error = std::string("dlopen(libnccl.so.2) failed: ") + dlerror();
      return;
    }
    api.h = h;
#define LOAD(name, sym)                                              \
  api.name = reinterpret_cast<decltype(api.name)>(dlsym(h, sym));    \
  if (!api.name) {                                                   \
    api.error = std::string("NCCL symbol missing: ") + sym;          \
    api.h = nullptr;                                                 \
    return;                                                          \
  }
    LOAD(GetUniqueId, "ncclGetUniqueId");
    LOAD(CommInitRank, "ncclCommInitRank");
    LOAD(CommAbort, "ncclCommAbort");
    LOAD(CommDestroy, "ncclCommDestroy");
    LOAD(AllReduce, "ncclAllReduce");
    LOAD(AllGather, "ncclAllGather");
    LOAD(GetErrorString, "ncclGetErrorString");
    LOAD(GetVersion, "ncclGetVersion");
#undef LOAD
  });
  return api.h ? &api : nullptr;
}

int nccl_fail(shd_ctx* ctx, ncclResult_t r, const char* what) {
  NcclApi* a = nccl_api();
  std::string m = std::string(what) + ": " + (a ? a->GetErrorString(r) : "NCCL unavailable");
  return shd_fail(ctx, SHD_ERR_NCCL, m);
}

}  // namespace

extern "C" int shd_tp_unique_id(void* out_128_bytes) {
  if (!out_128_bytes) return SHD_ERR_ARG;
  NcclApi* a = nccl_api();
  if (!a) return SHD_ERR_NCCL;
  ncclUniqueId id;
  if (a->GetUniqueId(&id) != ncclSuccess) return SHD_ERR_NCCL;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out_128_bytes, &id, 128);
  return SHD_OK;
}

extern "C" int shd_tp_init(shd_ctx* ctx, int rank, int world, const void* unique_id_128_bytes) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, world >= 1 && rank >= 0 && rank < world, "shd_tp_init: bad rank/world");
  SHD_REQUIRE(ctx, unique_id_128_bytes || world == 1, "shd_tp_init: null unique id");
  SHD_REQUIRE(ctx, ctx->nccl_comm == nullptr, "shd_tp_init: already initialised");
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  if (world == 1) return SHD_OK;
  NcclApi* a = nccl_api();
  if (!a) return shd_fail(ctx, SHD_ERR_NCCL, "shd_tp_init: NCCL could not be loaded (libnccl.so.2)");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId id;
  std::memcpy(&id, unique_id_128_bytes, 128);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = a->CommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclCommInitRank");
  ctx->nccl_comm = comm;
  return SHD_OK;
}

extern "C" int shd_tp_destroy(shd_ctx* ctx) {
  if (!ctx) return SHD_ERR_ARG;
  if (ctx->nccl_comm) {
    NcclApi* a = nccl_api();
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (a) a->CommDestroy(static_cast<ncclComm_t>(ctx->nccl_comm));
    ctx->nccl_comm = nullptr;
  }
  ctx->tp_world = 1;
  ctx->tp_rank = 0;
  return SHD_OK;
}

// Host-side bounded wait on a stream; on timeout the communicator is aborted so that the
// collective in flight errors out instead of hanging, and SHD_ERR_TIMEOUT is returned.
int shd_wait_stream(shd_ctx* ctx, cudaStream_t s, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return SHD_OK;
    if (e != cudaErrorNotReady) return shd_cuda_fail(ctx, e, "stream");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms > 0 && ms > timeout_ms) {
      if (ctx->nccl_comm) {
        NcclApi* a = nccl_api();
        if (a) a->CommAbort(static_cast<ncclComm_t>(ctx->nccl_comm));
        ctx->nccl_comm = nullptr;
      }
      return shd_fail(ctx, SHD_ERR_TIMEOUT, "collective did not complete within the timeout; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// shd_allreduce_shares: in-place sum of n floats over the TP group (both shares packed in buf),
// bounded by timeout_ms (<= 0: no bound).
extern "C" int shd_allreduce_shares(shd_ctx* ctx, float* buf, size_t n, int timeout_ms) {
  if (!ctx) return SHD_ERR_ARG;
  if (ctx->tp_world <= 1 || n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, buf && ctx->nccl_comm, "shd_allreduce_shares: not initialised");
  NcclApi* a = nccl_api();
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const ncclResult_t r = a->AllReduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(ctx->nccl_comm), ctx->stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce");
  return shd_wait_stream(ctx, ctx->stream, timeout_ms);
}

int shd_model::allreduce_sum(float* buf, size_t n) {
  if (ctx->tp_world <= 1) return SHD_OK;
  NcclApi* a = nccl_api();
  const ncclResult_t r = a->AllReduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(ctx->nccl_comm), stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce(shares)");
  return SHD_OK;
}

int shd_model::allreduce_max_keys(int M) {
  if (ctx->tp_world <= 1) return SHD_OK;
  NcclApi* a = nccl_api();
  const ncclResult_t r = a->AllReduce(amax, amax, (size_t)M, ncclUint64, ncclMax, static_cast<ncclComm_t>(ctx->nccl_comm), stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce(argmax keys)");
  return SHD_OK;
}

// Logit shares of the whole vocabulary to the host on every rank.
int shd_model::gather_logits(float* lc_host, float* ls_host) {
  if (ctx->tp_world <= 1) {
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(lc_host, LOGbuf, (size_t)V * 4, cudaMemcpyDeviceToHost, stream));
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(ls_host, LOGbuf + V, (size_t)V * 4, cudaMemcpyDeviceToHost, stream));
    return SHD_OK;
  }
  const int W = ctx->tp_world;
  const size_t cnt = ((size_t)cfg.vocab + W - 1) / W;  // padded per-rank count
  if (!gather_buf) {
    SHD_CHECK_CUDA(ctx, cudaMalloc(&gather_buf, (2 * cnt + 2 * cnt * W) * 4));
    owned.push_back(gather_buf);
  }
  float* send = gather_buf;
  float* recv = gather_buf + 2 * cnt;
  SHD_CHECK_CUDA(ctx, cudaMemsetAsync(send, 0, 2 * cnt * 4, stream));
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(send, LOGbuf, (size_t)V * 4, cudaMemcpyDeviceToDevice, stream));
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(send + cnt, LOGbuf + V, (size_t)V * 4, cudaMemcpyDeviceToDevice, stream));
  NcclApi* a = nccl_api();
  const ncclResult_t r = a->AllGather(send, recv, 2 * cnt, ncclFloat32, static_cast<ncclComm_t>(ctx->nccl_comm), stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllGather(logits)");
  // rank r's rows start at its vocab_begin; counts follow the plan of make_plan()
  for (int rr = 0; rr < W; ++rr) {
    const int b0 = (int)((long long)cfg.vocab * rr / W);
    const int cnt_r = (rr == W - 1) ? cfg.vocab - b0 : (int)((long long)cfg.vocab * (rr + 1) / W) - b0;
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(lc_host + b0, recv + (size_t)rr * 2 * cnt, (size_t)cnt_r * 4, cudaMemcpyDeviceToHost, stream));
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(ls_host + b0, recv + (size_t)rr * 2 * cnt + cnt, (size_t)cnt_r * 4, cudaMemcpyDeviceToHost, stream));
  }
  return SHD_OK;
}
