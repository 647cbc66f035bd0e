// Tensor parallelism over NVLink: NCCL, loaded at run time (dlopen of libnccl.so.2 -- inside a
// PyTorch process this resolves to the NCCL torch already loaded). All-reduce is linear over
// additive shares, so the client and server partial shares of a row-parallel projection are summed
// by ONE all-reduce of the packed [2][M][h] buffer. Vocabulary-parallel lm_head: the greedy token is
// a max-reduce of (orderable logit, global index) keys. Decode-sized messages and the keys go over
// NVLink peer memory (kernels below), larger ones through NCCL.
//
// The reference has no NCCL at all (crates/v2/core/src/comm.rs:95-136 sums on the host, TODO at
// :105); its only TP is the plaintext DistributedEngine (crates/v2/model/src/distributed.rs:312-624).
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "shd_model.cuh"
#include "shd_tc.cuh"

namespace {

using shd::kP2pCapacity;
using shd::kP2pCtas;
using shd::kP2pHeader;
using shd::kP2pMaxWorld;
using shd::kP2pSlotBytes;
using shd::kP2pThreads;
using shd::p2p_slot;

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

// ------------------------------------------------------------------------------------------------
// NVLink one-shot all-reduce (sum of f32 shares) for decode-sized messages; buffer layout, epochs
// and slot reuse in shd_p2p.cuh.
//
// Two forms. p2p_allreduce_kernel: every CTA stores its slice of the local partial shares into
// slot (parity, own rank) of EVERY rank (plain peer stores), then polls its slice of the slots of
// all sources and sums them in rank order 0..world-1 -- the same order on every rank, so all ranks
// hold identical sums. Fused form: the row-parallel GEMV's epilogue pushes each finished tile
// itself (GemvArgs::tp_peer), and p2p_recv_kernel only polls and sums; it starts polling as soon as
// it is resident, before the wait on the GEMV, and writes the sums after that wait (earlier
// kernels may still read the buffer until then).
// Call counters: p2p_allreduce_kernel advances its CTA's counter at its end and does not release
// its dependents early. p2p_recv_kernel advances it at its START, fenced, before releasing its
// dependents (the next GEMV's CTAs then stream their weights while the exchange completes): every
// later kernel is launched only after all of this kernel's CTAs released, so it reads the advanced
// counter. A pushing GEMV reads it at its start, before releasing its own dependents, since the
// next receive kernel advances it as soon as it is released. Slot reuse stays safe because a rank
// pushes call c + 2 only after its wait, i.e. after its receive of c + 1 completed, which needed
// every peer's push of c + 1, which each made after its own receive of c completed.
// ------------------------------------------------------------------------------------------------
constexpr int kP2pPer = (int)(kP2pCapacity / ((size_t)kP2pCtas * kP2pThreads));  // values per thread
static_assert(kP2pPer % 2 == 0, "values per thread come in pairs");

struct P2pArgs {
  float* buf;        // local partial shares in (allreduce form), sums out
  unsigned long long* keys;  // max-keys form: local keys in, the maximum over ranks out
  size_t n;          // values (keys)
  uint8_t* peer[kP2pMaxWorld];  // every rank's receive buffer (peer[me] = local)
  int me, world;
  int* err;
  unsigned long long* trace;  // launch timeline slot (nullable; TraceField in shd_common.cuh)
};

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// This CTA's call counter: written only by CTA blockIdx.x of earlier exchanges, all complete.
__device__ __forceinline__ int* p2p_counter(const P2pArgs& a) {
  return reinterpret_cast<int*>(a.peer[a.me]) + blockIdx.x;
}

// Value k of this thread: index base + k * (all threads of the launch).
__device__ __forceinline__ size_t p2p_index(int k) {
  return (size_t)blockIdx.x * kP2pThreads + threadIdx.x + (size_t)k * kP2pCtas * kP2pThreads;
}

// Poll this thread's values in the slots of every source until all carry `epoch`, two values at a
// time with every source's word loaded together, and sum each in rank order into acc. False when
// the wait outlives the limit.
__device__ bool p2p_collect(const P2pArgs& a, unsigned epoch, float (&acc)[kP2pPer]) {
  const unsigned long long* slot0 = p2p_slot(a.peer[a.me], (int)(epoch & 1u), a.world, 0);
  const size_t stride = kP2pSlotBytes / 8;
  const unsigned long long tag = (unsigned long long)epoch << 32;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll
  for (int k = 0; k < kP2pPer; k += 2) {
    const size_t i0 = p2p_index(k), i1 = p2p_index(k + 1);
    if (i0 >= a.n) break;
    const bool has1 = i1 < a.n;
    unsigned long long v0[kP2pMaxWorld], v1[kP2pMaxWorld];
#pragma unroll
    for (int r = 0; r < kP2pMaxWorld; ++r) {
      v0[r] = (r < a.world) ? ld_volatile_u64(slot0 + r * stride + i0) : tag;
      v1[r] = (r < a.world && has1) ? ld_volatile_u64(slot0 + r * stride + i1) : tag;
    }
    while (true) {
      bool all = true;
#pragma unroll
      for (int r = 0; r < kP2pMaxWorld; ++r) {
        if ((unsigned)(v0[r] >> 32) != epoch) {
          all = false;
          v0[r] = ld_volatile_u64(slot0 + r * stride + i0);
        }
        if ((unsigned)(v1[r] >> 32) != epoch) {
          all = false;
          v1[r] = ld_volatile_u64(slot0 + r * stride + i1);
        }
      }
      if (all) break;
      if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) return false;
      __nanosleep(64);  // polls share the SM with a GEMV still running beside this CTA
    }
    float s0 = __uint_as_float((unsigned)v0[0]), s1 = __uint_as_float((unsigned)v1[0]);
#pragma unroll
    for (int r = 1; r < kP2pMaxWorld; ++r)
      if (r < a.world) {
        s0 = __fadd_rn(s0, __uint_as_float((unsigned)v0[r]));
        s1 = __fadd_rn(s1, __uint_as_float((unsigned)v1[r]));
      }
    acc[k] = s0;
    acc[k + 1] = s1;
  }
  return true;
}

__device__ __forceinline__ void p2p_finish(const P2pArgs& a, const float (&acc)[kP2pPer], bool ok) {
  if (ok) {
#pragma unroll
    for (int k = 0; k < kP2pPer; ++k) {
      const size_t i = p2p_index(k);
      if (i < a.n) a.buf[i] = acc[k];
    }
  } else {
    atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
  }
}

__global__ void __launch_bounds__(kP2pThreads) p2p_allreduce_kernel(const __grid_constant__ P2pArgs a) {
  const unsigned epoch = (unsigned)*reinterpret_cast<const volatile int*>(p2p_counter(a)) + 1u;
  pdl_wait();  // the partial shares come from the previous kernel
  const unsigned long long tag = (unsigned long long)epoch << 32;
  const int p = (int)(epoch & 1u);
#pragma unroll
  for (int k = 0; k < kP2pPer; ++k) {
    const size_t i = p2p_index(k);
    if (i >= a.n) break;
    const unsigned long long v = tag | __float_as_uint(a.buf[i]);
    for (int q = 0; q < a.world; ++q) st_volatile_u64(p2p_slot(a.peer[q], p, a.world, a.me) + i, v);
  }
  float acc[kP2pPer];
  const bool ok = p2p_collect(a, epoch, acc);
  p2p_finish(a, acc, ok);
  __syncthreads();  // every thread of the CTA has read the counter
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(p2p_counter(a)) = (int)epoch;
}

__global__ void __launch_bounds__(kP2pThreads) p2p_recv_kernel(const __grid_constant__ P2pArgs a) {
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) {
    trace_both(a.trace, TR_ENTRY);
    const unsigned e = (unsigned)*reinterpret_cast<const volatile int*>(p2p_counter(a)) + 1u;
    *reinterpret_cast<volatile int*>(p2p_counter(a)) = (int)e;
    __threadfence();  // the advanced counter is visible before any dependent is released
    s_epoch = e;
    pdl_trigger();
  }
  __syncthreads();
  const unsigned epoch = s_epoch;
  // polling needs nothing from the previous kernel: only values tagged with this call's epoch count
  float acc[kP2pPer];
  const bool ok = p2p_collect(a, epoch, acc);
  if (threadIdx.x == 0) trace_last(a.trace, TR_READY);
  pdl_wait();  // kernels before the pushing GEMV may read the output buffer until it completes
  if (threadIdx.x == 0) trace_first(a.trace, TR_WAIT);
  p2p_finish(a, acc, ok);
  if (threadIdx.x == 0) trace_both(a.trace, TR_EXIT);
}

// Max-reduce of n greedy keys ((orderable logit bits) << 32 | vocabulary index) over the ranks, the
// vocabulary-parallel lm_head's argmax. A key does not fit one {value, epoch} word, so it travels as
// two: word 2i holds its high half, word 2i + 1 its low half, each tagged with the call's epoch. The
// call takes the same counter steps as p2p_allreduce_kernel (read at the start, advanced at the end,
// dependents not released early), so it interleaves with the other exchanges under one epoch
// sequence; only CTA 0 has keys to move (n <= kP2pThreads).
__global__ void __launch_bounds__(kP2pThreads) p2p_maxkeys_kernel(const __grid_constant__ P2pArgs a) {
  const unsigned epoch = (unsigned)*reinterpret_cast<const volatile int*>(p2p_counter(a)) + 1u;
  pdl_wait();  // the keys come from the lm_head kernel
  const unsigned long long tag = (unsigned long long)epoch << 32;
  const int p = (int)(epoch & 1u);
  const int i = threadIdx.x;
  if (blockIdx.x == 0 && i < (int)a.n) {
    const unsigned long long key = a.keys[i];
    const unsigned long long hi = tag | (key >> 32), lo = tag | (key & 0xffffffffull);
    for (int q = 0; q < a.world; ++q) {
      unsigned long long* dst = p2p_slot(a.peer[q], p, a.world, a.me);
      st_volatile_u64(dst + 2 * i, hi);
      st_volatile_u64(dst + 2 * i + 1, lo);
    }
    const unsigned long long* slot0 = p2p_slot(a.peer[a.me], p, a.world, 0);
    const size_t stride = kP2pSlotBytes / 8;
    unsigned long long best = 0ull;
    bool ok = true;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < a.world && ok; ++r) {
      unsigned long long h, l;
      while (true) {
        h = ld_volatile_u64(slot0 + r * stride + 2 * i);
        l = ld_volatile_u64(slot0 + r * stride + 2 * i + 1);
        if ((unsigned)(h >> 32) == epoch && (unsigned)(l >> 32) == epoch) break;
        if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
      const unsigned long long k = ((h & 0xffffffffull) << 32) | (l & 0xffffffffull);
      best = k > best ? k : best;
    }
    if (ok)
      a.keys[i] = best;
    else
      atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
  }
  __syncthreads();  // every thread of the CTA has read the counter
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(p2p_counter(a)) = (int)epoch;
}

int p2p_setup(shd_ctx* ctx) {
  NcclApi* api = nccl_api();
  const int W = ctx->tp_world;
  if (W > kP2pMaxWorld) return SHD_OK;  // NCCL only
  // Every rank takes part in both collectives below whatever happens locally (a rank that left
  // early would leave the others waiting); a local failure only votes the peer path off.
  bool ok = true;
  const size_t bytes = kP2pHeader + (size_t)2 * W * kP2pSlotBytes;
  void* local = nullptr;
  cudaIpcMemHandle_t mine;
  std::memset(&mine, 0, sizeof(mine));
  if (cudaMalloc(&local, bytes) != cudaSuccess) {
    local = nullptr;
    ok = false;
  } else if (cudaMemset(local, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
             cudaIpcGetMemHandle(&mine, local) != cudaSuccess) {
    ok = false;
  }
  cudaGetLastError();
  // exchange the handles with an NCCL all-gather
  void* d_handles = nullptr;
  if (cudaMalloc(&d_handles, (size_t)W * sizeof(cudaIpcMemHandle_t)) != cudaSuccess) {
    if (local) cudaFree(local);
    return shd_fail(ctx, SHD_ERR_CUDA, "p2p setup: handle buffer");
  }
  cudaMemcpy(static_cast<uint8_t*>(d_handles) + (size_t)ctx->tp_rank * sizeof(mine), &mine, sizeof(mine),
             cudaMemcpyHostToDevice);
  const ncclResult_t r = api->AllGather(static_cast<uint8_t*>(d_handles) + (size_t)ctx->tp_rank * sizeof(mine),
                                        d_handles, sizeof(mine), ncclUint8, static_cast<ncclComm_t>(ctx->nccl_comm),
                                        ctx->stream);
  std::vector<cudaIpcMemHandle_t> all(W);
  if (r == ncclSuccess) {
    cudaStreamSynchronize(ctx->stream);
    cudaMemcpy(all.data(), d_handles, (size_t)W * sizeof(mine), cudaMemcpyDeviceToHost);
  }
  cudaFree(d_handles);
  if (r != ncclSuccess) {
    if (local) cudaFree(local);
    return nccl_fail(ctx, r, "p2p setup: handle exchange");
  }
  for (int q = 0; q < W && ok; ++q) {
    if (q == ctx->tp_rank) {
      ctx->p2p_peer[q] = local;
      continue;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      ok = false;
      cudaGetLastError();
    }
    ctx->p2p_peer[q] = ptr;
  }
  // every rank must agree on whether the peer path is used: all-reduce the outcome
  int* d_ok = nullptr;
  int h_ok = ok ? 1 : 0;
  if (cudaMalloc(&d_ok, 4) == cudaSuccess) {
    cudaMemcpy(d_ok, &h_ok, 4, cudaMemcpyHostToDevice);
    if (api->AllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(ctx->nccl_comm), ctx->stream) ==
        ncclSuccess) {
      cudaStreamSynchronize(ctx->stream);
      cudaMemcpy(&h_ok, d_ok, 4, cudaMemcpyDeviceToHost);
    } else {
      h_ok = 0;
    }
    cudaFree(d_ok);
  } else {
    h_ok = 0;
  }
  if (!h_ok) {
    for (int q = 0; q < W; ++q)
      if (q != ctx->tp_rank && ctx->p2p_peer[q]) cudaIpcCloseMemHandle(ctx->p2p_peer[q]);
    for (int q = 0; q < kP2pMaxWorld; ++q) ctx->p2p_peer[q] = nullptr;
    if (local) cudaFree(local);
    return SHD_OK;
  }
  ctx->p2p_local = local;
  ctx->p2p_slot_bytes = kP2pSlotBytes;
  return SHD_OK;
}

void p2p_teardown(shd_ctx* ctx) {
  if (!ctx->p2p_local) return;
  for (int q = 0; q < ctx->tp_world && q < kP2pMaxWorld; ++q)
    if (q != ctx->tp_rank && ctx->p2p_peer[q]) cudaIpcCloseMemHandle(ctx->p2p_peer[q]);
  cudaFree(ctx->p2p_local);
  ctx->p2p_local = nullptr;
  for (int q = 0; q < kP2pMaxWorld; ++q) ctx->p2p_peer[q] = nullptr;
}

// Sum n floats of buf over the TP group on `stream`: the peer path when it is set up and the
// message fits a slot (decode), NCCL otherwise.
int allreduce_f32(shd_ctx* ctx, float* buf, size_t n, cudaStream_t stream) {
  if (ctx->p2p_local && n <= kP2pCapacity) {
    P2pArgs a{};
    a.buf = buf;
    a.n = n;
    for (int q = 0; q < ctx->tp_world; ++q) a.peer[q] = static_cast<uint8_t*>(ctx->p2p_peer[q]);
    a.me = ctx->tp_rank;
    a.world = ctx->tp_world;
    a.err = ctx->d_err;
    SHD_CHECK_CUDA(ctx, launch_pdl(p2p_allreduce_kernel, dim3(kP2pCtas), dim3(kP2pThreads), 0, stream, a));
    ctx->launches++;
    return SHD_OK;
  }
  NcclApi* api = nccl_api();
  const ncclResult_t r = api->AllReduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(ctx->nccl_comm), stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce(shares)");
  return SHD_OK;
}

// Receive half of the fused exchange: the previous kernel (a GEMV with push fields) has pushed this
// rank's partial shares; sum every rank's into buf.
int allreduce_recv_f32(shd_ctx* ctx, float* buf, size_t n, cudaStream_t stream,
                       unsigned long long* trace = nullptr) {
  P2pArgs a{};
  a.trace = trace;
  a.buf = buf;
  a.n = n;
  for (int q = 0; q < ctx->tp_world; ++q) a.peer[q] = static_cast<uint8_t*>(ctx->p2p_peer[q]);
  a.me = ctx->tp_rank;
  a.world = ctx->tp_world;
  a.err = ctx->d_err;
  SHD_CHECK_CUDA(ctx, launch_pdl(p2p_recv_kernel, dim3(kP2pCtas), dim3(kP2pThreads), 0, stream, a));
  ctx->launches++;
  return SHD_OK;
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
  return p2p_setup(ctx);
}

extern "C" int shd_tp_peer_path(const shd_ctx* ctx) { return (ctx && ctx->p2p_local) ? 1 : 0; }

extern "C" int shd_tp_destroy(shd_ctx* ctx) {
  if (!ctx) return SHD_ERR_ARG;
  if (ctx->nccl_comm) {
    NcclApi* a = nccl_api();
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    p2p_teardown(ctx);
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
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const int rc = allreduce_f32(ctx, buf, n, ctx->stream);
  if (rc) return rc;
  return shd_wait_stream(ctx, ctx->stream, timeout_ms);
}

int shd_model::allreduce_sum(float* buf, size_t n) {
  if (ctx->tp_world <= 1) return SHD_OK;
  return allreduce_f32(ctx, buf, n, stream);
}

// A row-parallel GEMV of M rows of w pushes its tiles to the peers itself when the peer path is up,
// the n-value message fits a slot and the GEMV (not the tensor-core linear) runs it; then fill g's
// push fields. allreduce_recv completes the sum.
bool shd_model::tp_push(shd::GemvArgs& g, const shd_weight* w, int M, size_t n) {
  if (ctx->tp_world <= 1 || !ctx->p2p_local || ctx->tp_world > kP2pMaxWorld || n > kP2pCapacity ||
      shd::tc_preferred(w, M))
    return false;
  for (int q = 0; q < ctx->tp_world; ++q) g.tp_peer[q] = static_cast<uint8_t*>(ctx->p2p_peer[q]);
  g.tp_me = ctx->tp_rank;
  g.tp_world = ctx->tp_world;
  return true;
}

int shd_model::allreduce_recv(float* buf, size_t n) {
  return allreduce_recv_f32(ctx, buf, n, stream, trace_slot(6));
}

int shd_model::allreduce_max_keys(int M) {
  if (ctx->tp_world <= 1) return SHD_OK;
  if (ctx->p2p_local && M <= kP2pThreads && (size_t)2 * M <= kP2pCapacity) {
    // over the peer-memory slots: no NCCL kernel in the decode step
    P2pArgs p{};
    p.keys = amax;
    p.n = (size_t)M;
    for (int q = 0; q < ctx->tp_world; ++q) p.peer[q] = static_cast<uint8_t*>(ctx->p2p_peer[q]);
    p.me = ctx->tp_rank;
    p.world = ctx->tp_world;
    p.err = ctx->d_err;
    SHD_CHECK_CUDA(ctx, launch_pdl(p2p_maxkeys_kernel, dim3(kP2pCtas), dim3(kP2pThreads), 0, stream, p));
    ctx->launches++;
    return SHD_OK;
  }
  NcclApi* a = nccl_api();
  const ncclResult_t r = a->AllReduce(amax, amax, (size_t)M, ncclUint64, ncclMax, static_cast<ncclComm_t>(ctx->nccl_comm), stream);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce(argmax keys)");
  return SHD_OK;
}

// Logit shares of the whole vocabulary to the host on every rank.
int shd_model::gather_logits(float* lc_host, float* ls_host, const float* src_c, const float* src_s) {
  if (!src_c) {
    src_c = LOGbuf;
    src_s = LOGbuf + V;
  }
  if (ctx->tp_world <= 1) {
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(lc_host, src_c, (size_t)V * 4, cudaMemcpyDeviceToHost, stream));
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(ls_host, src_s, (size_t)V * 4, cudaMemcpyDeviceToHost, stream));
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
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(send, src_c, (size_t)V * 4, cudaMemcpyDeviceToDevice, stream));
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(send + cnt, src_s, (size_t)V * 4, cudaMemcpyDeviceToDevice, stream));
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
