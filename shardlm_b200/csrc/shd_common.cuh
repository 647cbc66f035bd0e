// Shared device/host helpers for libshardlm_cuda: PTX wrappers for mbarriers and bulk (TMA) copies,
// bounded waits, the Philox counter generator, and the context structure.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/shardlm_cuda.h"

// ------------------------------------------------------------------------------------------------
// Device error word bits (written by kernels, read and cleared by shd_sync).
// ------------------------------------------------------------------------------------------------
#define SHD_DEVERR_TIMEOUT_FULL 0x1u   // consumer gave up waiting for a stage to fill
#define SHD_DEVERR_TIMEOUT_EMPTY 0x2u  // producer gave up waiting for a stage to drain
#define SHD_DEVERR_TIMEOUT_DRAIN 0x4u  // abort path gave up waiting for copies in flight
#define SHD_DEVERR_NONFINITE 0x8u      // greedy argmax saw NaN (the reference's unwrap panics)
#define SHD_DEVERR_ARG 0x10u           // device-side argument check failed (index out of range)

// A bounded wait gives up after this many nanoseconds of %globaltimer.
#define SHD_WAIT_LIMIT_NS 2000000000ull

struct shd_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  int* d_err = nullptr;          // device error word (SHD_DEVERR_* bits)
  float* d_partials = nullptr;   // split-K partial tiles
  size_t partial_floats = 0;
  int* d_counters = nullptr;     // per-tile arrival counters, left zero by every kernel
  int n_counters = 0;
  unsigned long long* d_scratch64 = nullptr;  // one word for synchronous result checks (encoders)
  void* d_stage = nullptr;  // staging of the synchronous per-call entry points (metadata, OT queries)
  size_t stage_bytes = 0;
  int num_sms = 148;
  int64_t launches = 0;
  // RoPE table (host-built with libm, as the reference's RopeFrequencies::new)
  float* d_rope_cos = nullptr;
  float* d_rope_sin = nullptr;
  int rope_head_dim = 0;
  int rope_max_seq = 0;
  float rope_theta = 0.f;
  // staging for activations whose rows are not 16-byte aligned (in_features % 4 != 0)
  void* d_xpad = nullptr;
  size_t xpad_bytes = 0;
  // split partials of the decode attention kernel
  // bf16 activation planes of the tensor-core linear
  void* d_tc_planes = nullptr;
  size_t tc_planes_elems = 0;
  void* d_tc_planes_next = nullptr;  // planes a producer writes for the next linear while this one reads
  size_t tc_planes_next_elems = 0;
  float* d_tc_ws = nullptr;  // split-K partial sums of the tensor-core linear
  size_t tc_ws_floats = 0;
  // NCCL (tensor parallelism), loaded at run time
  void* nccl_comm = nullptr;
  int tp_rank = 0, tp_world = 1;
  // NVLink one-shot all-reduce for decode-sized messages: a receive buffer per rank, mapped into
  // every rank through CUDA IPC (layout in shd_tp.cu); null when unavailable (NCCL is used instead)
  void* p2p_local = nullptr;
  void* p2p_peer[8] = {};
  size_t p2p_slot_bytes = 0;
};

int shd_fail(shd_ctx* ctx, int code, const std::string& msg);
int shd_cuda_fail(shd_ctx* ctx, cudaError_t e, const char* what);
// Device staging of at least `bytes` owned by the context, grown when needed (after the stream has
// drained); for entry points that synchronize before returning, so calls never overlap on it.
int shd_stage(shd_ctx* ctx, size_t bytes, void** out);

#define SHD_CHECK_CUDA(ctx, call)                                    \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess) return shd_cuda_fail((ctx), _e, #call);  \
  } while (0)

#define SHD_CHECK_LAUNCH(ctx, what)                                 \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) return shd_cuda_fail((ctx), _e, (what)); \
    (ctx)->launches++;                                              \
  } while (0)

#define SHD_REQUIRE(ctx, cond, msg) \
  do {                              \
    if (!(cond)) return shd_fail((ctx), SHD_ERR_ARG, (msg)); \
  } while (0)

static inline bool shd_aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ------------------------------------------------------------------------------------------------
// PTX wrappers (sm_100a). Bulk copies are the non-tensor cp.async.bulk form, without multicast.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete. Returns false when SHD_WAIT_LIMIT_NS of
// wall time passed first; the caller records the error and leaves the pipeline.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) return false;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy completing on `bar`. dst, src 16-byte aligned; bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 16-byte asynchronous global -> shared copy through L2 (cp.async.cg); `src_bytes` < 16 zero-fills
// the rest (0: nothing is read). Completion: cp_async_commit() groups, cp_async_wait<N>().
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Named barrier among `nthreads` threads (consumer warps only; id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: a kernel launched with launch_pdl() may start while the previous
// kernel of the stream is still running; pdl_wait() blocks until that kernel has completed and its
// writes are visible (a no-op without a programmatic dependency). Every kernel of this library calls
// pdl_wait() before reading anything another kernel produced; only constant weights are read before.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch timeline (a diagnostic of the captured decode step): each traced launch owns 8 u64 of a
// buffer preset to all ones; every field is an atomic minimum of %globaltimer, the "last" fields of
// its complement, so one launch records its first and last CTA at each point:
//   0 first CTA entry, 1 last CTA entry, 2 first return from the wait on the previous kernel,
//   3 last end of the prologue (the wait, plus the fused norm where there is one), 4 first exit,
//   5 last exit.
enum TraceField { TR_ENTRY = 0, TR_WAIT = 2, TR_READY = 3, TR_EXIT = 4 };
__device__ __forceinline__ void trace_first(unsigned long long* tr, int f) {
  if (tr) atomicMin(tr + f, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void trace_last(unsigned long long* tr, int f) {
  if (tr) atomicMin(tr + f, ~(unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void trace_both(unsigned long long* tr, int f) {
  if (tr) {
    const unsigned long long t = globaltimer_ns();
    atomicMin(tr + f, t);
    atomicMin(tr + f + 1, ~t);
  }
}

#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
#endif

__device__ __forceinline__ float bf16lo_to_f32(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t v) {
  return __uint_as_float(v & 0xffff0000u);
}

// ------------------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC'11). Counter = (block lo, block hi, stream lo, stream hi), key = seed.
// ------------------------------------------------------------------------------------------------
struct u32x4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ u32x4 philox4x32_10(uint64_t block, uint64_t stream,
                                                        uint64_t seed) {
  uint32_t c0 = (uint32_t)block, c1 = (uint32_t)(block >> 32);
  uint32_t c2 = (uint32_t)stream, c3 = (uint32_t)(stream >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c0 = n0;
    c1 = n1;
    c2 = n2;
    c3 = n3;
  }
  return {c0, c1, c2, c3};
}

// Word `idx` of the stream: block idx/4, lane idx%4.
__host__ __device__ __forceinline__ uint32_t philox_word(uint64_t seed, uint64_t stream,
                                                         uint64_t idx) {
  const u32x4 r = philox4x32_10(idx >> 2, stream, seed);
  switch (idx & 3) {
    case 0: return r.x;
    case 1: return r.y;
    case 2: return r.z;
    default: return r.w;
  }
}

// [0,1) with 24 random bits, the construction of rand's Standard f32 ((u >> 8) * 2^-24).
__host__ __device__ __forceinline__ float u32_to_unit_f32(uint32_t u) {
  return (float)(u >> 8) * 5.9604644775390625e-08f;
}

#ifdef __CUDACC__
__device__ __forceinline__ float uniform_f32(uint32_t u, float lo, float hi) {
  return __fadd_rn(lo, __fmul_rn(u32_to_unit_f32(u), __fsub_rn(hi, lo)));
}
#endif
