// Dual-share GEMV family for sm_100a.
//
// One CTA per SM streams a contiguous run of 16 KB weight blocks HBM -> shared memory with
// cp.async.bulk (one producer warp, an S-stage mbarrier ring), and eight consumer warps apply every
// block to BOTH additive shares and all M token rows, so each weight byte is read from HBM once per
// call (the reference reads it twice: two cuBLAS SGEMMs, crates/v2/sharing/src/secure_linear.rs:
// 357-404). Work is the linearised (row tile, K chunk) sequence split evenly over the grid
// ("stream-K"); a tile cut by a CTA boundary is finished by whichever contributor arrives last,
// which sums the partials in CTA order, so results do not depend on timing.
//
// Tiled weight format: block (t, c) holds rows [32t, 32t+32) x columns [256c, 256c+256) as
// [32 rows][256 bf16]; within a row, lane l's 16 bytes are columns {4l..4l+3, 128+4l..128+4l+3},
// so weight and activation shared-memory reads are both conflict-free 16-byte loads.
//
// The consumer inner loop uses packed f32x2 FMAs (two adjacent columns per instruction) for up to 4
// token rows. With the RMSNorm prologue, the activation vector is computed once per CTA into shared
// memory (reconstruct, normalize, reshare) while the producer already streams weights; otherwise
// activation chunks travel with each weight block. Kernels are launched with programmatic
// dependent launch: the producer prefetches weights before the previous kernel has finished.
#include <algorithm>

#include "shd_gemv.cuh"
#include "shd_gemv_dev.cuh"
#include "shd_tc.cuh"

namespace shd {

constexpr int kSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100
// Measured on B200: a pure cp.async.bulk stream sustains ~6.8 TB/s with 4 x 16 KB stages per CTA
// but only ~6.2 TB/s with 12; two or three CTAs per SM with 4-6 stages each reach ~7.1 TB/s.
constexpr int kMaxStages = 6;
constexpr int kSmemPerCta2 = 115712;  // dynamic shared memory per CTA at two CTAs per SM
constexpr int kTailBytes = 4608;    // tile result, barriers, flags, reduction scratch

// Called by all 32 lanes of the producer warp: lane 0 streams the weights; after the wait on the
// previous kernel every lane issues the activation copies of some prefetched stages (each bulk copy
// costs its issuing thread ~0.1 us, so one thread issuing them all delayed the first blocks).
template <int M, int CHUNK, typename XT>
__device__ void gemv_producer(const PipeSmem& sm, const uint8_t* W, const XT* Xc, const XT* Xs,
                              int ldx, int K, int nKC, long long u0, long long u1, bool staged_x,
                              int* err, int lane) {
  const uint64_t pol_w = l2_policy_evict_first();
  const uint64_t pol_x = l2_policy_evict_last();
  const int S = sm.S;
  const long long n = u1 - u0;
  const int npre = (int)std::min<long long>(S, n);
  auto xbytes_of = [&](long long u) -> uint32_t {
    const int c = (int)(u % nKC);
    return (uint32_t)min(CHUNK, K - c * CHUNK) * 4u;
  };
  auto issue_x = [&](int s, long long u) {
    const int c = (int)(u % nKC);
    const uint32_t xb = xbytes_of(u);
    uint8_t* st = sm.stages + (size_t)s * sm.stage_bytes;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      bulk_g2s(st + kBlockBytes + (m * 2 + 0) * (CHUNK * 4), Xc + (size_t)m * ldx + (size_t)c * CHUNK, xb,
               &sm.full[s], pol_x);
      bulk_g2s(st + kBlockBytes + (m * 2 + 1) * (CHUNK * 4), Xs + (size_t)m * ldx + (size_t)c * CHUNK, xb,
               &sm.full[s], pol_x);
    }
  };
  // phase A: weights of the first npre units (no dependency on earlier kernels)
  if (lane == 0) {
    for (int i = 0; i < npre; ++i) {
      const long long u = u0 + i;
      const uint32_t tx = (uint32_t)kBlockBytes + (staged_x ? (uint32_t)(M * 2) * xbytes_of(u) : 0u);
      mbar_arrive_expect_tx(&sm.full[i], tx);
      bulk_g2s(sm.stages + (size_t)i * sm.stage_bytes, W + (size_t)u * kBlockBytes, kBlockBytes, &sm.full[i], pol_w);
    }
  }
  if (staged_x) {
    __syncwarp();  // every stage's expected bytes are set before any lane's copies
    pdl_wait();
    for (int i = lane; i < npre; i += 32) issue_x(i, u0 + i);
  }
  if (lane != 0) return;
  // phase B: the rest, refilling stages as consumers release them
  int s = 0;
  uint32_t ph = 0;  // parity of the empty-barrier phase to wait for
  long long i = npre;
  for (; i < n; ++i) {
    if (!mbar_wait_bounded(&sm.empty[s], ph)) {
      atomicOr(err, SHD_DEVERR_TIMEOUT_EMPTY);
      sm.flags[0] = 1;
      break;
    }
    if (sm.flags[0]) break;
    const long long u = u0 + i;
    const uint32_t tx = (uint32_t)kBlockBytes + (staged_x ? (uint32_t)(M * 2) * xbytes_of(u) : 0u);
    mbar_arrive_expect_tx(&sm.full[s], tx);
    bulk_g2s(sm.stages + (size_t)s * sm.stage_bytes, W + (size_t)u * kBlockBytes, kBlockBytes, &sm.full[s], pol_w);
    if (staged_x) issue_x(s, u);
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
  if (i < n) {
    // Aborted: wait (bounded) for the last copy issued into every stage before leaving, so that no
    // bulk copy lands in shared memory of a CTA that has exited.
    for (long long k = std::max<long long>(0, i - S); k < i; ++k) {
      const int ks = (int)(k % S);
      if (!mbar_wait_bounded(&sm.full[ks], (uint32_t)((k / S) & 1))) atomicOr(err, SHD_DEVERR_TIMEOUT_DRAIN);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// f32-share GEMV kernel (bf16 weights)
// ------------------------------------------------------------------------------------------------
template <int M, int EPI, bool NORM, int MINB>
__global__ void __launch_bounds__(kGemvThreads, MINB) gemv_f32_kernel(const __grid_constant__ GemvArgs a) {
  constexpr bool USE2 = (M <= 4);
  constexpr int V = 4 * 2 * M;
  constexpr int VP = (V <= 8) ? 8 : (V <= 16) ? 16 : (V <= 32) ? 32 : 64;
  constexpr int TSUM = kTileRows * 2 * M;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int S = a.nstages;
  const int KP = a.nKC * kChunkBf16;
  PipeSmem sm;
  sm.stages = smem;
  sm.S = S;
  sm.stage_bytes = kBlockBytes + (NORM ? 0 : M * 2 * kChunkBf16 * 4);
  float* xres = reinterpret_cast<float*>(smem + (size_t)S * sm.stage_bytes);
  float* tsum = xres + (NORM ? (size_t)M * 2 * KP : 0);
  sm.full = reinterpret_cast<uint64_t*>(tsum + TSUM);
  sm.empty = sm.full + S;
  sm.cbar = sm.empty + S;
  sm.flags = reinterpret_cast<volatile int*>(sm.cbar + 2);
  sm.red = reinterpret_cast<float*>(sm.cbar + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = (long long)a.nT * a.nKC;
  const int G = gridDim.x, g = blockIdx.x;
  const long long u0 = unit_begin(U, G, g), u1 = unit_begin(U, G, g + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(sm.cbar, kConsumerWarps);
    sm.flags[0] = 0;
    sm.flags[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // A tensor-parallel push takes the exchange call after the last one whose receive kernel has
    // started: that kernel advanced the call counter before releasing its dependents, and the next
    // receive kernel (which advances it again) cannot start before this kernel releases its own.
    if (a.tp_peer[0]) sm.flags[2] = *reinterpret_cast<const volatile int*>(a.tp_peer[a.tp_me]) + 1;
    pdl_trigger();
    trace_both(a.trace, TR_ENTRY);
  }

  if (warp == kConsumerWarps) {
    gemv_producer<M, kChunkBf16, float>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC, u0, u1, !NORM, a.err, lane);
    return;
  }

  const int ctid = threadIdx.x;  // 0..255 among consumers
  uint32_t cphase = 0;
  NormGamma ngam;
  if constexpr (NORM) norm_gamma_preload(a, ctid, ngam);
  pdl_wait();  // activations, positions and scratch come from earlier kernels
  if (ctid == 0) trace_first(a.trace, TR_WAIT);
  if constexpr (NORM) {
    if (!norm_prologue<M>(a, sm, cphase, xres, KP, ctid, lane, warp, g == 0, &ngam)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
  }
  if (ctid == 0) trace_last(a.trace, TR_READY);

  const int first_tile = (int)(u0 / a.nKC);
  unsigned long long acc2[USE2 ? V : 1];
  float acc[VP];
#pragma unroll
  for (int j = 0; j < VP; ++j) acc[j] = 0.f;
  if constexpr (USE2) {
#pragma unroll
    for (int j = 0; j < V; ++j) acc2[j] = 0ull;
  }

  int t = first_tile, c = (int)(u0 % a.nKC);
  int s = 0;
  uint32_t ph = 0;
  for (long long u = u0; u < u1; ++u) {
    if (!warp_wait(&sm.full[s], ph)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    const uint8_t* st = sm.stages + (size_t)s * sm.stage_bytes;
    const uint4* wv = reinterpret_cast<const uint4*>(st);
    // activation chunk: resident (zero padded) or staged with the block (masked at the K tail)
    const float* xbase;
    int xstride;
    bool okA = true, okB = true;
    if constexpr (NORM) {
      xbase = xres + (size_t)c * kChunkBf16;
      xstride = KP;
    } else {
      xbase = reinterpret_cast<const float*>(st + kBlockBytes);
      xstride = kChunkBf16;
      okA = c * kChunkBf16 + 4 * lane < a.K;
      okB = c * kChunkBf16 + 128 + 4 * lane < a.K;
    }
    mac_block<M, V, VP>(wv, xbase, xstride, okA, okB, warp, lane, acc2, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }

    const int ct = t, cc = c;
    if (++c == a.nKC) {
      c = 0;
      ++t;
    }
    const bool tile_end = (cc == a.nKC - 1) || (u == u1 - 1);
    if (!tile_end) continue;

    // ---- this CTA's contribution to tile ct is complete ----
    tile_reduce<M, V, VP>(acc2, acc, tsum, warp, lane);

    const bool full_tile = ((long long)ct * a.nKC >= u0) && (cc == a.nKC - 1);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    if (!full_tile) {
      const int r = split_tile_close<float>(sm, cphase, tsum, a.partials, a.counters, TSUM, U, G, g, ct,
                                            a.nKC, u0, u1, ctid, lane);
      if (r < 0) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      if (r == 0) continue;
    }
    epilogue_f32<M, EPI>(a, ct, tsum, ctid, a.err, (unsigned)sm.flags[2]);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
  }
  if (ctid == 0) trace_both(a.trace, TR_EXIT);
}

// ------------------------------------------------------------------------------------------------
// Ring (Z_2^32) GEMV kernel (i32 weights): acc = sum x*W in wrapping i64, y = (i32)(acc >> scale).
// Tiled format: block (t, c) = rows [32t, 32t+32) x columns [128c, 128c+128) as [32][128] i32.
// ------------------------------------------------------------------------------------------------
template <int M>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_ring_kernel(const __grid_constant__ RingArgs a) {
  constexpr int V = 4 * 2 * M;  // M in {1, 2, 4, 8}: a power of two
  constexpr int TSUM = kTileRows * 2 * M;
  extern __shared__ __align__(1024) uint8_t smem[];
  PipeSmem sm;
  sm.stages = smem;
  sm.stage_bytes = kBlockBytes + M * 2 * kChunkI32 * 4;
  {
    const int fit = (kSmemLimit - kTailBytes) / sm.stage_bytes;
    sm.S = fit < kMaxStages ? fit : kMaxStages;
  }
  const int S = sm.S;
  long long* tsum = reinterpret_cast<long long*>(smem + (size_t)S * sm.stage_bytes);
  sm.full = reinterpret_cast<uint64_t*>(tsum + TSUM);
  sm.empty = sm.full + S;
  sm.cbar = sm.empty + S;
  sm.flags = reinterpret_cast<volatile int*>(sm.cbar + 2);
  sm.red = reinterpret_cast<float*>(sm.cbar + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = (long long)a.nT * a.nKC;
  const int G = gridDim.x, g = blockIdx.x;
  const long long u0 = unit_begin(U, G, g), u1 = unit_begin(U, G, g + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(sm.cbar, kConsumerWarps);
    sm.flags[0] = 0;
    sm.flags[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == kConsumerWarps) {
    gemv_producer<M, kChunkI32, int32_t>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC, u0, u1, true, a.err, lane);
    return;
  }

  const int ctid = threadIdx.x;
  pdl_wait();
  const int first_tile = (int)(u0 / a.nKC);
  uint32_t cphase = 0;
  long long acc[V];
#pragma unroll
  for (int j = 0; j < V; ++j) acc[j] = 0;

  int t = first_tile, c = (int)(u0 % a.nKC);
  int s = 0;
  uint32_t ph = 0;
  for (long long u = u0; u < u1; ++u) {
    if (!warp_wait(&sm.full[s], ph)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    const uint8_t* st = sm.stages + (size_t)s * sm.stage_bytes;
    const int32_t* xsm = reinterpret_cast<const int32_t*>(st + kBlockBytes);
    const bool ok = c * kChunkI32 + 4 * lane < a.K;
    const int4* wv = reinterpret_cast<const int4*>(st);
    int4 wq[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) wq[r] = wv[(warp * 4 + r) * 32 + lane];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int sh = 0; sh < 2; ++sh) {
        const int4 x = ok ? *reinterpret_cast<const int4*>(xsm + (m * 2 + sh) * kChunkI32 + 4 * lane)
                          : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          long long v = acc[(r * 2 + sh) * M + m];
          v += (long long)wq[r].x * x.x;
          v += (long long)wq[r].y * x.y;
          v += (long long)wq[r].z * x.z;
          v += (long long)wq[r].w * x.w;
          acc[(r * 2 + sh) * M + m] = v;
        }
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
    const int ct = t, cc = c;
    if (++c == a.nKC) {
      c = 0;
      ++t;
    }
    const bool tile_end = (cc == a.nKC - 1) || (u == u1 - 1);
    if (!tile_end) continue;

    int base, cnt;
    unsigned dup;
    warp_reduce_scatter<long long, V>(acc, lane, base, cnt, dup);
    if ((lane & dup) == 0) {
#pragma unroll
      for (int j = 0; j < V; ++j)
        if (j < cnt) tsum[warp * V + base + j] = acc[j];
    }
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = 0;

    const bool full_tile = ((long long)ct * a.nKC >= u0) && (cc == a.nKC - 1);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    if (!full_tile) {
      const int r = split_tile_close<long long>(sm, cphase, tsum, a.partials, a.counters, TSUM, U, G, g, ct,
                                                a.nKC, u0, u1, ctid, lane);
      if (r < 0) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      if (r == 0) continue;
    }
    // epilogue: arithmetic shift of the wrapped 64-bit sum, truncation to i32, wrapping bias add
    for (int idx = ctid; idx < kTileRows * M; idx += kConsumerWarps * 32) {
      const int r = idx % kTileRows, m = idx / kTileRows;
      const int n = ct * kTileRows + r;
      if (n >= a.N) continue;
      const int32_t yc = (int32_t)(tsum[(r * 2 + 0) * M + m] >> a.scale);
      int32_t ys = (int32_t)(tsum[(r * 2 + 1) * M + m] >> a.scale);
      if (a.bias) ys = (int32_t)((uint32_t)ys + (uint32_t)a.bias[n]);
      a.Yc[(size_t)m * a.ldy + n] = yc;
      a.Ys[(size_t)m * a.ldy + n] = ys;
    }
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------------
template <typename Kern>
static int set_smem_attr(shd_ctx* ctx, Kern kernel, unsigned& devices) {
  if (!(devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    devices |= 1u << (ctx->device & 31);
  }
  return SHD_OK;
}

// Grid of a GEMV launch. Stream-K over min(U, per_sm * SMs) CTAs in general; when the weight has at
// most per_sm * SMs row tiles of at most 16 chunks (256 KB), one CTA per tile instead: every CTA
// then streams whole tiles and no tile is split, which removes the split-tile exchange from the
// tail of latency-bound projections (q/k/v, o, and every projection of a tensor-parallel slice).
static int gemv_grid(const shd_ctx* ctx, const shd_weight* w, long long U, int per_sm) {
  const long long cap = (long long)per_sm * ctx->num_sms;
  if (w->nT <= cap && w->nKC <= 16) return w->nT;
  return (int)std::min<long long>(U, cap);
}

// Launch shape of the f32-share GEMV for M rows of `w` (with or without the fused norm).
// Two CTAs per SM (one streams while the other is in its prologue, split-tile exchange or
// epilogue) when at least 4 stages fit in half the shared memory and M <= 2 keeps the registers
// under the two-CTA limit; otherwise one CTA per SM.
// At most one tile per SM: one CTA per SM, with as many stages as the tile has chunks (or as fit
// in shared memory). The whole tile is then in flight at once and most of it loads before the
// wait on the previous kernel, instead of paying one memory latency per 6 chunks after it.
// (Loading the activations whole after the wait, instead of with every block, measured slower:
// the first block then waits for the whole vector.)
// Fewer row tiles than half the SMs (the q/k/v slice of a tensor-parallel rank): one tile per CTA
// would leave most SMs idle and stream a whole tile through each busy one, so the (tile, chunk)
// units are spread over one CTA per SM instead, every unit of a CTA in flight at once, and the
// split tiles are finished by their owners.
GemvPlan gemv_plan(const shd_ctx* ctx, const shd_weight* w, int M, bool norm) {
  GemvPlan p{};
  const int stage = kBlockBytes + (norm ? 0 : M * 2 * kChunkBf16 * 4);
  const size_t xres = norm ? (size_t)M * 2 * w->nKC * kChunkBf16 * 4 : 0;
  const long long U = (long long)w->nT * w->nKC;
  const long long s2 = ((long long)kSmemPerCta2 - kTailBytes - (long long)xres) / stage;
  const long long s1 = ((long long)kSmemLimit - kTailBytes - (long long)xres) / stage;
  const bool few_tiles = 2 * (long long)w->nT < ctx->num_sms && w->nKC >= 4 && s1 >= 2;
  const bool deep_tiles = !few_tiles && w->nT <= ctx->num_sms && w->nKC <= 16 &&
                          s1 >= std::min<long long>(w->nKC, 8);
  p.U = U;
  if (M <= 2 && s2 >= 4 && !deep_tiles && !few_tiles) {
    p.per_sm = 2;
    p.nstages = (int)std::min<long long>(kMaxStages, s2);
    p.G = gemv_grid(ctx, w, U, 2);
  } else {
    p.per_sm = 1;
    p.G = gemv_grid(ctx, w, U, 1);
    long long want = deep_tiles ? std::max(w->nKC, 2) : kMaxStages;
    if (few_tiles) {
      p.G = (int)std::min<long long>(U, ctx->num_sms);
      want = std::max<long long>((U + p.G - 1) / p.G, 2);
    }
    p.nstages = (int)std::min<long long>(want, s1);
  }
  p.smem = (size_t)p.nstages * stage + xres + kTailBytes;
  return p;
}

template <int M, int EPI, bool NORM>
static int launch_f32_t(shd_ctx* ctx, const shd_weight* w, GemvArgs a) {
  static unsigned attr1 = 0, attr2 = 0;
  const GemvPlan p = gemv_plan(ctx, w, M, NORM);
  if (p.nstages < 2) return shd_fail(ctx, SHD_ERR_ARG, "gemv: activation vector too long for the fused norm");
  a.nstages = p.nstages;
  if constexpr (M <= 2) {
    if (p.per_sm == 2) {
      const int rc = set_smem_attr(ctx, gemv_f32_kernel<M, EPI, NORM, 2>, attr2);
      if (rc) return rc;
      SHD_CHECK_CUDA(ctx, launch_pdl(gemv_f32_kernel<M, EPI, NORM, 2>, dim3(p.G), dim3(kGemvThreads), p.smem,
                                     ctx->stream, a));
      ctx->launches++;
      return SHD_OK;
    }
  }
  (void)attr2;
  const int rc = set_smem_attr(ctx, gemv_f32_kernel<M, EPI, NORM, 1>, attr1);
  if (rc) return rc;
  SHD_CHECK_CUDA(ctx, launch_pdl(gemv_f32_kernel<M, EPI, NORM, 1>, dim3(p.G), dim3(kGemvThreads), p.smem,
                                 ctx->stream, a));
  ctx->launches++;
  return SHD_OK;
}

template <int EPI, bool NORM>
static int launch_f32_m(shd_ctx* ctx, const shd_weight* w, int M, GemvArgs a) {
  switch (M) {
    case 1: return launch_f32_t<1, EPI, NORM>(ctx, w, a);
    case 2: return launch_f32_t<2, EPI, NORM>(ctx, w, a);
    case 3: return launch_f32_t<3, EPI, NORM>(ctx, w, a);
    case 4: return launch_f32_t<4, EPI, NORM>(ctx, w, a);
    case 5: return launch_f32_t<5, EPI, NORM>(ctx, w, a);
    case 6: return launch_f32_t<6, EPI, NORM>(ctx, w, a);
    case 7: return launch_f32_t<7, EPI, NORM>(ctx, w, a);
    case 8: return launch_f32_t<8, EPI, NORM>(ctx, w, a);
    default: return shd_fail(ctx, SHD_ERR_ARG, "gemv: M must be 1..8 for one launch");
  }
}

int gemv_prepare(shd_ctx* ctx, const shd_weight* w, GemvArgs& a, bool norm) {
  a.W = reinterpret_cast<const uint8_t*>(w->d_tiles);
  a.N = w->N;
  a.K = (w->K + 3) / 4 * 4;  // x extent copied per row (rows padded to 16 bytes)
  a.nT = w->nT;
  a.nKC = w->nKC;
  a.partials = ctx->d_partials;
  a.counters = ctx->d_counters;
  a.err = ctx->d_err;
  if (w->kind != WK_BF16) return shd_fail(ctx, SHD_ERR_ARG, "gemv: need a bf16 weight");
  if (w->nT > ctx->n_counters) return shd_fail(ctx, SHD_ERR_ARG, "gemv: too many row tiles");
  if (norm) {
    if (w->K % 4 != 0) return shd_fail(ctx, SHD_ERR_ARG, "gemv: fused norm needs in_features % 4 == 0");
    a.K = w->K;
  }
  return SHD_OK;
}

int launch_gemv_f32(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs a, bool norm) {
  const int rc = gemv_prepare(ctx, w, a, norm);
  if (rc) return rc;
  if (norm) {
    switch (epi) {
      case EPI_STORE: return launch_f32_m<EPI_STORE, true>(ctx, w, M, a);
      case EPI_QKV: return launch_f32_m<EPI_QKV, true>(ctx, w, M, a);
      case EPI_GATEUP: return launch_f32_m<EPI_GATEUP, true>(ctx, w, M, a);
      case EPI_LOGITS: return launch_f32_m<EPI_LOGITS, true>(ctx, w, M, a);
      default: return shd_fail(ctx, SHD_ERR_ARG, "gemv: unknown epilogue");
    }
  }
  switch (epi) {
    case EPI_STORE: return launch_f32_m<EPI_STORE, false>(ctx, w, M, a);
    case EPI_QKV: return launch_f32_m<EPI_QKV, false>(ctx, w, M, a);
    case EPI_GATEUP: return launch_f32_m<EPI_GATEUP, false>(ctx, w, M, a);
    case EPI_LOGITS: return launch_f32_m<EPI_LOGITS, false>(ctx, w, M, a);
    default: return shd_fail(ctx, SHD_ERR_ARG, "gemv: unknown epilogue");
  }
}

template <int M>
static int launch_ring_t(shd_ctx* ctx, const shd_weight* w, RingArgs a) {
  static unsigned attr_devices = 0;
  const int rc = set_smem_attr(ctx, gemv_ring_kernel<M>, attr_devices);
  if (rc) return rc;
  const int stage = kBlockBytes + M * 2 * kChunkI32 * 4;
  const int S = std::min(kMaxStages, (kSmemLimit - kTailBytes) / stage);
  const size_t smem = (size_t)S * stage + kTailBytes;
  const long long U = (long long)w->nT * w->nKC;
  const int G = (int)std::min<long long>(U, ctx->num_sms);
  SHD_CHECK_CUDA(ctx, launch_pdl(gemv_ring_kernel<M>, dim3(G), dim3(kGemvThreads), smem, ctx->stream, a));
  ctx->launches++;
  return SHD_OK;
}

int launch_gemv_ring(shd_ctx* ctx, const shd_weight* w, int M, RingArgs a) {
  a.W = reinterpret_cast<const uint8_t*>(w->d_tiles);
  a.N = w->N;
  a.K = (w->K + 3) / 4 * 4;
  a.nT = w->nT;
  a.nKC = w->nKC;
  a.partials = reinterpret_cast<long long*>(ctx->d_partials);
  a.counters = ctx->d_counters;
  a.err = ctx->d_err;
  if (w->nT > ctx->n_counters) return shd_fail(ctx, SHD_ERR_ARG, "gemv: too many row tiles");
  switch (M) {
    case 1: return launch_ring_t<1>(ctx, w, a);
    case 2: return launch_ring_t<2>(ctx, w, a);
    case 4: return launch_ring_t<4>(ctx, w, a);
    case 8: return launch_ring_t<8>(ctx, w, a);
    default: return shd_fail(ctx, SHD_ERR_ARG, "ring gemv: M must be 1, 2, 4 or 8 for one launch");
  }
}

}  // namespace shd

// ------------------------------------------------------------------------------------------------
// C ABI: linear layers
// ------------------------------------------------------------------------------------------------
using namespace shd;

// Copy [M][K] 4-byte rows into [M][K4] rows (K4 = K rounded up to 4, zero tail) so every row
// starts on a 16-byte boundary, as the bulk copies require.
__global__ void pad_rows_kernel(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                                uint32_t* __restrict__ pa, uint32_t* __restrict__ pb, int M, int K,
                                int K4) {
  pdl_wait();
  const long long n = (long long)M * K4;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < n;
       v += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(v / K4), k = (int)(v % K4);
    pa[v] = k < K ? a[(size_t)m * K + k] : 0u;
    pb[v] = k < K ? b[(size_t)m * K + k] : 0u;
  }
}

static int stage_padded(shd_ctx* ctx, const void* xc, const void* xs, int M, int K, int K4,
                        const void** oc, const void** os) {
  const size_t need = (size_t)2 * M * K4 * 4;
  if (need > ctx->xpad_bytes) {
    SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->d_xpad);
    ctx->d_xpad = nullptr;
    ctx->xpad_bytes = 0;
    SHD_CHECK_CUDA(ctx, cudaMalloc(&ctx->d_xpad, need));
    ctx->xpad_bytes = need;
  }
  uint32_t* pa = reinterpret_cast<uint32_t*>(ctx->d_xpad);
  uint32_t* pb = pa + (size_t)M * K4;
  const long long n = (long long)M * K4;
  int grid = (int)std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 8);
  pad_rows_kernel<<<grid < 1 ? 1 : grid, 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint32_t*>(xc), reinterpret_cast<const uint32_t*>(xs), pa, pb, M, K, K4);
  SHD_CHECK_LAUNCH(ctx, "pad_rows_kernel");
  *oc = pa;
  *os = pb;
  return SHD_OK;
}

// Split M into launches of up to 8 rows (the ring kernel takes 1, 2, 4 or 8).
static int next_m(int rem) { return rem >= 8 ? 8 : rem; }
static int next_m_ring(int rem) { return rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : 1; }

extern "C" int shd_linear_dual_f32(shd_ctx* ctx, const shd_weight* w, const float* bias,
                                   const float* xc, const float* xs, float* yc, float* ys, int M,
                                   const float* residual_c, const float* residual_s) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, w && w->kind == WK_BF16, "shd_linear_dual_f32: need a bf16 weight");
  SHD_REQUIRE(ctx, w->rows == SHD_ROWS_PLAIN, "shd_linear_dual_f32: weight must be in plain row order");
  SHD_REQUIRE(ctx, M >= 0, "shd_linear_dual_f32: M < 0");
  if (M == 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && yc && ys, "shd_linear_dual_f32: null share pointer");
  SHD_REQUIRE(ctx, (residual_c == nullptr) == (residual_s == nullptr),
              "shd_linear_dual_f32: residual_c and residual_s must both be set or both null");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  int ldx = w->K;
  if (w->K % 4 != 0 || !shd_aligned16(xc) || !shd_aligned16(xs)) {
    ldx = (w->K + 3) / 4 * 4;
    const void *pc, *ps;
    const int rc = stage_padded(ctx, xc, xs, M, w->K, ldx, &pc, &ps);
    if (rc) return rc;
    xc = reinterpret_cast<const float*>(pc);
    xs = reinterpret_cast<const float*>(ps);
  }
  if (tc_preferred(w, M)) {
    // many rows: the tensor-core path (one pass over the weights for all rows)
    GemvArgs a{};
    a.Xc = xc;
    a.Xs = xs;
    a.ldx = ldx;
    a.bias = bias ? bias : w->d_bias;
    a.Rc = residual_c;
    a.Rs = residual_s;
    a.ldr = w->N;
    a.Yc = yc;
    a.Ys = ys;
    a.ldy = w->N;
    return launch_linear_tc(ctx, w, M, EPI_STORE, a);
  }
  for (int m0 = 0; m0 < M;) {
    const int mm = next_m(M - m0);
    GemvArgs a{};
    a.Xc = xc + (size_t)m0 * ldx;
    a.Xs = xs + (size_t)m0 * ldx;
    a.ldx = ldx;
    a.bias = bias ? bias : w->d_bias;
    a.Rc = residual_c ? residual_c + (size_t)m0 * w->N : nullptr;
    a.Rs = residual_s ? residual_s + (size_t)m0 * w->N : nullptr;
    a.ldr = w->N;
    a.Yc = yc + (size_t)m0 * w->N;
    a.Ys = ys + (size_t)m0 * w->N;
    a.ldy = w->N;
    const int rc = launch_gemv_f32(ctx, w, mm, EPI_STORE, a);
    if (rc) return rc;
    m0 += mm;
  }
  return SHD_OK;
}

extern "C" int shd_linear_dual_ring(shd_ctx* ctx, const shd_weight* w, const int32_t* bias,
                                    const int32_t* xc, const int32_t* xs, int32_t* yc, int32_t* ys,
                                    int M, int scale) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, w && w->kind == WK_I32, "shd_linear_dual_ring: need an i32 ring weight");
  SHD_REQUIRE(ctx, M >= 0, "shd_linear_dual_ring: M < 0");
  SHD_REQUIRE(ctx, scale >= 0 && scale <= 30, "shd_linear_dual_ring: scale outside 0..30 (MAX_SCALE)");
  if (M == 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && yc && ys, "shd_linear_dual_ring: null share pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  int ldx = w->K;
  if (w->K % 4 != 0 || !shd_aligned16(xc) || !shd_aligned16(xs)) {
    ldx = (w->K + 3) / 4 * 4;
    const void *pc, *ps;
    const int rc = stage_padded(ctx, xc, xs, M, w->K, ldx, &pc, &ps);
    if (rc) return rc;
    xc = reinterpret_cast<const int32_t*>(pc);
    xs = reinterpret_cast<const int32_t*>(ps);
  }
  for (int m0 = 0; m0 < M;) {
    const int mm = next_m_ring(M - m0);
    RingArgs a{};
    a.Xc = xc + (size_t)m0 * ldx;
    a.Xs = xs + (size_t)m0 * ldx;
    a.ldx = ldx;
    a.bias = bias ? bias : w->d_bias_i32;
    a.Yc = yc + (size_t)m0 * w->N;
    a.Ys = ys + (size_t)m0 * w->N;
    a.ldy = w->N;
    a.scale = scale;
    const int rc = launch_gemv_ring(ctx, w, mm, a);
    if (rc) return rc;
    m0 += mm;
  }
  return SHD_OK;
}
