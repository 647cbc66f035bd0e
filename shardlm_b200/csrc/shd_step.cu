// Persistent decode step for sm_100a: one launch per generated token (decode engine 1).
//
// The per-kernel decode path (shd_model.cu, engine 0) launches ~5 kernels per layer chained by
// programmatic dependent launch. Here the CTAs (one or two per SM, all resident) stay for the whole
// step and work through a job list: embedding shares, then per layer RMSNorm + q/k/v + RoPE + KV
// write, attention, o, RMSNorm + gate/up + SwiGLU, down, then final norm + lm_head + argmax and the
// token update.
//
//  * the producer warp streams the weight blocks of every GEMV job of the step through one
//    cp.async.bulk ring, in job order, gated only by free ring slots: weights do not depend on
//    activations, so it runs ahead across job boundaries while the consumers wait at a barrier, run
//    attention or finish a split tile;
//  * activations that travel with a weight block (staged x of the o and down projections) are
//    copied only once the job's inputs are complete (grid-barrier count observed, acquire fence,
//    then a proxy fence for the bulk-copy engine); the block's weight copy is already in flight;
//  * the eight consumer warps run each job after a grid barrier on the previous one: the GEMV
//    blocks with the same multiply-accumulate, split-tile close and epilogues as the per-kernel
//    path; attention as (row, head group, position split) items whose partials split 0's CTA
//    combines in split order; embedding and standalone norms as grid-strided loops.
//
// Measured on B200 (7B, batch 1) this engine is slower than engine 0 (~260 vs ~330 tok/s): the five
// grid barriers per layer and the latency-bound small jobs (q/k/v, o, attention) leave HBM idle for
// longer than the ring can cover, and prefetching further ahead into L2 lowered the streaming rate.
//
// Every wait is bounded (%globaltimer); a CTA that gives up raises the abort flag, which every other
// wait polls, so a failed step ends with an error word instead of a hang. All CTAs must be resident
// at once: the launch uses the cooperative launch attribute and checks the occupancy first.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "shd_gemv_dev.cuh"
#include "shd_step.cuh"

namespace shd {

namespace {

constexpr int kStepMaxStages = 6;
constexpr int kStepTail = 4608;  // tsum (<= 2 KB at M = 8), ring barriers, flags, reduction scratch
constexpr int kStepSmemLimit = 232448 - 1024;  // dynamic shared memory; the rest holds the job arguments
constexpr int kStepSmemPerCta2 = 115712 - 1024;  // the same at two CTAs per SM
constexpr int kATile = 16;   // attention positions per tile (lanes 16..31 idle in the score phase)
constexpr int kAGroup = 4;   // query heads per attention item (one kv head)
constexpr int kANW = kConsumerWarps;
constexpr int kAThreads = kConsumerWarps * 32;

template <int HD>
struct AttnTile {
  static constexpr int KS = HD + 4;  // padded K row stride (conflict-free column reads)
  float k[kATile][KS];
  float v[kATile][HD];
  float q[kAGroup][HD];
  float spart[kANW][kAGroup][32];
  float p[kAGroup][32];
  float m[kAGroup], l[kAGroup], alpha[kAGroup];
  int last;
};

// Barrier polling uses relaxed loads (an acquire load may invalidate the SM's L1 on every poll);
// the caller issues one acquire fence once the count is reached.
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}


union JobArgsSmem {
  GemvArgs g;
  AttnArgs at;
  EmbedArgs ea;
  NormArgs na;
};

struct StepCtx {
  const StepArgs* a;
  PipeSmem sm;
  float* aux;
  float* tsum;
  JobArgsSmem* js;
  int G, g, warp, lane, ctid;
  uint32_t cphase;  // consumer-group barrier phase
  int s;            // ring slot of the next unit
  uint32_t ph;      // its full-barrier parity
};

__device__ __forceinline__ bool aborted(const StepArgs& a) {
  return *reinterpret_cast<volatile unsigned long long*>(a.sync + 1) != 0ull;
}

__device__ __forceinline__ void raise_abort(const StepArgs& a, unsigned bits) {
  atomicOr(a.err, (int)bits);
  atomicExch(a.sync + 1, 1ull);
}

// Grid barrier: all G CTAs have finished jobs [0, j) once the arrival count reaches G * j.
// Thread ctid 0 polls; the caller distributes the outcome with a consumer-group barrier.
__device__ bool wait_jobs_done(const StepArgs& a, int G, int j) {
  const unsigned long long target = (unsigned long long)G * (unsigned long long)j;
  if (ld_relaxed_u64(a.sync) >= target) {
    fence_acquire_gpu();
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (ld_relaxed_u64(a.sync) >= target) {
        fence_acquire_gpu();
        return true;
      }
    if (aborted(a)) return false;
    if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) {
      raise_abort(a, SHD_DEVERR_TIMEOUT_FULL);
      return false;
    }
  }
}

// CTAs taking part in a GEMV job of U units: the first min(G, U) CTAs, so that every participant
// owns at least one unit and the contributors to a split tile are consecutive CTAs (the split-tile
// fixup counts them as such).
__device__ __forceinline__ int job_ctas(long long U, int G) { return (int)(U < G ? U : G); }

// ------------------------------------------------------------------------------------------------
// Producer
// ------------------------------------------------------------------------------------------------
// Where a job's staged activations come from (kept in registers by the producer).
struct XSrc {
  const float* xc;
  const float* xs;
  int ldx, nKC, K;
};

struct PendingX {
  int s;
  int job;
  int c;  // K chunk of the unit
  XSrc x;
};

template <int M>
__device__ void step_producer(const StepArgs& a, const PipeSmem& sm, int G, int g) {
  const uint64_t pol_w = l2_policy_evict_first();
  const uint64_t pol_x = l2_policy_evict_last();
  const int S = sm.S;
  PendingX pend[kStepMaxStages];
  int p_head = 0, p_n = 0;
  int ready = 0;  // jobs [0, ready) are complete everywhere: job j may read its inputs once j <= ready
  long long issued = 0;
  int s = 0;
  bool ok = true;

  auto inputs_ready = [&](int j) -> bool {
    if (j <= ready) return true;
    const unsigned long long v = ld_relaxed_u64(a.sync);
    const int done = (int)(v / (unsigned long long)G);  // jobs completed by every CTA
    if (done > ready) {
      fence_acquire_gpu();
      ready = done;
    }
    return j <= ready;
  };
  int fenced_job[2] = {0, -1};  // proxy fence issued after the inputs of job [1] became visible
  auto issue_x = [&](int st, const XSrc& x, int c) {
    const uint32_t xb = (uint32_t)min(kChunkBf16, x.K - c * kChunkBf16) * 4u;
    uint8_t* dst = sm.stages + (size_t)st * sm.stage_bytes + kBlockBytes;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      bulk_g2s(dst + (m * 2 + 0) * (kChunkBf16 * 4), x.xc + (size_t)m * x.ldx + (size_t)c * kChunkBf16, xb,
               &sm.full[st], pol_x);
      bulk_g2s(dst + (m * 2 + 1) * (kChunkBf16 * 4), x.xs + (size_t)m * x.ldx + (size_t)c * kChunkBf16, xb,
               &sm.full[st], pol_x);
    }
  };
  // issue the activation copies of pending stages whose job inputs are complete (in order)
  auto flush = [&](bool force) {
    bool fenced = false;
    while (p_n > 0) {
      const PendingX& p = pend[p_head];
      if (!force && !inputs_ready(p.job)) break;
      if (!fenced) {
        fence_proxy_async_global();
        fenced = true;
        fenced_job[0] = 1;
        fenced_job[1] = p.job;
      }
      issue_x(p.s, p.x, p.c);
      p_head = (p_head + 1 == S) ? 0 : p_head + 1;
      --p_n;
    }
  };

  for (int j = 0; j < a.n_jobs && ok; ++j) {
    const StepJob* J = a.jobs + j;
    if (J->type != JOB_GEMV) continue;
    const GemvArgs* ga = &J->g;
    // the job's fields in registers (the unit loop below issues no other global loads)
    const int nKC = ga->nKC, Kx = ga->K;
    const long long U = (long long)ga->nT * nKC;
    const int Gj = job_ctas(U, G);
    if (g >= Gj) continue;
    const long long u0 = unit_begin(U, Gj, g), u1 = unit_begin(U, Gj, g + 1);
    const bool staged = J->norm == 0;
    const uint8_t* W = ga->W;
    const XSrc xs{ga->Xc, ga->Xs, ga->ldx, nKC, Kx};
    int c = (int)(u0 % nKC);
    for (long long u = u0; u < u1; ++u) {
      if (issued >= S) {
        const uint32_t par = (uint32_t)(((issued / S) - 1) & 1);
        if (!mbar_try_wait(&sm.empty[s], par)) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&sm.empty[s], par)) {
            if (p_n > 0) flush(false);
            if (aborted(a)) {
              ok = false;
              break;
            }
            if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) {
              raise_abort(a, SHD_DEVERR_TIMEOUT_EMPTY);
              ok = false;
              break;
            }
          }
          if (!ok) break;
        }
      }
      uint32_t tx = (uint32_t)kBlockBytes;
      if (staged) tx += (uint32_t)(M * 2) * (uint32_t)min(kChunkBf16, Kx - c * kChunkBf16) * 4u;
      mbar_arrive_expect_tx(&sm.full[s], tx);
      bulk_g2s(sm.stages + (size_t)s * sm.stage_bytes, W + (size_t)u * kBlockBytes, kBlockBytes, &sm.full[s], pol_w);
      if (staged) {
        if (p_n == 0 && inputs_ready(j)) {
          if (!fenced_job[0] || fenced_job[1] != j) {
            fence_proxy_async_global();
            fenced_job[0] = 1;
            fenced_job[1] = j;
          }
          issue_x(s, xs, c);
        } else {
          pend[(p_head + p_n) % S] = PendingX{s, j, c, xs};
          ++p_n;
        }
      }
      ++issued;
      s = (s + 1 == S) ? 0 : s + 1;
      if (++c == nKC) c = 0;
      if (p_n > 0) flush(false);
    }
  }
  if (ok) {
    // the last pending activations: their jobs' inputs complete before the consumers get there
    const uint64_t t0 = globaltimer_ns();
    while (p_n > 0) {
      flush(false);
      if (p_n == 0) break;
      if (aborted(a)) {
        ok = false;
        break;
      }
      if (globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) {
        raise_abort(a, SHD_DEVERR_TIMEOUT_EMPTY);
        ok = false;
        break;
      }
    }
  }
  if (!ok) {
    // Leaving early: complete every stage still expecting bytes (pending activation copies read
    // valid, if stale, memory), then wait for the copies in flight so none lands after exit.
    flush(true);
    for (long long k = std::max<long long>(0, issued - S); k < issued; ++k) {
      const int ks = (int)(k % S);
      if (!mbar_wait_bounded(&sm.full[ks], (uint32_t)((k / S) & 1))) atomicOr(a.err, SHD_DEVERR_TIMEOUT_DRAIN);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Consumer jobs
// ------------------------------------------------------------------------------------------------
template <int M>
__device__ bool gemv_job(StepCtx& C, int epi, bool norm) {
  constexpr int V = 4 * 2 * M;
  constexpr int VP = (V <= 8) ? 8 : (V <= 16) ? 16 : (V <= 32) ? 32 : 64;
  constexpr int TSUM = kTileRows * 2 * M;
  const GemvArgs& ga = C.js->g;
  const int G = C.G, g = C.g, lane = C.lane, warp = C.warp, ctid = C.ctid;
  const int nKC = ga.nKC;
  const int KP = nKC * kChunkBf16;
  const long long U = (long long)ga.nT * nKC;
  const int Gj = job_ctas(U, G);
  const long long u0 = g < Gj ? unit_begin(U, Gj, g) : 0, u1 = g < Gj ? unit_begin(U, Gj, g + 1) : 0;
  // CTA 0 also writes the residual stream h = D + H, so it runs the prologue even without units
  if (norm && (u0 < u1 || g == 0)) {
    if (!norm_prologue<M>(ga, C.sm, C.cphase, C.aux, KP, ctid, lane, warp, g == 0)) return false;
  }
  if (u0 >= u1) return true;
  unsigned long long acc2[(M <= 4) ? V : 1];
  float acc[VP];
#pragma unroll
  for (int j = 0; j < VP; ++j) acc[j] = 0.f;
  if constexpr (M <= 4) {
#pragma unroll
    for (int j = 0; j < V; ++j) acc2[j] = 0ull;
  }
  const int first_tile = (int)(u0 / nKC);
  int t = first_tile, c = (int)(u0 % nKC);
  for (long long u = u0; u < u1; ++u) {
    if (!warp_wait(&C.sm.full[C.s], C.ph)) {
      if (lane == 0) raise_abort(*C.a, SHD_DEVERR_TIMEOUT_FULL);
      return false;
    }
    const uint8_t* st = C.sm.stages + (size_t)C.s * C.sm.stage_bytes;
    const uint4* wv = reinterpret_cast<const uint4*>(st);
    const float* xbase;
    int xstride;
    bool okA = true, okB = true;
    if (norm) {
      xbase = C.aux + (size_t)c * kChunkBf16;
      xstride = KP;
    } else {
      xbase = reinterpret_cast<const float*>(st + kBlockBytes);
      xstride = kChunkBf16;
      okA = c * kChunkBf16 + 4 * lane < ga.K;
      okB = c * kChunkBf16 + 128 + 4 * lane < ga.K;
    }
    mac_block<M, V, VP>(wv, xbase, xstride, okA, okB, warp, lane, acc2, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&C.sm.empty[C.s]);
    if (++C.s == C.sm.S) {
      C.s = 0;
      C.ph ^= 1u;
    }
    const int ct = t, cc = c;
    if (++c == nKC) {
      c = 0;
      ++t;
    }
    const bool tile_end = (cc == nKC - 1) || (u == u1 - 1);
    if (!tile_end) continue;
    tile_reduce<M, V, VP>(acc2, acc, C.tsum, warp, lane);
    const bool full_tile = ((long long)ct * nKC >= u0) && (cc == nKC - 1);
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;
    if (!full_tile) {
      const int r = split_tile_close<float>(C.sm, C.cphase, C.tsum, ga.partials, ga.counters, TSUM, U, Gj, g, ct,
                                            nKC, u0, u1, ctid, lane,
                                            reinterpret_cast<const volatile unsigned long long*>(C.a->sync + 1));
      if (r < 0) {
        if (lane == 0) raise_abort(*C.a, SHD_DEVERR_TIMEOUT_FULL);
        return false;
      }
      if (r == 0) continue;
    }
    switch (epi) {
      case EPI_STORE: epilogue_f32<M, EPI_STORE>(ga, ct, C.tsum, ctid, ga.err); break;
      case EPI_QKV: epilogue_f32<M, EPI_QKV>(ga, ct, C.tsum, ctid, ga.err); break;
      case EPI_GATEUP: epilogue_f32<M, EPI_GATEUP>(ga, ct, C.tsum, ctid, ga.err); break;
      default: epilogue_f32<M, EPI_LOGITS>(ga, ct, C.tsum, ctid, ga.err); break;
    }
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;
  }
  return true;
}

// One attention item: query row m, head group gi (<= 4 query heads of one kv head), position split
// r of nsplit. Same tile algorithm as the cluster kernel (K/V tile staged in shared memory, warps
// over head_dim slices for the scores, online softmax, weighted V in registers); the split's
// (max, sum, weighted V) goes to global partials and the last arriving split combines all splits
// in split order.
template <int HD>
__device__ bool attn_item(StepCtx& C, int item) {
  const AttnArgs& a = C.js->at;
  AttnTile<HD>& S = *reinterpret_cast<AttnTile<HD>*>(C.aux);
  const int lane = C.lane, warp = C.warp, tid = C.ctid;
  constexpr int DW = HD / kANW;
  constexpr int GPT = kAGroup * HD / kAThreads;  // heads per thread in the PV phase
  const int per_row = a.n_groups * a.nsplit;
  const int m = item / per_row, gi = (item % per_row) / a.nsplit, r = item % a.nsplit;
  const int4 grp = a.groups[gi];
  const int kvh = grp.x, qh0 = grp.y, Gh = grp.z;
  const int kv_len = __ldcg(a.pos + m) + 1;
  const int sq = a.seq ? __ldcg(a.seq + m) : 0;
  const int per = (kv_len + a.nsplit - 1) / a.nsplit;
  const int t0 = min(r * per, kv_len), t1 = min(t0 + per, kv_len);
  const float* K = a.Kcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const float* Vp = a.Vcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const bool mpc = a.variant == SHD_NL_MPC;

  for (int i = tid; i < kAGroup * HD; i += kAThreads) {
    const int gq = i / HD, d = i % HD;
    S.q[gq][d] = (gq < Gh) ? __ldcg(a.Q + (size_t)m * a.ldq + (size_t)(qh0 + gq) * HD + d) : 0.0f;
  }
  if (tid < kAGroup) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.0f;
  }
  float acc[GPT];
#pragma unroll
  for (int j = 0; j < GPT; ++j) acc[j] = 0.0f;
  const int pd = tid % HD, pg0 = tid / HD;
  if (!consumer_sync(C.sm, C.cphase, lane)) return false;
  for (int tb = t0; tb < t1; tb += kATile) {
    const int nt = min(kATile, t1 - tb);
    for (int i = tid; i < kATile * (HD / 4); i += kAThreads) {
      const int rr = i / (HD / 4), c4 = i % (HD / 4);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (rr < nt) {
        kv = __ldcg(reinterpret_cast<const float4*>(K + (size_t)(tb + rr) * a.kvd + 4 * c4));
        vv = __ldcg(reinterpret_cast<const float4*>(Vp + (size_t)(tb + rr) * a.kvd + 4 * c4));
      }
      *reinterpret_cast<float4*>(&S.k[rr][4 * c4]) = kv;
      *reinterpret_cast<float4*>(&S.v[rr][4 * c4]) = vv;
    }
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;
    {
      float part[kAGroup];
#pragma unroll
      for (int gq = 0; gq < kAGroup; ++gq) part[gq] = 0.0f;
#pragma unroll
      for (int j = 0; j < DW; j += 4) {
        const float4 kk = *reinterpret_cast<const float4*>(&S.k[lane & (kATile - 1)][warp * DW + j]);
#pragma unroll
        for (int gq = 0; gq < kAGroup; ++gq) {
          const float4 qq = *reinterpret_cast<const float4*>(&S.q[gq][warp * DW + j]);
          part[gq] = __fmaf_rn(qq.x, kk.x, part[gq]);
          part[gq] = __fmaf_rn(qq.y, kk.y, part[gq]);
          part[gq] = __fmaf_rn(qq.z, kk.z, part[gq]);
          part[gq] = __fmaf_rn(qq.w, kk.w, part[gq]);
        }
      }
#pragma unroll
      for (int gq = 0; gq < kAGroup; ++gq) S.spart[warp][gq][lane] = part[gq];
    }
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;
    if (warp < Gh) {
      const int gq = warp;
      float sc = 0.0f;
#pragma unroll
      for (int w = 0; w < kANW; ++w) sc = __fadd_rn(sc, S.spart[w][gq][lane]);
      sc = (lane < nt) ? __fmul_rn(sc, a.scale) : -INFINITY;
      float tmax = sc;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mold = S.m[gq];
      const float mnew = fmaxf(mold, tmax);
      float x = __fsub_rn(sc, mnew);
      if (!mpc) x = fminf(fmaxf(x, -40.0f), 40.0f);
      const float pe = (lane < nt) ? expf(x) : 0.0f;
      float tsum = pe;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) tsum = __fadd_rn(tsum, __shfl_xor_sync(0xffffffffu, tsum, o));
      S.p[gq][lane] = pe;
      __syncwarp();
      if (lane == 0) {
        const float al = (mold == -INFINITY) ? 0.0f : expf(__fsub_rn(mold, mnew));
        S.alpha[gq] = al;
        S.l[gq] = __fmaf_rn(S.l[gq], al, tsum);
        S.m[gq] = mnew;
      }
    }
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;
#pragma unroll
    for (int j = 0; j < GPT; ++j) {
      const int gq = pg0 + j * (kAThreads / HD);
      if (gq < Gh) {
        float v = __fmul_rn(acc[j], S.alpha[gq]);
        for (int rr = 0; rr < nt; ++rr) v = __fmaf_rn(S.p[gq][rr], S.v[rr][pd], v);
        acc[j] = v;
      }
    }
    if (!consumer_sync(C.sm, C.cphase, lane)) return false;  // tile buffers are reused
  }

  // this split's partial: [group head][m, l, weighted V...]
  constexpr int PW = HD + 2;
  float* part = a.partials + ((size_t)(m * a.n_groups + gi) * a.nsplit + r) * (kAGroup * PW);
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int gq = pg0 + j * (kAThreads / HD);
    if (gq < Gh) part[gq * PW + 2 + pd] = acc[j];
  }
  if (tid < Gh) {
    part[tid * PW + 0] = S.m[tid];
    part[tid * PW + 1] = S.l[tid];
  }
  if (!consumer_sync(C.sm, C.cphase, lane)) return false;
  // Split 0's CTA owns the combine: the other splits publish with a release increment and leave;
  // the owner waits (bounded) for all of them. Items of one group are consecutive and every CTA runs
  // its items in increasing order, so an owner only ever waits for later items of other CTAs.
  int* cnt = a.counters + (m * a.n_groups + gi);
  if (r != 0) {
    if (tid == 0) {
      __threadfence();
      red_release_add(cnt, 1);
    }
    return true;
  }
  if (tid == 0) {
    bool ok = true;
    if (ld_relaxed_s32(cnt) < a.nsplit - 1) {
      const uint64_t w0 = globaltimer_ns();
      while (ld_relaxed_s32(cnt) < a.nsplit - 1) {
        if (aborted(*C.a)) {
          ok = false;
          break;
        }
        if (globaltimer_ns() - w0 > SHD_WAIT_LIMIT_NS) {
          raise_abort(*C.a, SHD_DEVERR_TIMEOUT_FULL);
          ok = false;
          break;
        }
      }
    }
    if (ok) {
      __threadfence();
      *cnt = 0;
    }
    S.last = ok ? 1 : 0;
  }
  if (!consumer_sync(C.sm, C.cphase, lane)) return false;
  if (!S.last) return false;

  // Combine in split order. The splits' (max, sum) pairs are gathered into shared memory by all
  // threads at once (the tile buffers are free now), the split weights exp(m_r - max) computed once
  // per (head, split), then every (head, dim) thread sums its weighted V partials with independent
  // loads in flight.
  const float* base = a.partials + (size_t)(m * a.n_groups + gi) * a.nsplit * (kAGroup * PW);
  const int ns = a.nsplit;
  float* wsm = &S.k[0][0];          // [kAGroup][ns] split weights
  float* lsm = wsm + kAGroup * ns;  // [kAGroup][ns] split sums
  float* msm = lsm + kAGroup * ns;  // [kAGroup][ns] split maxima
  for (int i = tid; i < Gh * ns; i += kAThreads) {
    const int gq = i / ns, rr = i % ns;
    const float* pr = base + (size_t)rr * (kAGroup * PW) + gq * PW;
    msm[gq * ns + rr] = __ldcg(pr);
    lsm[gq * ns + rr] = __ldcg(pr + 1);
  }
  if (!consumer_sync(C.sm, C.cphase, lane)) return false;
  if (tid < Gh) {
    float Mx = -INFINITY;
    for (int rr = 0; rr < ns; ++rr) Mx = fmaxf(Mx, msm[tid * ns + rr]);
    float L = 0.0f;
    for (int rr = 0; rr < ns; ++rr) {
      const float mr = msm[tid * ns + rr];
      const float w = (mr == -INFINITY) ? 0.0f : expf(__fsub_rn(mr, Mx));
      wsm[tid * ns + rr] = w;
      if (mr != -INFINITY) L = __fmaf_rn(lsm[tid * ns + rr], w, L);
    }
    S.l[tid] = L;
  }
  if (!consumer_sync(C.sm, C.cphase, lane)) return false;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int gq = pg0 + j * (kAThreads / HD);
    if (gq >= Gh) continue;
    const float L = S.l[gq];
    float out = 0.0f;
    int rr = 0;
    for (; rr + 4 <= ns; rr += 4) {
      float v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = __ldcg(base + (size_t)(rr + q) * (kAGroup * PW) + gq * PW + 2 + pd);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (msm[gq * ns + rr + q] != -INFINITY) out = __fmaf_rn(v[q], wsm[gq * ns + rr + q], out);
    }
    for (; rr < ns; ++rr)
      if (msm[gq * ns + rr] != -INFINITY)
        out = __fmaf_rn(__ldcg(base + (size_t)rr * (kAGroup * PW) + gq * PW + 2 + pd), wsm[gq * ns + rr], out);
    if (mpc && !(L > 1e-10f && isfinite(L))) {
      // compute_mpc_attention_on_shares: weights 1/seq_len when the sum is not usable
      float uo = 0.0f;
      for (int tt = 0; tt < kv_len; ++tt)
        uo = __fmaf_rn(__fdiv_rn(1.0f, (float)kv_len), __ldcg(Vp + (size_t)tt * a.kvd + pd), uo);
      out = uo;
    } else {
      out = __fdiv_rn(out, L);
    }
    const int hh = qh0 + gq;
    const size_t o = (size_t)m * a.ldo + (size_t)hh * HD + pd;
    const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + (size_t)hh * HD + pd] : 0.0f;
    a.Oc[o] = __fsub_rn(out, mk);
    a.Os[o] = mk;
  }
  return true;
}

template <int M>
__device__ bool attn_job(StepCtx& C) {
  const AttnArgs& a = C.js->at;
  const int items = M * a.n_groups * a.nsplit;
  for (int it = C.g; it < items; it += C.G) {
    const bool ok = (a.head_dim == 128) ? attn_item<128>(C, it) : attn_item<64>(C, it);
    if (!ok) return false;
    if (!consumer_sync(C.sm, C.cphase, C.lane)) return false;  // the tile scratch is reused
  }
  return true;
}

template <int M>
__device__ void embed_job(StepCtx& C) {
  const EmbedArgs& a = C.js->ea;
  const int total = M * a.hidden;
  for (int idx = C.g * kAThreads + C.ctid; idx < total; idx += C.G * kAThreads) {
    const int m = idx / a.hidden, k = idx % a.hidden;
    const int tok = __ldcg(a.tokens + m);
    if (tok < 0 || tok >= a.vocab) {
      if (k == 0) atomicOr(a.err, SHD_DEVERR_ARG);
      continue;
    }
    const uint64_t counter = (a.slot_counter ? ((uint64_t)m << 32) : a.counter_base) +
                             (uint64_t)(a.pos ? __ldcg(a.pos + m) : m);
    const float e = __uint_as_float((uint32_t)a.table[(size_t)tok * a.hidden + k] << 16);
    const float s = u32_to_unit_f32(philox_word(a.seed, 7, counter * (uint64_t)a.hidden + (uint64_t)k));
    a.Hc[(size_t)m * a.ldh + k] = __fsub_rn(e, s);
    a.Hs[(size_t)m * a.ldh + k] = s;
    if (a.Dc) {
      a.Dc[(size_t)m * a.ldh + k] = 0.0f;
      a.Ds[(size_t)m * a.ldh + k] = 0.0f;
    }
  }
  if (a.amax && C.g == 0 && C.ctid < M) a.amax[C.ctid] = 0ull;
}

// Standalone RMSNorm + reshare of row m into global X (used when the fused prologue does not fit).
template <int M>
__device__ bool norm_job(StepCtx& C) {
  const NormArgs& a = C.js->na;
  for (int m = C.g; m < M; m += C.G) {
    const float* hc = a.Hc + (size_t)m * a.ldh;
    const float* hs = a.Hs + (size_t)m * a.ldh;
    const float* dc = a.Dc ? a.Dc + (size_t)m * a.ldh : nullptr;
    const float* ds = a.Ds ? a.Ds + (size_t)m * a.ldh : nullptr;
    float* oc = a.Hout_c ? a.Hout_c + (size_t)m * a.ldh : nullptr;
    float* os = a.Hout_s ? a.Hout_s + (size_t)m * a.ldh : nullptr;
    float sq = 0.0f;
    for (int i = C.ctid; i < a.n; i += kAThreads) {
      float c = __ldcg(hc + i), s = __ldcg(hs + i);
      if (dc) {
        c = __fadd_rn(__ldcg(dc + i), c);
        s = __fadd_rn(__ldcg(ds + i), s);
        if (oc) {
          oc[i] = c;
          os[i] = s;
        }
      }
      const float x = __fadd_rn(c, s);
      sq = __fmaf_rn(x, x, sq);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
    if (C.lane == 0) C.sm.red[C.warp] = sq;
    if (!consumer_sync(C.sm, C.cphase, C.lane)) return false;
    float sum_sq = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) sum_sq = __fadd_rn(sum_sq, C.sm.red[w]);
    const float mean_sq = __fdiv_rn(sum_sq, (float)a.n);
    float inv;
    if (a.variant == SHD_NL_GPU) {
      inv = rsqrtf(__fadd_rn(mean_sq, a.eps));
    } else {
      const float rms = __fsqrt_rn(__fadd_rn(mean_sq, a.eps));
      if (a.variant == SHD_NL_MPC)
        inv = (rms > 1e-6f && isfinite(rms)) ? __fdiv_rn(1.0f, rms) : 1.0f;
      else
        inv = __fdiv_rn(1.0f, rms);
    }
    float* xc = a.Xc + (size_t)m * a.ldx;
    float* xs = a.Xs + (size_t)m * a.ldx;
    const float* mk = a.mask ? a.mask + (size_t)m * a.ldmask : nullptr;
    for (int i = C.ctid; i < a.n; i += kAThreads) {
      float c = __ldcg(hc + i), s = __ldcg(hs + i);
      if (dc) {
        c = __fadd_rn(__ldcg(dc + i), c);
        s = __fadd_rn(__ldcg(ds + i), s);
      }
      const float x = __fadd_rn(c, s);
      float r = __fmul_rn(__fmul_rn(x, inv), a.gamma[i]);
      if (a.variant == SHD_NL_MPC && !isfinite(r)) r = 0.0f;
      const float mv = mk ? mk[i] : 0.0f;
      xc[i] = __fsub_rn(r, mv);
      xs[i] = mv;
    }
    if (!consumer_sync(C.sm, C.cphase, C.lane)) return false;  // red reuse
  }
  return true;
}

template <int M>
__device__ void step_consumers(StepCtx& C) {
  const StepArgs& a = *C.a;
  const int ctid = C.ctid;
  constexpr int kArgWords = (int)(sizeof(JobArgsSmem) / 4);
  for (int j = 0; j < a.n_jobs; ++j) {
    const StepJob* J = a.jobs + j;
    const int type = J->type;
    // copy this job's arguments to shared memory while thread 0 waits for the previous jobs
    {
      const uint32_t* src;
      int words;
      switch (type) {
        case JOB_GEMV: src = reinterpret_cast<const uint32_t*>(&J->g); words = (int)(sizeof(GemvArgs) / 4); break;
        case JOB_ATTN: src = reinterpret_cast<const uint32_t*>(&J->at); words = (int)(sizeof(AttnArgs) / 4); break;
        case JOB_EMBED: src = reinterpret_cast<const uint32_t*>(&J->ea); words = (int)(sizeof(EmbedArgs) / 4); break;
        default: src = reinterpret_cast<const uint32_t*>(&J->na); words = (int)(sizeof(NormArgs) / 4); break;
      }
      uint32_t* dst = reinterpret_cast<uint32_t*>(C.js);
      for (int i = ctid; i < words && i < kArgWords; i += kAThreads) dst[i] = src[i];
    }
    if (ctid == 0) {
      const bool ok = (j == 0) || wait_jobs_done(a, C.G, j);
      C.sm.flags[0] = ok ? 0 : 1;
      if (ok && a.prof_t) atomicMin(a.prof_t + j, (unsigned long long)globaltimer_ns());
    }
    if (!consumer_sync(C.sm, C.cphase, C.lane) || C.sm.flags[0]) return;
    bool ok = true;
    switch (type) {
      case JOB_GEMV: ok = gemv_job<M>(C, J->epi, J->norm != 0); break;
      case JOB_ATTN: ok = attn_job<M>(C); break;
      case JOB_EMBED: embed_job<M>(C); break;
      default: ok = norm_job<M>(C); break;
    }
    if (!ok) return;
    if (!consumer_sync(C.sm, C.cphase, C.lane)) return;
    if (ctid == 0) {
      if (a.prof_t) atomicMax(a.prof_t + a.n_jobs + j, (unsigned long long)globaltimer_ns());
      __threadfence();
      atomicAdd(a.sync, 1ull);
    }
  }
  if (C.g != 0) return;
  // the greedy token update once every CTA has finished the head
  if (ctid == 0) {
    const bool ok = wait_jobs_done(a, C.G, a.n_jobs);
    C.sm.flags[0] = ok ? 0 : 1;
  }
  if (!consumer_sync(C.sm, C.cphase, C.lane) || C.sm.flags[0]) return;
  const unsigned long long s = *reinterpret_cast<volatile unsigned long long*>(a.step);
  if (ctid < a.M) {
    const int tok = (int)(__ldcg(a.amax + ctid) & 0xffffffffu);
    a.tokens[ctid] = tok;
    a.hist[(size_t)(s % (unsigned long long)a.hist_cap) * a.M + ctid] = tok;
    a.pos[ctid] = __ldcg(a.pos + ctid) + 1;
  }
  if (a.prof_acc) {
    for (int j = ctid; j < a.n_jobs; j += kAThreads) {
      const unsigned long long t0 = a.prof_t[j], t1 = a.prof_t[a.n_jobs + j];
      if (t1 > t0) a.prof_acc[j] += t1 - t0;
      a.prof_t[j] = ~0ull;
      a.prof_t[a.n_jobs + j] = 0ull;
    }
    if (ctid == 0) a.prof_acc[a.n_jobs] += 1ull;
  }
  if (!consumer_sync(C.sm, C.cphase, C.lane)) return;
  if (ctid == 0) *a.step = s + 1;
}

template <int M>
__global__ void __launch_bounds__(kGemvThreads, (M == 1) ? 2 : 1) step_kernel(const __grid_constant__ StepArgs a) {
  constexpr int TSUM = kTileRows * 2 * M;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ JobArgsSmem js;
  StepCtx C;
  C.a = &a;
  C.sm.stages = smem;
  C.sm.S = a.nstages;
  C.sm.stage_bytes = a.stage_bytes;
  C.aux = reinterpret_cast<float*>(smem + (size_t)a.nstages * a.stage_bytes);
  C.tsum = C.aux + a.aux_floats;
  C.sm.full = reinterpret_cast<uint64_t*>(C.tsum + TSUM);
  C.sm.empty = C.sm.full + a.nstages;
  C.sm.cbar = C.sm.empty + a.nstages;
  C.sm.flags = reinterpret_cast<volatile int*>(C.sm.cbar + 2);
  C.sm.red = reinterpret_cast<float*>(C.sm.cbar + 4);
  C.js = &js;
  C.G = gridDim.x;
  C.g = blockIdx.x;
  C.warp = threadIdx.x >> 5;
  C.lane = threadIdx.x & 31;
  C.ctid = threadIdx.x;
  C.cphase = 0;
  C.s = 0;
  C.ph = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&C.sm.full[s], 1);
      mbar_init(&C.sm.empty[s], kConsumerWarps);
    }
    mbar_init(C.sm.cbar, kConsumerWarps);
    C.sm.flags[0] = 0;
    C.sm.flags[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (C.warp == kConsumerWarps) {
    if (C.lane == 0) step_producer<M>(a, C.sm, C.G, C.g);
    return;
  }
  step_consumers<M>(C);
}

template <int M>
int launch_step_t(shd_ctx* ctx, const StepPlan& p, const StepArgs& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SHD_CHECK_CUDA(ctx, cudaLaunchKernelEx(&cfg, step_kernel<M>, a));
  ctx->launches++;
  return SHD_OK;
}

// Allow the plan's dynamic shared memory and report how many CTAs fit on one SM.
template <int M>
cudaError_t step_occupancy(size_t smem, int* per_sm) {
  cudaError_t e = cudaFuncSetAttribute(step_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmemLimit);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, step_kernel<M>, kGemvThreads, smem);
}

}  // namespace

int step_plan_build(shd_ctx* ctx, StepPlan& plan, std::vector<StepJob>& jobs, int M) {
  step_plan_free(plan);
  SHD_REQUIRE(ctx, M >= 1 && M <= 8, "step: rows must be 1..8");
  SHD_REQUIRE(ctx, !jobs.empty(), "step: empty job list");
  // geometry: stage = weight block + staged activations; aux = fused-norm activations or the
  // attention tile, whichever is larger
  size_t aux = 64;
  int n_groups = 0, head_dim = 0;
  for (auto& j : jobs) {
    if (j.type == JOB_GEMV && j.norm) aux = std::max(aux, (size_t)M * 2 * j.g.nKC * kChunkBf16);
    if (j.type == JOB_ATTN) {
      SHD_REQUIRE(ctx, j.at.head_dim == 64 || j.at.head_dim == 128, "step: head_dim must be 64 or 128");
      n_groups = std::max(n_groups, j.at.n_groups);
      head_dim = j.at.head_dim;
      const size_t tile = (j.at.head_dim == 128 ? sizeof(AttnTile<128>) : sizeof(AttnTile<64>)) / 4;
      aux = std::max(aux, tile);
    }
  }
  aux = (aux + 3) / 4 * 4;
  const int stage = kBlockBytes + M * 2 * kChunkBf16 * 4;
  // Two CTAs per SM stream faster than one with the same bytes in flight (two producers, twice the
  // consumer warps); single rows (M = 1) use them when at least 3 stages fit, else one CTA per SM.
  int per_sm_want = 1;
  int S = 0;
  if (M == 1) {
    const long long room2 = (long long)kStepSmemPerCta2 - (long long)aux * 4 - kStepTail;
    const int S2 = (int)std::min<long long>(kStepMaxStages, room2 / stage);
    if (S2 >= 3) {
      per_sm_want = 2;
      S = S2;
    }
  }
  if (per_sm_want == 1) {
    const long long room = (long long)kStepSmemLimit - (long long)aux * 4 - kStepTail;
    S = (int)std::min<long long>(kStepMaxStages, room / stage);
  }
  if (S < 2) return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "step: activations too wide for one CTA per SM");
  const int G = per_sm_want * ctx->num_sms;
  plan.grid = G;
  plan.nstages = S;
  plan.stage_bytes = stage;
  plan.aux_floats = (int)aux;
  plan.smem = (size_t)S * stage + aux * 4 + kStepTail;
  plan.M = M;
  plan.n_jobs = (int)jobs.size();
  // attention: about one (row, group, split) item per CTA
  // (at most 64 splits: the combine keeps 3 floats per head and split in the K tile buffer)
  const int nsplit = n_groups > 0 ? std::min(64, std::max(1, G / (M * n_groups))) : 1;
  const size_t part_floats = (size_t)M * std::max(n_groups, 1) * nsplit * kAGroup * (std::max(head_dim, 64) + 2);
  auto fail = [&](cudaError_t e, const char* what) {
    step_plan_free(plan);
    return shd_cuda_fail(ctx, e, what);
  };
  cudaError_t e = cudaMalloc(&plan.d_attn_part, part_floats * 4);
  if (e != cudaSuccess) return fail(e, "step: attention partials");
  e = cudaMalloc(&plan.d_attn_cnt, (size_t)M * std::max(n_groups, 1) * 4);
  if (e != cudaSuccess) return fail(e, "step: attention counters");
  e = cudaMemset(plan.d_attn_cnt, 0, (size_t)M * std::max(n_groups, 1) * 4);
  if (e != cudaSuccess) return fail(e, "step: attention counters");
  for (auto& j : jobs) {
    if (j.type != JOB_ATTN) continue;
    j.at.nsplit = nsplit;
    j.at.partials = plan.d_attn_part;
    j.at.counters = plan.d_attn_cnt;
  }
  e = cudaMalloc(&plan.d_jobs, jobs.size() * sizeof(StepJob));
  if (e != cudaSuccess) return fail(e, "step: job table");
  e = cudaMemcpy(plan.d_jobs, jobs.data(), jobs.size() * sizeof(StepJob), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(e, "step: job table upload");
  e = cudaMalloc(&plan.d_sync, 2 * sizeof(unsigned long long));
  if (e != cudaSuccess) return fail(e, "step: barrier");
  const size_t nprof = 2 * jobs.size() + jobs.size() + 1;
  e = cudaMalloc(&plan.d_prof, nprof * sizeof(unsigned long long));
  if (e != cudaSuccess) return fail(e, "step: profile");
  std::vector<unsigned long long> init(nprof, 0ull);
  for (size_t i = 0; i < jobs.size(); ++i) init[i] = ~0ull;
  e = cudaMemcpy(plan.d_prof, init.data(), nprof * sizeof(unsigned long long), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(e, "step: profile");
  plan.kinds.clear();
  plan.bytes.clear();
  for (auto& j : jobs) {
    plan.kinds.push_back(j.kind);
    plan.bytes.push_back(j.bytes);
  }
  // every CTA must be resident at once
  int per_sm = 0;
  cudaError_t oe;
  switch (M) {
    case 1: oe = step_occupancy<1>(plan.smem, &per_sm); break;
    case 2: oe = step_occupancy<2>(plan.smem, &per_sm); break;
    case 3: oe = step_occupancy<3>(plan.smem, &per_sm); break;
    case 4: oe = step_occupancy<4>(plan.smem, &per_sm); break;
    case 5: oe = step_occupancy<5>(plan.smem, &per_sm); break;
    case 6: oe = step_occupancy<6>(plan.smem, &per_sm); break;
    case 7: oe = step_occupancy<7>(plan.smem, &per_sm); break;
    default: oe = step_occupancy<8>(plan.smem, &per_sm); break;
  }
  if (oe != cudaSuccess) return fail(oe, "step: occupancy");
  if (per_sm < per_sm_want) {
    step_plan_free(plan);
    return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "step: the grid does not fit on the GPU at once");
  }
  return SHD_OK;
}

void step_plan_free(StepPlan& p) {
  for (void* q : {(void*)p.d_jobs, (void*)p.d_sync, (void*)p.d_attn_part, (void*)p.d_attn_cnt, (void*)p.d_prof})
    if (q) cudaFree(q);
  p = StepPlan{};
}

int step_launch(shd_ctx* ctx, const StepPlan& p, cudaStream_t stream, const unsigned long long* amax, int* tokens,
                int* pos, int* hist, int hist_cap, unsigned long long* step, bool profile) {
  SHD_REQUIRE(ctx, p.d_jobs != nullptr, "step: no plan");
  SHD_CHECK_CUDA(ctx, cudaMemsetAsync(p.d_sync, 0, 2 * sizeof(unsigned long long), stream));
  StepArgs a{};
  a.jobs = p.d_jobs;
  a.n_jobs = p.n_jobs;
  a.sync = p.d_sync;
  a.err = ctx->d_err;
  a.amax = amax;
  a.tokens = tokens;
  a.pos = pos;
  a.hist = hist;
  a.hist_cap = hist_cap;
  a.step = step;
  a.M = p.M;
  a.nstages = p.nstages;
  a.stage_bytes = p.stage_bytes;
  a.aux_floats = p.aux_floats;
  a.prof_t = profile ? p.d_prof : nullptr;
  a.prof_acc = profile ? p.d_prof + 2 * p.n_jobs : nullptr;
  switch (p.M) {
    case 1: return launch_step_t<1>(ctx, p, a, stream);
    case 2: return launch_step_t<2>(ctx, p, a, stream);
    case 3: return launch_step_t<3>(ctx, p, a, stream);
    case 4: return launch_step_t<4>(ctx, p, a, stream);
    case 5: return launch_step_t<5>(ctx, p, a, stream);
    case 6: return launch_step_t<6>(ctx, p, a, stream);
    case 7: return launch_step_t<7>(ctx, p, a, stream);
    default: return launch_step_t<8>(ctx, p, a, stream);
  }
}

int step_prof_reset(shd_ctx* ctx, const StepPlan& p, cudaStream_t stream) {
  if (!p.d_prof) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaMemsetAsync(p.d_prof, 0xff, (size_t)p.n_jobs * 8, stream));
  SHD_CHECK_CUDA(ctx, cudaMemsetAsync(p.d_prof + p.n_jobs, 0, ((size_t)p.n_jobs + p.n_jobs + 1) * 8, stream));
  return SHD_OK;
}

int step_prof_read(shd_ctx* ctx, const StepPlan& p, float* ms_out6, double* bytes_out6) {
  std::vector<unsigned long long> acc((size_t)p.n_jobs + 1);
  SHD_CHECK_CUDA(ctx, cudaMemcpy(acc.data(), p.d_prof + 2 * p.n_jobs, acc.size() * 8, cudaMemcpyDeviceToHost));
  const double n = (double)acc[p.n_jobs];
  for (int k = 0; k < 6; ++k) {
    ms_out6[k] = 0.f;
    bytes_out6[k] = 0.0;
  }
  if (n <= 0) return SHD_OK;
  for (int j = 0; j < p.n_jobs; ++j) {
    const int k = p.kinds[j];
    if (k < 0 || k > 5) continue;
    ms_out6[k] += (float)((double)acc[j] / n * 1e-6);
    bytes_out6[k] += p.bytes[j];
  }
  return SHD_OK;
}

}  // namespace shd
