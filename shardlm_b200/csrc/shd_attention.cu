// Decode attention over the device-resident reconstructed KV cache (secure_attention_approx,
// crates/v2/sharing/src/secure_nonlinear.rs:287-333, and compute_mpc_attention_on_shares,
// crates/v2/server/src/routes/secure_inference_mpc.rs:568-663), followed by the reshare.
//
// Cluster flash decode. A cluster of 8 CTAs (64 warps) serves one (query row, head group), a group
// being up to 4 query heads that share one kv head, so each K/V row is read once for the group
// (groups of 8 heads, for batched rows, run the tile kernel further down). Positions are dealt to the warps in chunks of 32 / group positions; a warp
// holds its chunk's K and V rows in registers (each lane 1/32 of a row, coalesced 16-byte loads),
// computes the chunk's 32 (position, head) scores with one reduce-scatter over the warp and keeps
// an online softmax (running max, sum, weighted V sum) per head. There is no block barrier until
// the warps combine: decode latency is the loads in flight before the wait on the q/k/v kernel,
// one chunk of arithmetic and the two combines (warps in order through shared memory, then the
// cluster's CTAs in rank order in CTA 0 through distributed shared memory), so the result does not
// depend on timing.
//
// Against the reference's two-pass softmax (max over all scores, clamp(s - max, -40, 40), exp, sum,
// divide, weighted sum) the online form differs only in rounding and in applying the -40 clamp
// relative to a running instead of the global maximum (weights below e^-40 of the largest, i.e.
// contributions under 4.3e-18 of the total).
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "shd_nonlinear.cuh"

namespace cg = cooperative_groups;

namespace shd {

constexpr int kAttnCluster = 8;   // CTAs per (row, group)
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnGroup = 4;     // query heads per group (kAttnGroupMax bounds the scratch)

template <int HD, int GS>
struct AttnSmem {
  float wpart[kAttnWarps][GS][HD + 2];    // per warp: running max, sum, weighted V sum
  float gather[kAttnCluster][GS][HD + 2];  // CTA 0: the combined partial of every CTA of the cluster
};

// One lane's slice of a K or V row: DPL = HD / 32 consecutive floats at column DPL * lane.
template <int DPL>
__device__ __forceinline__ void load_slice(const float* row, int lane, float (&r)[DPL]) {
  if constexpr (DPL == 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(row) + lane);
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
  } else {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(row) + lane);
    r[0] = v.x; r[1] = v.y;
  }
}

// v[32] per lane -> the sum over the warp of v[lane] (reduce-scatter butterfly, 31 shuffles).
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j < n / 2) {
        const float send = up ? v[j] : v[j + n / 2];
        const float keep = up ? v[j + n / 2] : v[j];
        v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    }
  }
  return v[0];
}

// Chunk of CH = 32 / GS positions held by one warp: lane l's slices of the K and V rows.
template <int CH, int DPL>
struct KvChunk {
  float k[CH][DPL];
  float v[CH][DPL];
};

// Global chunk c of a row (positions [c CH, c CH + CH)); positions past kv_len and `skip` read as 0.
template <int CH, int DPL>
__device__ __forceinline__ void load_chunk(KvChunk<CH, DPL>& ch, const float* K, const float* V, size_t ld, int c,
                                           int kv_len, int skip, int lane) {
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int p = c * CH + j;
    if (p < kv_len && p != skip) {
      load_slice<DPL>(K + (size_t)p * ld, lane, ch.k[j]);
      load_slice<DPL>(V + (size_t)p * ld, lane, ch.v[j]);
    } else {
#pragma unroll
      for (int d = 0; d < DPL; ++d) ch.k[j][d] = ch.v[j][d] = 0.0f;
    }
  }
}

// Online-softmax state of one warp for GS heads: running max and sum (the same in every lane) and
// the lane's slice of the weighted V sum.
template <int GS, int DPL>
struct WarpSoftmax {
  float m[GS], l[GS], acc[GS][DPL];
};

// Fold one chunk into the warp's state. Scores: the 32 (position, head) dot products of the chunk
// are summed over the warp by a reduce-scatter, so lane l holds pair l = (l / GS, l % GS); the
// chunk's maximum and sum per head are xor reductions over the lanes of that head.
template <int GS, int DPL>
__device__ __forceinline__ void fold_chunk(WarpSoftmax<GS, DPL>& st, const KvChunk<32 / GS, DPL>& ch,
                                           const float (&q)[GS][DPL], int c, int kv_len, float scale, bool mpc,
                                           int lane) {
  constexpr int CH = 32 / GS;
  float part[32];
#pragma unroll
  for (int j = 0; j < CH; ++j)
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) s = __fmaf_rn(q[g][d], ch.k[j][d], s);
      part[j * GS + g] = s;
    }
  const float dot = warp_reduce_scatter32(part, lane);
  const int my_g = lane % GS;
  const bool valid = c * CH + lane / GS < kv_len;
  const float s = valid ? __fmul_rn(dot, scale) : -INFINITY;
  float cm = s;
#pragma unroll
  for (int o = GS; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
  float alpha[GS], mine = 0.0f;
#pragma unroll
  for (int g = 0; g < GS; ++g) {
    const float mn = fmaxf(st.m[g], __shfl_sync(0xffffffffu, cm, g));
    alpha[g] = (st.m[g] == -INFINITY) ? 0.0f : expf(__fsub_rn(st.m[g], mn));
    st.m[g] = mn;
    if (g == my_g) mine = mn;
  }
  float x = __fsub_rn(s, mine);
  if (!mpc) x = fminf(fmaxf(x, -40.0f), 40.0f);
  const float w = valid ? expf(x) : 0.0f;
  float cs = w;
#pragma unroll
  for (int o = GS; o < 32; o <<= 1) cs = __fadd_rn(cs, __shfl_xor_sync(0xffffffffu, cs, o));
#pragma unroll
  for (int g = 0; g < GS; ++g) {
    st.l[g] = __fmaf_rn(st.l[g], alpha[g], __shfl_sync(0xffffffffu, cs, g));
#pragma unroll
    for (int d = 0; d < DPL; ++d) st.acc[g][d] = __fmul_rn(st.acc[g][d], alpha[g]);
  }
#pragma unroll
  for (int j = 0; j < CH; ++j)
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      const float wj = __shfl_sync(0xffffffffu, w, j * GS + g);
#pragma unroll
      for (int d = 0; d < DPL; ++d) st.acc[g][d] = __fmaf_rn(wj, ch.v[j][d], st.acc[g][d]);
    }
}

// Grid (kAttnCluster, head groups, rows), clusters of kAttnCluster CTAs along x: one cluster per
// (query row, head group). The row's positions are cut into chunks of 32 / GS positions, dealt
// round-robin to the cluster's 64 warps; every warp keeps its own online softmax over its chunks
// with K and V in registers, the next chunk loading while one is folded. In decode the first two
// chunks of every warp (all chunks up to 1024 positions at GS = 4) are requested before the wait on
// the q/k/v kernel, except the one row it writes. Warps combine in order within a CTA, CTAs in
// rank order in CTA 0 (distributed shared memory), so results do not depend on timing.
template <int HD, int GS>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_kernel(const AttnArgs a) {
  constexpr int DPL = HD / 32;
  constexpr int CH = 32 / GS;
  constexpr int NW = kAttnCluster * kAttnWarps;  // warps per (row, group)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  AttnSmem<HD, GS>& S = *reinterpret_cast<AttnSmem<HD, GS>*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int gi = blockIdx.y, m = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    pdl_trigger();
    trace_both(a.trace, TR_ENTRY);
  }
  // the head groups are copied in before any kernel of the launch sequence runs
  const int4 grp = a.groups[gi];
  const int kvh = grp.x, qh0 = grp.y, G = grp.z;
  const bool early = a.early_kv != 0;
  if (!early) pdl_wait();  // positions, queries and the cache come from earlier kernels
  const int kv_len = __ldcg(a.pos + m) + 1;
  const int sq = a.seq ? __ldcg(a.seq + m) : 0;
  const float* K = a.Kcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const float* V = a.Vcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const size_t ld = (size_t)a.kvd;
  const bool mpc = a.variant == SHD_NL_MPC;
  const int n_chunks = (kv_len + CH - 1) / CH;
  const int wi = rank * kAttnWarps + warp;
  const int fresh = early ? kv_len - 1 : -1;  // the row the q/k/v kernel of this step writes

  KvChunk<CH, DPL> ca, cb;
  load_chunk<CH, DPL>(ca, K, V, ld, wi, kv_len, fresh, lane);
  load_chunk<CH, DPL>(cb, K, V, ld, wi + NW, kv_len, fresh, lane);
  if (early) {
    pdl_wait();  // queries and this step's K/V row come from the q/k/v kernel
    if (tid == 0) {
      trace_first(a.trace, TR_WAIT);
      trace_last(a.trace, TR_READY);
    }
    const int fc = fresh / CH, fj = fresh % CH;
    if (fc == wi || fc == wi + NW) {
      KvChunk<CH, DPL>& f = (fc == wi) ? ca : cb;
#pragma unroll
      for (int j = 0; j < CH; ++j)
        if (j == fj) {
          load_slice<DPL>(K + (size_t)fresh * ld, lane, f.k[j]);
          load_slice<DPL>(V + (size_t)fresh * ld, lane, f.v[j]);
        }
    }
  }
  float q[GS][DPL];
#pragma unroll
  for (int g = 0; g < GS; ++g) {
    if (g < G) {
      load_slice<DPL>(a.Q + (size_t)m * a.ldq + (size_t)(qh0 + g) * HD, lane, q[g]);
    } else {
#pragma unroll
      for (int d = 0; d < DPL; ++d) q[g][d] = 0.0f;
    }
  }
  WarpSoftmax<GS, DPL> st;
#pragma unroll
  for (int g = 0; g < GS; ++g) {
    st.m[g] = -INFINITY;
    st.l[g] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) st.acc[g][d] = 0.0f;
  }
  for (int c = wi; c < n_chunks; c += 2 * NW) {
    fold_chunk<GS, DPL>(st, ca, q, c, kv_len, a.scale, mpc, lane);
    if (c + 2 * NW < n_chunks) load_chunk<CH, DPL>(ca, K, V, ld, c + 2 * NW, kv_len, -1, lane);
    if (c + NW >= n_chunks) break;
    fold_chunk<GS, DPL>(st, cb, q, c + NW, kv_len, a.scale, mpc, lane);
    if (c + 3 * NW < n_chunks) load_chunk<CH, DPL>(cb, K, V, ld, c + 3 * NW, kv_len, -1, lane);
  }

  // warps -> CTA partial (in warp order), written into CTA 0's gather slot of this rank
#pragma unroll
  for (int g = 0; g < GS; ++g) {
    if (lane == 0) {
      S.wpart[warp][g][0] = st.m[g];
      S.wpart[warp][g][1] = st.l[g];
    }
#pragma unroll
    for (int d = 0; d < DPL; ++d) S.wpart[warp][g][2 + lane * DPL + d] = st.acc[g][d];
  }
  __syncthreads();
  AttnSmem<HD, GS>* root = cluster.map_shared_rank(&S, 0);
  for (int i = tid; i < GS * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;
    float Mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) Mx = fmaxf(Mx, S.wpart[w][g][0]);
    float L = 0.0f, O = 0.0f;
    if (Mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = S.wpart[w][g][0];
        if (mw == -INFINITY) continue;
        const float e = expf(__fsub_rn(mw, Mx));
        L = __fmaf_rn(S.wpart[w][g][1], e, L);
        O = __fmaf_rn(S.wpart[w][g][2 + d], e, O);
      }
    }
    root->gather[rank][g][2 + d] = O;
    if (d == 0) {
      root->gather[rank][g][0] = Mx;
      root->gather[rank][g][1] = L;
    }
  }
  cluster.sync();
  if (rank != 0) {
    if (tid == 0) trace_both(a.trace, TR_EXIT);
    return;
  }

  for (int i = tid; i < GS * HD; i += kAttnThreads) {
    const int g = i / HD, pd = i % HD;
    if (g >= G) continue;
    float Mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kAttnCluster; ++r) Mx = fmaxf(Mx, S.gather[r][g][0]);
    float L = 0.0f, out = 0.0f;
#pragma unroll
    for (int r = 0; r < kAttnCluster; ++r) {
      const float mr = S.gather[r][g][0];
      if (mr == -INFINITY) continue;
      const float w = expf(__fsub_rn(mr, Mx));
      L = __fmaf_rn(S.gather[r][g][1], w, L);
      out = __fmaf_rn(S.gather[r][g][2 + pd], w, out);
    }
    if (mpc && !(L > 1e-10f && isfinite(L))) {
      // compute_mpc_attention_on_shares: weights 1/seq_len when the sum is not usable
      float u = 0.0f;
      for (int tt = 0; tt < kv_len; ++tt) u = __fmaf_rn(__fdiv_rn(1.0f, (float)kv_len), V[(size_t)tt * ld + pd], u);
      out = u;
    } else {
      out = __fdiv_rn(out, L);
    }
    const int h = qh0 + g;
    const size_t o = (size_t)m * a.ldo + (size_t)h * HD + pd;
    const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + (size_t)h * HD + pd] : 0.0f;
    a.Oc[o] = __fsub_rn(out, mk);
    a.Os[o] = mk;
  }
  if (tid == 0) trace_both(a.trace, TR_EXIT);
}

// Wide groups (8 query heads: batched rows, one group per kv head) use the tile kernel below: per
// position the register-chunk kernel's shuffles double at 8 heads and its registers allow one CTA per
// SM, while here a CTA walks its eighth of the positions in 32-position tiles staged in shared
// memory (double-buffered cp.async), warps split head_dim and lanes the positions for the scores,
// and two CTAs fit an SM. Measured on the 14B 8-row step: 40 us per layer against 63 us.
constexpr int kAttnTile = 32;     // positions per tile

template <int HD, int GS>
struct TileSmem {
  static constexpr int KS = HD + 4;  // padded row stride (conflict-free column reads)
  float k[2][kAttnTile][KS];         // double-buffered: the next tile loads during this one
  float v[2][kAttnTile][HD];
  float q[GS][HD];
  float spart[kAttnThreads / 32][GS][kAttnTile];  // per-warp partial dots
  float p[GS][kAttnTile];                         // tile weights
  float m[GS], l[GS], alpha[GS];
  float gather[kAttnCluster][GS][HD + 2];         // CTA 0: partials of the cluster
};

template <int HD, int GS>
__global__ void __launch_bounds__(kAttnThreads) attn_tile_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  TileSmem<HD, GS>& S = *reinterpret_cast<TileSmem<HD, GS>*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int gi = blockIdx.y, m = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = kAttnThreads / 32;  // 8 warps
  constexpr int DW = HD / NW;            // dims per warp in the score phase (16 or 8)
  if (tid == 0) {
    pdl_trigger();
    trace_both(a.trace, TR_ENTRY);
  }
  // the head groups are copied in before any kernel of the launch sequence runs
  const int4 grp = a.groups[gi];
  const int kvh = grp.x, qh0 = grp.y, G = grp.z;
  const bool early = a.early_kv != 0;
  if (!early) pdl_wait();  // positions, queries and the cache come from earlier kernels
  const int kv_len = __ldcg(a.pos + m) + 1;
  const int sq = a.seq ? __ldcg(a.seq + m) : 0;
  const int per = (kv_len + kAttnCluster - 1) / kAttnCluster;
  const int t0 = min(rank * per, kv_len), t1 = min(t0 + per, kv_len);
  const float* K = a.Kcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const float* V = a.Vcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * HD;
  const bool mpc = a.variant == SHD_NL_MPC;

  // K and V rows [tb + r_lo, tb + r_hi) of a tile: 16-byte asynchronous copies (L2 only); rows of
  // the tile past the split's end are zero-filled with the first part
  auto stage_rows = [&](int buf, int tb, int r_lo, int r_hi) {
    const int nt = min(kAttnTile, t1 - tb);
    for (int i = tid; i < (r_hi - r_lo) * (HD / 4); i += kAttnThreads) {
      const int r = r_lo + i / (HD / 4), c4 = i % (HD / 4);
      const int row = (r < nt) ? tb + r : tb;  // an in-range address even when nothing is copied
      const uint32_t bytes = (r < nt) ? 16u : 0u;
      cp_async16(&S.k[buf][r][4 * c4], K + (size_t)row * a.kvd + 4 * c4, bytes);
      cp_async16(&S.v[buf][r][4 * c4], V + (size_t)row * a.kvd + 4 * c4, bytes);
    }
    cp_async_commit();
  };
  auto stage_tile = [&](int buf, int tb) { stage_rows(buf, tb, 0, kAttnTile); };
  if (early) {
    // every row of tile 0 but this step's own (kv_len - 1) before the wait, that row after it
    const int r_new = kv_len - 1 - t0;  // within tile 0 when 0 <= r_new < kAttnTile
    if (t0 < t1) {
      if (r_new >= 0 && r_new < kAttnTile) {
        stage_rows(0, t0, 0, r_new);
        stage_rows(0, t0, r_new + 1, kAttnTile);
      } else {
        stage_tile(0, t0);
      }
    }
    pdl_wait();  // queries and this step's K/V row come from the q/k/v kernel
    if (tid == 0) {
      trace_first(a.trace, TR_WAIT);
      trace_last(a.trace, TR_READY);
    }
    if (t0 < t1 && r_new >= 0 && r_new < kAttnTile) stage_rows(0, t0, r_new, r_new + 1);
  } else if (t0 < t1) {
    stage_tile(0, t0);  // in flight while the queries load
  }

  for (int i = tid; i < GS * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;
    S.q[g][d] = (g < G) ? a.Q[(size_t)m * a.ldq + (size_t)(qh0 + g) * HD + d] : 0.0f;
  }
  if (tid < GS) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.0f;
  }
  // PV mapping: thread -> dim d, heads g0 and g0 + 2 (kAttnThreads = 2 * HD for HD = 128)
  constexpr int GPT = GS * HD / kAttnThreads;  // heads per thread: 2 (HD 128) or 1 (HD 64)
  float acc[GPT];
#pragma unroll
  for (int j = 0; j < GPT; ++j) acc[j] = 0.0f;
  const int pd = tid % HD, pg0 = tid / HD;  // head of acc[j] = pg0 + j * (kAttnThreads / HD)
  __syncthreads();

  // this warp's slice of the queries: in registers for groups of up to 4 heads, read from shared
  // memory (the same float4 for every lane) for wider groups
  constexpr bool kQReg = GS <= 4;
  float qreg[kQReg ? GS : 1][kQReg ? DW : 1];
  if constexpr (kQReg) {
#pragma unroll
    for (int g = 0; g < GS; ++g)
#pragma unroll
      for (int j = 0; j < DW; ++j) qreg[g][j] = S.q[g][warp * DW + j];
  }

  int buf = 0;
  for (int tb = t0; tb < t1; tb += kAttnTile, buf ^= 1) {
    const int nt = min(kAttnTile, t1 - tb);
    if (tb + kAttnTile < t1) {
      stage_tile(buf ^ 1, tb + kAttnTile);
      cp_async_wait<1>();  // this tile's copies have landed (the next tile's may be in flight)
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // partial dots: warp = dim slice, lane = position
    {
      float part[GS];
#pragma unroll
      for (int g = 0; g < GS; ++g) part[g] = 0.0f;
#pragma unroll
      for (int j = 0; j < DW; j += 4) {
        const float4 kk = *reinterpret_cast<const float4*>(&S.k[buf][lane][warp * DW + j]);
#pragma unroll
        for (int g = 0; g < GS; ++g) {
          float4 qq;
          if constexpr (kQReg)
            qq = make_float4(qreg[g][j + 0], qreg[g][j + 1], qreg[g][j + 2], qreg[g][j + 3]);
          else
            qq = *reinterpret_cast<const float4*>(&S.q[g][warp * DW + j]);
          part[g] = __fmaf_rn(qq.x, kk.x, part[g]);
          part[g] = __fmaf_rn(qq.y, kk.y, part[g]);
          part[g] = __fmaf_rn(qq.z, kk.z, part[g]);
          part[g] = __fmaf_rn(qq.w, kk.w, part[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < GS; ++g) S.spart[warp][g][lane] = part[g];
    }
    __syncthreads();
    // scores and online softmax: warp g (< G) owns head g, lane = position
    if (warp < G) {
      const int g = warp;
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s = __fadd_rn(s, S.spart[w][g][lane]);
      s = (lane < nt) ? __fmul_rn(s, a.scale) : -INFINITY;
      float tmax = s;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mold = S.m[g];
      const float mnew = fmaxf(mold, tmax);
      float x = __fsub_rn(s, mnew);
      if (!mpc) x = fminf(fmaxf(x, -40.0f), 40.0f);
      const float pe = (lane < nt) ? expf(x) : 0.0f;
      float tsum = pe;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) tsum = __fadd_rn(tsum, __shfl_xor_sync(0xffffffffu, tsum, o));
      S.p[g][lane] = pe;
      __syncwarp();
      if (lane == 0) {
        const float al = (mold == -INFINITY) ? 0.0f : expf(__fsub_rn(mold, mnew));
        S.alpha[g] = al;
        S.l[g] = __fmaf_rn(S.l[g], al, tsum);
        S.m[g] = mnew;
      }
    }
    __syncthreads();
    // weighted V: thread -> (dim, its heads). Wide groups: each V element is loaded once for all of
    // the thread's heads and the weights 4 positions at a time (rows past the tile's end have p = 0
    // and V = 0); measured faster at 8-head groups, slower at 4 (single-row decode), which keeps
    // the per-head loop.
    if constexpr (GS <= 4) {
#pragma unroll
      for (int j = 0; j < GPT; ++j) {
        const int g = pg0 + j * (kAttnThreads / HD);
        if (g < G) {
          float v = __fmul_rn(acc[j], S.alpha[g]);
          for (int r = 0; r < nt; ++r) v = __fmaf_rn(S.p[g][r], S.v[buf][r][pd], v);
          acc[j] = v;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < GPT; ++j) {
        const int g = pg0 + j * (kAttnThreads / HD);
        if (g < G) acc[j] = __fmul_rn(acc[j], S.alpha[g]);
      }
      for (int r = 0; r < nt; r += 4) {
        const float v0 = S.v[buf][r][pd], v1 = S.v[buf][r + 1][pd];
        const float v2 = S.v[buf][r + 2][pd], v3 = S.v[buf][r + 3][pd];
#pragma unroll
        for (int j = 0; j < GPT; ++j) {
          const int g = pg0 + j * (kAttnThreads / HD);
          if (g < G) {
            const float4 pp = *reinterpret_cast<const float4*>(&S.p[g][r]);
            float v = acc[j];
            v = __fmaf_rn(pp.x, v0, v);
            v = __fmaf_rn(pp.y, v1, v);
            v = __fmaf_rn(pp.z, v2, v);
            v = __fmaf_rn(pp.w, v3, v);
            acc[j] = v;
          }
        }
      }
    }
    __syncthreads();  // this buffer is refilled two tiles later
  }

  // gather the cluster's partials into CTA 0 (distributed shared memory), then combine in rank order
  TileSmem<HD, GS>* root = cluster.map_shared_rank(&S, 0);
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int g = pg0 + j * (kAttnThreads / HD);
    if (g < G) root->gather[rank][g][2 + pd] = acc[j];
  }
  if (tid < G) {
    root->gather[rank][tid][0] = S.m[tid];
    root->gather[rank][tid][1] = S.l[tid];
  }
  cluster.sync();
  if (rank != 0) {
    if (tid == 0) trace_both(a.trace, TR_EXIT);
    return;
  }

#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int g = pg0 + j * (kAttnThreads / HD);
    if (g >= G) continue;
    float Mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kAttnCluster; ++r) Mx = fmaxf(Mx, S.gather[r][g][0]);
    float L = 0.0f, out = 0.0f;
#pragma unroll
    for (int r = 0; r < kAttnCluster; ++r) {
      const float mr = S.gather[r][g][0];
      if (mr == -INFINITY) continue;
      const float w = expf(__fsub_rn(mr, Mx));
      L = __fmaf_rn(S.gather[r][g][1], w, L);
      out = __fmaf_rn(S.gather[r][g][2 + pd], w, out);
    }
    if (mpc && !(L > 1e-10f && isfinite(L))) {
      // compute_mpc_attention_on_shares: weights 1/seq_len when the sum is not usable
      float u = 0.0f;
      for (int tt = 0; tt < kv_len; ++tt) u = __fmaf_rn(__fdiv_rn(1.0f, (float)kv_len), V[(size_t)tt * a.kvd + pd], u);
      out = u;
    } else {
      out = __fdiv_rn(out, L);
    }
    const int h = qh0 + g;
    const size_t o = (size_t)m * a.ldo + (size_t)h * HD + pd;
    const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + (size_t)h * HD + pd] : 0.0f;
    a.Oc[o] = __fsub_rn(out, mk);
    a.Os[o] = mk;
  }
  if (tid == 0) trace_both(a.trace, TR_EXIT);
}

template <typename Kern>
static int launch_cluster(shd_ctx* ctx, Kern kernel, size_t smem, unsigned& attr_devices, const AttnArgs& a,
                          int M) {
  if (!(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_devices |= 1u << (ctx->device & 31);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kAttnCluster, a.n_groups, M);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kAttnCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  SHD_CHECK_CUDA(ctx, cudaLaunchKernelEx(&cfg, kernel, a));
  ctx->launches++;
  return SHD_OK;
}

// Groups of up to 4 query heads: the register-chunk kernel; 8-head groups: the tile kernel.
template <int HD, int GS>
static int launch_attn_t(shd_ctx* ctx, const AttnArgs& a, int M) {
  static unsigned attr_devices = 0;
  if constexpr (GS == 8)
    return launch_cluster(ctx, attn_tile_kernel<HD, GS>, sizeof(TileSmem<HD, GS>), attr_devices, a, M);
  else
    return launch_cluster(ctx, attn_decode_kernel<HD, GS>, sizeof(AttnSmem<HD, GS>), attr_devices, a, M);
}

int launch_attention(shd_ctx* ctx, const AttnArgs& a, int M) {
  // group_cap 8: groups of up to 8 q heads (one per kv head for groups of 5-8), else up to 4
  if (a.group_cap == 8) {
    if (a.head_dim == 128) return launch_attn_t<128, 8>(ctx, a, M);
    if (a.head_dim == 64) return launch_attn_t<64, 8>(ctx, a, M);
  }
  if (a.head_dim == 128) return launch_attn_t<128, kAttnGroup>(ctx, a, M);
  if (a.head_dim == 64) return launch_attn_t<64, kAttnGroup>(ctx, a, M);
  return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
}

// Consecutive local q heads with the same kv head, cut into near-equal groups of <= cap.
std::vector<int4> attn_groups(int q_begin, int q_count, int kv_begin, int group, int cap) {
  std::vector<int4> out;
  int i = 0;
  while (i < q_count) {
    const int kv = (q_begin + i) / group;
    int n = 0;
    while (i + n < q_count && (q_begin + i + n) / group == kv) ++n;
    const int parts = (n + cap - 1) / cap;
    int done = 0;
    for (int p = 0; p < parts; ++p) {
      const int cnt = (n - done) / (parts - p);
      out.push_back(make_int4(kv - kv_begin, i + done, cnt, 0));
      done += cnt;
    }
    i += n;
  }
  return out;
}

}  // namespace shd

using namespace shd;


extern "C" int shd_attn_decode(shd_ctx* ctx, const float* q, const float* k_cache,
                               const float* v_cache, int kv_capacity, int H, int Hkv, int head_dim,
                               const int32_t* pos_host, int M, int variant, const float* mask,
                               float* out_c, float* out_s) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, q && k_cache && v_cache && pos_host && out_c && out_s, "shd_attn_decode: null pointer");
  SHD_REQUIRE(ctx, H > 0 && Hkv > 0 && H % Hkv == 0, "shd_attn_decode: num_heads must be a multiple of num_kv_heads");
  SHD_REQUIRE(ctx, head_dim == 64 || head_dim == 128, "shd_attn_decode: head_dim must be 64 or 128");
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_attn_decode: unknown variant");
  SHD_REQUIRE(ctx, M > 0 && kv_capacity > 0, "shd_attn_decode: bad shape");
  for (int i = 0; i < M; ++i)
    SHD_REQUIRE(ctx, pos_host[i] >= 0 && pos_host[i] < kv_capacity, "shd_attn_decode: position outside the cache");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  // from 4 rows, one group of up to 8 q heads per kv head (each K/V row read once), as the model does
  const int cap = (M >= 4 && H / Hkv > kAttnGroup) ? 8 : kAttnGroup;
  const std::vector<int4> groups = attn_groups(0, H, 0, H / Hkv, cap);
  const int ng = (int)groups.size();
  // staging of groups and positions (the context's buffer: the call synchronizes before returning)
  int* d_meta = nullptr;
  const size_t meta_bytes = (size_t)ng * 16 + (size_t)M * 4;
  {
    void* p = nullptr;
    const int src = shd_stage(ctx, meta_bytes, &p);
    if (src) return src;
    d_meta = static_cast<int*>(p);
  }
  std::vector<int> meta(meta_bytes / 4);
  std::memcpy(meta.data(), groups.data(), (size_t)ng * 16);
  for (int i = 0; i < M; ++i) meta[4 * ng + i] = pos_host[i];
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(d_meta, meta.data(), meta_bytes, cudaMemcpyHostToDevice, ctx->stream));
  AttnArgs a{};
  a.Q = q;
  a.ldq = H * head_dim;
  a.Kcache = k_cache;
  a.Vcache = v_cache;
  a.kvd = Hkv * head_dim;
  a.kv_seq_stride = (int64_t)kv_capacity * a.kvd;
  a.groups = reinterpret_cast<const int4*>(d_meta);
  a.n_groups = ng;
  a.head_dim = head_dim;
  a.pos = d_meta + 4 * ng;
  a.seq = nullptr;
  a.variant = variant;
  a.scale = 1.0f / sqrtf((float)head_dim);
  a.mask = mask;
  a.ldmask = H * head_dim;
  a.Oc = out_c;
  a.Os = out_s;
  a.ldo = H * head_dim;
  a.group_cap = cap;
  a.err = ctx->d_err;
  int rc = launch_attention(ctx, a, M);
  // the host staging vector must outlive the async copy
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return shd_cuda_fail(ctx, e, "shd_attn_decode");
  return rc;
}

extern "C" int shd_attn_prefill(shd_ctx* ctx, const float* q, const float* k_cache, const float* v_cache,
                                int kv_capacity, int H, int Hkv, int head_dim, int pos0, int M, int variant,
                                const float* mask, float* out_c, float* out_s) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, q && k_cache && v_cache && out_c && out_s, "shd_attn_prefill: null pointer");
  SHD_REQUIRE(ctx, H > 0 && Hkv > 0 && H % Hkv == 0, "shd_attn_prefill: num_heads must be a multiple of num_kv_heads");
  SHD_REQUIRE(ctx, head_dim == 128, "shd_attn_prefill: head_dim must be 128");
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_attn_prefill: unknown variant");
  SHD_REQUIRE(ctx, M > 0 && pos0 >= 0 && pos0 + M <= kv_capacity, "shd_attn_prefill: positions outside the cache");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const std::vector<int4> groups = attn_groups(0, H, 0, H / Hkv, 8);
  const int ng = (int)groups.size();
  int* d_meta = nullptr;
  const size_t meta_bytes = (size_t)ng * 16 + 16;
  {
    void* p = nullptr;
    const int src = shd_stage(ctx, meta_bytes, &p);
    if (src) return src;
    d_meta = static_cast<int*>(p);
  }
  std::vector<int> meta(meta_bytes / 4, 0);
  std::memcpy(meta.data(), groups.data(), (size_t)ng * 16);
  meta[4 * ng] = pos0;
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(d_meta, meta.data(), meta_bytes, cudaMemcpyHostToDevice, ctx->stream));
  AttnArgs a{};
  a.Q = q;
  a.ldq = H * head_dim;
  a.Kcache = k_cache;
  a.Vcache = v_cache;
  a.kvd = Hkv * head_dim;
  a.kv_seq_stride = (int64_t)kv_capacity * a.kvd;
  a.groups = reinterpret_cast<const int4*>(d_meta);
  a.n_groups = ng;
  a.head_dim = head_dim;
  a.pos = d_meta + 4 * ng;
  a.seq = nullptr;
  a.variant = variant;
  a.scale = 1.0f / sqrtf((float)head_dim);
  a.mask = mask;
  a.ldmask = H * head_dim;
  a.Oc = out_c;
  a.Os = out_s;
  a.ldo = H * head_dim;
  a.group_cap = 8;
  a.err = ctx->d_err;
  int rc = flash_prefill_supported(a, M) ? launch_flash_prefill(ctx, a, M)
                                         : shd_fail(ctx, SHD_ERR_ARG, "shd_attn_prefill: rows must be 16-byte aligned");
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return shd_cuda_fail(ctx, e, "shd_attn_prefill");
  return rc;
}
