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
#include <algorithm>

#include "shd_gemv.cuh"

namespace shd {

// Dynamic shared memory available per CTA on sm_100 (227 KB) minus room for the tile result and
// the barriers; the pipeline gets as many stages as fit, at most 12.
constexpr int kSmemBudget = 232448 - 4608;
constexpr int stages_for(int stage_bytes) {
  return (kSmemBudget / stage_bytes) > 12 ? 12 : (kSmemBudget / stage_bytes);
}

template <int M>
struct F32Cfg {
  static constexpr int XB = kChunkBf16 * 4;             // bytes of one (row, share) x chunk
  static constexpr int STAGE = kBlockBytes + M * 2 * XB;
  static constexpr int S = stages_for(STAGE);           // pipeline depth
  static constexpr int V = 4 * 2 * M;                   // accumulators per lane
  static constexpr int TSUM = kTileRows * 2 * M;        // floats of one tile's result
  static constexpr size_t SMEM = (size_t)S * STAGE + TSUM * 4 + (2 * S + 2) * 8 + 16;
};

template <int M>
struct RingCfg {
  static constexpr int XB = kChunkI32 * 4;
  static constexpr int STAGE = kBlockBytes + M * 2 * XB;
  static constexpr int S = stages_for(STAGE);
  static constexpr int V = 4 * 2 * M;
  static constexpr int TSUM = kTileRows * 2 * M;
  static constexpr size_t SMEM = (size_t)S * STAGE + TSUM * 8 + (2 * S + 2) * 8 + 16;
};

// Stream-K bookkeeping: CTA g owns units [b_g, b_{g+1}), b_g = floor(U g / G).
__device__ __forceinline__ long long unit_begin(long long U, int G, int g) {
  return U * g / G;
}
__device__ __forceinline__ int unit_owner(long long U, int G, long long u) {
  return (int)(((u + 1) * (long long)G - 1) / U);
}

// Reduce V per-lane values over the warp with a reduce-scatter butterfly. Afterwards this lane
// holds `cnt` fully reduced values with flat indices [base, base+cnt); lanes with any bit of
// `dup` set hold duplicates and must not write.
template <typename T, int V>
__device__ __forceinline__ void warp_reduce_scatter(T (&v)[V], int lane, int& base, int& cnt,
                                                    unsigned& dup) {
  int n = V;
  base = 0;
  dup = 0;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const int half = n / 2;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < V / 2; ++j) {
        if (j < half) {
          const T lo = v[j], hi = v[j + half];
          const T send = up ? lo : hi;
          const T keep = up ? hi : lo;
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      if (up) base += half;
      n = half;
    } else {
      v[0] = v[0] + __shfl_xor_sync(0xffffffffu, v[0], o);
      dup |= (unsigned)o;
    }
  }
  cnt = n;
}

// Warp-uniform bounded wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  bool ok = mbar_wait_bounded(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

struct PipeSmem {
  uint8_t* stages;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* cbar;  // consumer-group barrier (8 warp arrivals)
  volatile int* flags;  // [0] abort, [1] last-arriver flag
};

// Producer: one elected lane streams the weight block and the x chunks of every unit.
template <int S, int STAGE, int M, int CHUNK, typename XT>
__device__ void gemv_producer(const PipeSmem& sm, const uint8_t* W, const XT* Xc, const XT* Xs,
                              int ldx, int K, int nKC, long long u0, long long u1, int* err) {
  const uint64_t pol_w = l2_policy_evict_first();
  const uint64_t pol_x = l2_policy_evict_last();
  int i = 0;
  long long u = u0;
  for (; u < u1; ++u, ++i) {
    const int s = i % S;
    const uint32_t ph = (uint32_t)(i / S) & 1u;
    if (i >= S) {
      if (!mbar_wait_bounded(&sm.empty[s], ph ^ 1u)) {
        atomicOr(err, SHD_DEVERR_TIMEOUT_EMPTY);
        sm.flags[0] = 1;
        break;
      }
    }
    if (sm.flags[0]) break;
    const int c = (int)(u % nKC);
    const int rem = min(CHUNK, K - c * CHUNK);
    const uint32_t xbytes = (uint32_t)rem * 4u;
    uint8_t* st = sm.stages + (size_t)s * STAGE;
    mbar_arrive_expect_tx(&sm.full[s], (uint32_t)kBlockBytes + (uint32_t)(M * 2) * xbytes);
    bulk_g2s(st, W + (size_t)u * kBlockBytes, kBlockBytes, &sm.full[s], pol_w);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      bulk_g2s(st + kBlockBytes + (m * 2 + 0) * (CHUNK * 4), Xc + (size_t)m * ldx + (size_t)c * CHUNK,
               xbytes, &sm.full[s], pol_x);
      bulk_g2s(st + kBlockBytes + (m * 2 + 1) * (CHUNK * 4), Xs + (size_t)m * ldx + (size_t)c * CHUNK,
               xbytes, &sm.full[s], pol_x);
    }
  }
  if (u < u1) {
    // Aborted: wait (bounded) for the last copy issued into every stage before leaving, so that no
    // bulk copy lands in shared memory of a CTA that has exited.
    const int issued = i;
    for (int k = max(0, issued - S); k < issued; ++k) {
      const int s = k % S;
      if (!mbar_wait_bounded(&sm.full[s], (uint32_t)(k / S) & 1u)) {
        atomicOr(err, SHD_DEVERR_TIMEOUT_DRAIN);
      }
    }
  }
}

// Consumer-group barrier over the 8 consumer warps, bounded.
__device__ __forceinline__ bool consumer_sync(const PipeSmem& sm, uint32_t& phase, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.cbar);
  const bool ok = warp_wait(sm.cbar, phase);
  phase ^= 1u;
  return ok;
}

// ------------------------------------------------------------------------------------------------
// f32-share epilogues. tsum layout: [(row * 2 + share) * M + m].
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float silu_variant(float g, int variant) {
  if (variant == SHD_NL_APPROX) {
    // secure_swiglu_approx: sigmoid of the clamped gate times the unclamped gate.
    const float gc = fminf(fmaxf(g, -20.0f), 20.0f);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gc)));
    return __fmul_rn(g, sig);
  } else if (variant == SHD_NL_GPU) {
    // silu_kernel: x / (1 + expf(-x)).
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  } else {
    // secure_swiglu_mpc: exact SiLU, zero for non-finite input.
    if (!isfinite(g)) return 0.0f;
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(g, sig);
  }
}

__device__ __forceinline__ float swiglu_variant(float g, float u, int variant) {
  const float s = silu_variant(g, variant);
  if (variant == SHD_NL_MPC) {
    if (!(isfinite(s) && isfinite(u))) return 0.0f;
    const float p = __fmul_rn(s, u);
    return isfinite(p) ? p : 0.0f;
  }
  return __fmul_rn(s, u);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal in the reference; tie -> later index
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned)idx;
}

template <int M, int EPI>
__device__ void epilogue_f32(const GemvArgs& a, int t, const float* tsum, int ctid, int* err) {
  if constexpr (EPI == EPI_STORE) {
    for (int idx = ctid; idx < kTileRows * M; idx += kConsumerWarps * 32) {
      const int r = idx % kTileRows, m = idx / kTileRows;
      const int n = t * kTileRows + r;
      if (n >= a.N) continue;
      float yc = tsum[(r * 2 + 0) * M + m];
      float ys = tsum[(r * 2 + 1) * M + m];
      if (a.bias) ys = __fadd_rn(ys, a.bias[n]);
      if (a.Rc) {
        yc = __fadd_rn(yc, a.Rc[(size_t)m * a.ldr + n]);
        ys = __fadd_rn(ys, a.Rs[(size_t)m * a.ldr + n]);
      }
      a.Yc[(size_t)m * a.ldy + n] = yc;
      a.Ys[(size_t)m * a.ldy + n] = ys;
    }
  } else if constexpr (EPI == EPI_QKV) {
    const int hd = a.head_dim, half = hd >> 1;
    for (int idx = ctid; idx < (kTileRows / 2) * M; idx += kConsumerWarps * 32) {
      const int pr = idx % (kTileRows / 2), m = idx / (kTileRows / 2);
      const int r0 = 2 * pr, r1 = r0 + 1;
      const int np = t * kTileRows + r0;  // permuted row index of the pair's first row
      if (np >= a.N) continue;
      const int head = np / hd;
      const int p = (np % hd) >> 1;
      const int n0 = head * hd + p, n1 = n0 + half;  // output indices
      float x0c = tsum[(r0 * 2 + 0) * M + m], x0s = tsum[(r0 * 2 + 1) * M + m];
      float x1c = tsum[(r1 * 2 + 0) * M + m], x1s = tsum[(r1 * 2 + 1) * M + m];
      if (a.bias) {
        x0s = __fadd_rn(x0s, a.bias[np]);
        x1s = __fadd_rn(x1s, a.bias[np + 1]);
      }
      const int pos = a.pos ? a.pos[m] : 0;
      const bool rot = n0 < a.q_dim + a.kv_dim;
      if (rot) {
        if (pos < 0 || pos >= a.rope_max_seq) {
          atomicOr(err, SHD_DEVERR_ARG);
          continue;
        }
        // RopeFrequencies::apply_to_share (secure_attention.rs:84-121), each share on its own:
        // [x0 c - x1 s, x0 s + x1 c], no fused multiply-add.
        const float cs = a.rope_cos[(size_t)pos * half + p];
        const float sn = a.rope_sin[(size_t)pos * half + p];
        const float y0c = __fsub_rn(__fmul_rn(x0c, cs), __fmul_rn(x1c, sn));
        const float y1c = __fadd_rn(__fmul_rn(x0c, sn), __fmul_rn(x1c, cs));
        const float y0s = __fsub_rn(__fmul_rn(x0s, cs), __fmul_rn(x1s, sn));
        const float y1s = __fadd_rn(__fmul_rn(x0s, sn), __fmul_rn(x1s, cs));
        x0c = y0c;
        x1c = y1c;
        x0s = y0s;
        x1s = y1s;
      }
      if (a.Yc) {
        a.Yc[(size_t)m * a.ldy + n0] = x0c;
        a.Yc[(size_t)m * a.ldy + n1] = x1c;
        a.Ys[(size_t)m * a.ldy + n0] = x0s;
        a.Ys[(size_t)m * a.ldy + n1] = x1s;
      }
      const float v0 = __fadd_rn(x0c, x0s), v1 = __fadd_rn(x1c, x1s);
      if (n0 < a.q_dim) {
        if (a.Q) {
          a.Q[(size_t)m * a.ldq + n0] = v0;
          a.Q[(size_t)m * a.ldq + n1] = v1;
        }
      } else {
        float* cache = (n0 < a.q_dim + a.kv_dim) ? a.Kcache : a.Vcache;
        const int off = (n0 < a.q_dim + a.kv_dim) ? (n0 - a.q_dim) : (n0 - a.q_dim - a.kv_dim);
        if (cache) {
          const int sq = a.seq ? a.seq[m] : 0;
          float* row = cache + (size_t)sq * a.kv_seq_stride + (size_t)pos * a.kv_dim;
          row[off] = v0;
          row[off + half] = v1;
        }
      }
    }
  } else if constexpr (EPI == EPI_GATEUP) {
    const int I = a.N >> 1;
    for (int idx = ctid; idx < (kTileRows / 2) * M; idx += kConsumerWarps * 32) {
      const int r = idx % (kTileRows / 2), m = idx / (kTileRows / 2);
      const int i = t * (kTileRows / 2) + r;
      if (i >= I) continue;
      const float g = __fadd_rn(tsum[(r * 2 + 0) * M + m], tsum[(r * 2 + 1) * M + m]);
      const int ru = r + kTileRows / 2;
      const float u = __fadd_rn(tsum[(ru * 2 + 0) * M + m], tsum[(ru * 2 + 1) * M + m]);
      const float y = swiglu_variant(g, u, a.variant);
      const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + i] : 0.0f;
      a.Yc[(size_t)m * a.ldy + i] = __fsub_rn(y, mk);
      a.Ys[(size_t)m * a.ldy + i] = mk;
    }
  } else {  // EPI_LOGITS
    const int lane = ctid & 31;
    for (int base = 0; base < kTileRows * M; base += kConsumerWarps * 32) {
      const int idx = base + ctid;
      const int r = idx % kTileRows, m = idx / kTileRows;
      const int n = t * kTileRows + r;
      unsigned long long key = 0ull;
      bool nan = false;
      if (idx < kTileRows * M && n < a.N) {
        const float yc = tsum[(r * 2 + 0) * M + m];
        const float ys = tsum[(r * 2 + 1) * M + m];
        if (a.Yc) {
          a.Yc[(size_t)m * a.ldy + n] = yc;
          a.Ys[(size_t)m * a.ldy + n] = ys;
        }
        const float l = __fadd_rn(yc, ys);
        nan = isnan(l);
        key = argmax_key(l, n + a.idx_offset);
      }
      if (__any_sync(0xffffffffu, nan) && lane == 0) atomicOr(err, SHD_DEVERR_NONFINITE);
      // a warp's 32 entries share one m because 32 divides the tile height
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane == 0 && idx < kTileRows * M && key != 0ull) atomicMax(&a.amax[m], key);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// f32-share GEMV kernel (bf16 weights)
// ------------------------------------------------------------------------------------------------
template <int M, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_f32_kernel(const __grid_constant__ GemvArgs a) {
  using C = F32Cfg<M>;
  extern __shared__ __align__(1024) uint8_t smem[];
  PipeSmem sm;
  sm.stages = smem;
  float* tsum = reinterpret_cast<float*>(smem + (size_t)C::S * C::STAGE);
  sm.full = reinterpret_cast<uint64_t*>(tsum + C::TSUM);
  sm.empty = sm.full + C::S;
  sm.cbar = sm.empty + C::S;
  sm.flags = reinterpret_cast<volatile int*>(sm.cbar + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = (long long)a.nT * a.nKC;
  const int G = gridDim.x, g = blockIdx.x;
  const long long u0 = unit_begin(U, G, g), u1 = unit_begin(U, G, g + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(sm.cbar, kConsumerWarps);
    sm.flags[0] = 0;
    sm.flags[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0)
      gemv_producer<C::S, C::STAGE, M, kChunkBf16, float>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC,
                                                          u0, u1, a.err);
    return;
  }

  const int ctid = threadIdx.x;  // 0..255 among consumers
  const int first_tile = (int)(u0 / a.nKC);
  uint32_t cphase = 0;
  float acc[C::V];
#pragma unroll
  for (int j = 0; j < C::V; ++j) acc[j] = 0.f;

  int i = 0;
  for (long long u = u0; u < u1; ++u, ++i) {
    const int s = i % C::S;
    const uint32_t ph = (uint32_t)(i / C::S) & 1u;
    if (!warp_wait(&sm.full[s], ph)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    const int t = (int)(u / a.nKC), c = (int)(u % a.nKC);
    const uint8_t* st = sm.stages + (size_t)s * C::STAGE;
    const float* xsm = reinterpret_cast<const float*>(st + kBlockBytes);
    const bool okA = c * kChunkBf16 + 4 * lane < a.K;
    const bool okB = c * kChunkBf16 + 128 + 4 * lane < a.K;
    const uint4* wv = reinterpret_cast<const uint4*>(st);
    float wf[4][8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint4 q = wv[(warp * 4 + r) * 32 + lane];
      wf[r][0] = bf16lo_to_f32(q.x);
      wf[r][1] = bf16hi_to_f32(q.x);
      wf[r][2] = bf16lo_to_f32(q.y);
      wf[r][3] = bf16hi_to_f32(q.y);
      wf[r][4] = bf16lo_to_f32(q.z);
      wf[r][5] = bf16hi_to_f32(q.z);
      wf[r][6] = bf16lo_to_f32(q.w);
      wf[r][7] = bf16hi_to_f32(q.w);
    }
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int sh = 0; sh < 2; ++sh) {
        const float* xp = xsm + (m * 2 + sh) * kChunkBf16;
        const float4 xa = okA ? *reinterpret_cast<const float4*>(xp + 4 * lane) : z4;
        const float4 xb = okB ? *reinterpret_cast<const float4*>(xp + 128 + 4 * lane) : z4;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = acc[(r * 2 + sh) * M + m];
          v = fmaf(wf[r][0], xa.x, v);
          v = fmaf(wf[r][1], xa.y, v);
          v = fmaf(wf[r][2], xa.z, v);
          v = fmaf(wf[r][3], xa.w, v);
          v = fmaf(wf[r][4], xb.x, v);
          v = fmaf(wf[r][5], xb.y, v);
          v = fmaf(wf[r][6], xb.z, v);
          v = fmaf(wf[r][7], xb.w, v);
          acc[(r * 2 + sh) * M + m] = v;
        }
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);

    const bool tile_end = (c == a.nKC - 1) || (u == u1 - 1);
    if (!tile_end) continue;

    // ---- this CTA's contribution to tile t is complete ----
    int base, cnt;
    unsigned dup;
    warp_reduce_scatter<float, C::V>(acc, lane, base, cnt, dup);
    if ((lane & dup) == 0) {
#pragma unroll
      for (int j = 0; j < C::V; ++j)
        if (j < cnt) tsum[warp * C::V + base + j] = acc[j];
    }
#pragma unroll
    for (int j = 0; j < C::V; ++j) acc[j] = 0.f;

    const bool full_tile = ((long long)t * a.nKC >= u0) && (c == a.nKC - 1);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    if (!full_tile) {
      const int slot = (t == first_tile) ? 0 : 1;
      float* part = a.partials + ((size_t)g * 2 + slot) * C::TSUM;
      for (int k = ctid; k < C::TSUM; k += kConsumerWarps * 32) part[k] = tsum[k];
      __threadfence();
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      const int gf = unit_owner(U, G, (long long)t * a.nKC);
      const int gl = unit_owner(U, G, (long long)(t + 1) * a.nKC - 1);
      if (ctid == 0) {
        const int old = atomicAdd(&a.counters[t], 1);
        const int last = (old == gl - gf);
        if (last) a.counters[t] = 0;
        sm.flags[1] = last;
      }
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      const bool last = sm.flags[1] != 0;
      if (!last) continue;
      __threadfence();
      for (int k = ctid; k < C::TSUM; k += kConsumerWarps * 32) {
        float sum = 0.f;
        for (int gg = gf; gg <= gl; ++gg) {
          const int ft = (int)(unit_begin(U, G, gg) / a.nKC);
          const int sl = (t == ft) ? 0 : 1;
          sum = (gg == gf) ? __ldcg(a.partials + ((size_t)gg * 2 + sl) * C::TSUM + k)
                           : __fadd_rn(sum, __ldcg(a.partials + ((size_t)gg * 2 + sl) * C::TSUM + k));
        }
        tsum[k] = sum;
      }
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
    }
    epilogue_f32<M, EPI>(a, t, tsum, ctid, a.err);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Ring (Z_2^32) GEMV kernel (i32 weights): acc = sum x*W in wrapping i64, y = (i32)(acc >> scale).
// Tiled format: block (t, c) = rows [32t, 32t+32) x columns [128c, 128c+128) as [32][128] i32.
// ------------------------------------------------------------------------------------------------
template <int M>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_ring_kernel(const __grid_constant__ RingArgs a) {
  using C = RingCfg<M>;
  extern __shared__ __align__(1024) uint8_t smem[];
  PipeSmem sm;
  sm.stages = smem;
  long long* tsum = reinterpret_cast<long long*>(smem + (size_t)C::S * C::STAGE);
  sm.full = reinterpret_cast<uint64_t*>(tsum + C::TSUM);
  sm.empty = sm.full + C::S;
  sm.cbar = sm.empty + C::S;
  sm.flags = reinterpret_cast<volatile int*>(sm.cbar + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = (long long)a.nT * a.nKC;
  const int G = gridDim.x, g = blockIdx.x;
  const long long u0 = unit_begin(U, G, g), u1 = unit_begin(U, G, g + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(sm.cbar, kConsumerWarps);
    sm.flags[0] = 0;
    sm.flags[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0)
      gemv_producer<C::S, C::STAGE, M, kChunkI32, int32_t>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC,
                                                           u0, u1, a.err);
    return;
  }

  const int ctid = threadIdx.x;
  const int first_tile = (int)(u0 / a.nKC);
  uint32_t cphase = 0;
  long long acc[C::V];
#pragma unroll
  for (int j = 0; j < C::V; ++j) acc[j] = 0;

  int i = 0;
  for (long long u = u0; u < u1; ++u, ++i) {
    const int s = i % C::S;
    const uint32_t ph = (uint32_t)(i / C::S) & 1u;
    if (!warp_wait(&sm.full[s], ph)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    const int t = (int)(u / a.nKC), c = (int)(u % a.nKC);
    const uint8_t* st = sm.stages + (size_t)s * C::STAGE;
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

    const bool tile_end = (c == a.nKC - 1) || (u == u1 - 1);
    if (!tile_end) continue;

    int base, cnt;
    unsigned dup;
    warp_reduce_scatter<long long, C::V>(acc, lane, base, cnt, dup);
    if ((lane & dup) == 0) {
#pragma unroll
      for (int j = 0; j < C::V; ++j)
        if (j < cnt) tsum[warp * C::V + base + j] = acc[j];
    }
#pragma unroll
    for (int j = 0; j < C::V; ++j) acc[j] = 0;

    const bool full_tile = ((long long)t * a.nKC >= u0) && (c == a.nKC - 1);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    if (!full_tile) {
      const int slot = (t == first_tile) ? 0 : 1;
      long long* part = a.partials + ((size_t)g * 2 + slot) * C::TSUM;
      for (int k = ctid; k < C::TSUM; k += kConsumerWarps * 32) part[k] = tsum[k];
      __threadfence();
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      const int gf = unit_owner(U, G, (long long)t * a.nKC);
      const int gl = unit_owner(U, G, (long long)(t + 1) * a.nKC - 1);
      if (ctid == 0) {
        const int old = atomicAdd(&a.counters[t], 1);
        const int last = (old == gl - gf);
        if (last) a.counters[t] = 0;
        sm.flags[1] = last;
      }
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      if (!sm.flags[1]) continue;
      __threadfence();
      for (int k = ctid; k < C::TSUM; k += kConsumerWarps * 32) {
        long long sum = 0;
        for (int gg = gf; gg <= gl; ++gg) {
          const int ft = (int)(unit_begin(U, G, gg) / a.nKC);
          const int sl = (t == ft) ? 0 : 1;
          sum += __ldcg(a.partials + ((size_t)gg * 2 + sl) * C::TSUM + k);
        }
        tsum[k] = sum;
      }
      if (!consumer_sync(sm, cphase, lane)) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
    }
    // epilogue: arithmetic shift of the wrapped 64-bit sum, truncation to i32, wrapping bias add
    for (int idx = ctid; idx < kTileRows * M; idx += kConsumerWarps * 32) {
      const int r = idx % kTileRows, m = idx / kTileRows;
      const int n = t * kTileRows + r;
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
template <int M, int EPI>
static int launch_f32_t(shd_ctx* ctx, const shd_weight* w, GemvArgs a) {
  using C = F32Cfg<M>;
  static unsigned attr_devices = 0;  // bit d: attribute set on device d
  if (!(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(gemv_f32_kernel<M, EPI>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_devices |= 1u << (ctx->device & 31);
  }
  const long long U = (long long)w->nT * w->nKC;
  const int G = (int)std::min<long long>(U, ctx->num_sms);
  gemv_f32_kernel<M, EPI><<<G, kGemvThreads, C::SMEM, ctx->stream>>>(a);
  SHD_CHECK_LAUNCH(ctx, "gemv_f32_kernel");
  return SHD_OK;
}

template <int EPI>
static int launch_f32_m(shd_ctx* ctx, const shd_weight* w, int M, GemvArgs a) {
  switch (M) {
    case 1: return launch_f32_t<1, EPI>(ctx, w, a);
    case 2: return launch_f32_t<2, EPI>(ctx, w, a);
    case 4: return launch_f32_t<4, EPI>(ctx, w, a);
    case 8: return launch_f32_t<8, EPI>(ctx, w, a);
    default: return shd_fail(ctx, SHD_ERR_ARG, "gemv: M must be 1, 2, 4 or 8 for one launch");
  }
}

int launch_gemv_f32(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs a) {
  a.W = reinterpret_cast<const uint8_t*>(w->d_tiles);
  a.N = w->N;
  a.K = (w->K + 3) / 4 * 4;  // x extent copied per row (rows padded to 16 bytes)
  a.nT = w->nT;
  a.nKC = w->nKC;
  a.partials = ctx->d_partials;
  a.counters = ctx->d_counters;
  a.err = ctx->d_err;
  if (w->nT > ctx->n_counters) return shd_fail(ctx, SHD_ERR_ARG, "gemv: too many row tiles");
  switch (epi) {
    case EPI_STORE: return launch_f32_m<EPI_STORE>(ctx, w, M, a);
    case EPI_QKV: return launch_f32_m<EPI_QKV>(ctx, w, M, a);
    case EPI_GATEUP: return launch_f32_m<EPI_GATEUP>(ctx, w, M, a);
    case EPI_LOGITS: return launch_f32_m<EPI_LOGITS>(ctx, w, M, a);
    default: return shd_fail(ctx, SHD_ERR_ARG, "gemv: unknown epilogue");
  }
}

template <int M>
static int launch_ring_t(shd_ctx* ctx, const shd_weight* w, RingArgs a) {
  using C = RingCfg<M>;
  static unsigned attr_devices = 0;
  if (!(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(gemv_ring_kernel<M>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_devices |= 1u << (ctx->device & 31);
  }
  const long long U = (long long)w->nT * w->nKC;
  const int G = (int)std::min<long long>(U, ctx->num_sms);
  gemv_ring_kernel<M><<<G, kGemvThreads, C::SMEM, ctx->stream>>>(a);
  SHD_CHECK_LAUNCH(ctx, "gemv_ring_kernel");
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

// Split M into launches of 8, 4, 2, 1 rows.
static int next_m(int rem) { return rem >= 8 ? 8 : rem >= 4 ? 4 : rem >= 2 ? 2 : 1; }

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
    const int mm = next_m(M - m0);
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
