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

namespace shd {

constexpr int kSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100
// Measured on B200: a pure cp.async.bulk stream sustains ~6.8 TB/s with 4 x 16 KB stages per CTA
// but only ~6.2 TB/s with 12; two or three CTAs per SM with 4-6 stages each reach ~7.1 TB/s.
constexpr int kMaxStages = 6;
constexpr int kSmemPerCta2 = 115712;  // dynamic shared memory per CTA at two CTAs per SM
constexpr int kTailBytes = 4608;    // tile result, barriers, flags, reduction scratch

// Stream-K bookkeeping: CTA g owns units [b_g, b_{g+1}), b_g = floor(U g / G).
__device__ __forceinline__ long long unit_begin(long long U, int G, int g) { return U * g / G; }
__device__ __forceinline__ int unit_owner(long long U, int G, long long u) {
  return (int)(((u + 1) * (long long)G - 1) / U);
}

// Reduce V (a power of two) per-lane values over the warp with a reduce-scatter butterfly.
// Afterwards this lane holds `cnt` fully reduced values with flat indices [base, base+cnt); lanes
// with any bit of `dup` set hold duplicates and must not write.
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
  int stage_bytes;
  int S;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* cbar;       // consumer-group barrier (8 warp arrivals)
  volatile int* flags;  // [0] abort, [1] last-arriver flag
  float* red;           // 16 floats of block-reduction scratch
};

// Consumer-group barrier over the 8 consumer warps, bounded.
__device__ __forceinline__ bool consumer_sync(const PipeSmem& sm, uint32_t& phase, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.cbar);
  const bool ok = warp_wait(sm.cbar, phase);
  phase ^= 1u;
  return ok;
}

// Producer: one elected lane streams the weight block (and, unless the activations are resident,
// the x chunks) of every unit. Weights for the first S units are requested before waiting on the
// previous kernel (they do not depend on it); activation copies only after.
template <int M, int CHUNK, typename XT>
__device__ void gemv_producer(const PipeSmem& sm, const uint8_t* W, const XT* Xc, const XT* Xs,
                              int ldx, int K, int nKC, long long u0, long long u1, bool staged_x,
                              int* err) {
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
  for (int i = 0; i < npre; ++i) {
    const long long u = u0 + i;
    const uint32_t tx = (uint32_t)kBlockBytes + (staged_x ? (uint32_t)(M * 2) * xbytes_of(u) : 0u);
    mbar_arrive_expect_tx(&sm.full[i], tx);
    bulk_g2s(sm.stages + (size_t)i * sm.stage_bytes, W + (size_t)u * kBlockBytes, kBlockBytes, &sm.full[i], pol_w);
  }
  if (staged_x) {
    pdl_wait();
    for (int i = 0; i < npre; ++i) issue_x(i, u0 + i);
  }
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

// Partial-tile exchange of stream-K. All consumer threads store this CTA's tile partial; one thread
// publishes it with a release fence + counter increment; the last contributor reads every
// contributor's partial (acquire) and sums them in CTA order into tsum. Returns 1 if this CTA must
// run the epilogue, 0 if another CTA will, -1 on a barrier timeout.
template <typename T>
__device__ int split_tile_fixup(const PipeSmem& sm, uint32_t& cphase, T* tsum, T* partials,
                                int* counters, int tsum_len, long long U, int G, int g, int t,
                                int nKC, int first_tile, int ctid, int lane) {
  const int slot = (t == first_tile) ? 0 : 1;
  T* part = partials + ((size_t)g * 2 + slot) * tsum_len;
  for (int k = ctid; k < tsum_len; k += kConsumerWarps * 32) part[k] = tsum[k];
  if (!consumer_sync(sm, cphase, lane)) return -1;
  const int gf = unit_owner(U, G, (long long)t * nKC);
  const int gl = unit_owner(U, G, (long long)(t + 1) * nKC - 1);
  if (ctid == 0) {
    __threadfence();  // release: the CTA's partial (ordered before by the barrier) before the count
    const int old = atomicAdd(&counters[t], 1);
    const int last = (old == gl - gf);
    if (last) {
      counters[t] = 0;
      __threadfence();  // acquire side of the other contributors' releases
    }
    sm.flags[1] = last;
  }
  if (!consumer_sync(sm, cphase, lane)) return -1;
  if (!sm.flags[1]) return 0;
  for (int k = ctid; k < tsum_len; k += kConsumerWarps * 32) {
    T sum = T(0);
    for (int gg = gf; gg <= gl; ++gg) {
      const int ft = (int)(unit_begin(U, G, gg) / nKC);
      const int sl = (t == ft) ? 0 : 1;
      const T v = __ldcg(partials + ((size_t)gg * 2 + sl) * tsum_len + k);
      sum = (gg == gf) ? v : sum + v;
    }
    tsum[k] = sum;
  }
  if (!consumer_sync(sm, cphase, lane)) return -1;
  return 1;
}

// ---- packed f32x2 helpers ----
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float sum2(unsigned long long v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
__device__ __forceinline__ void fma2(unsigned long long& acc, unsigned long long w, unsigned long long x) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(w), "l"(x));
}
__device__ __forceinline__ unsigned long long bf16pair(uint32_t q) {
  return pack2(__uint_as_float(q << 16), __uint_as_float(q & 0xffff0000u));
}

// RMSNorm prologue: x = reshare(RMSNorm(D + H)) for M rows into xres[m][share][KP] (zero padded).
// Every CTA computes the identical values (same thread mapping, fixed reduction order). Each thread
// owns float4 groups i = ctid + 256 j; the loads of a block of kNormGroups groups (and of gamma and
// the mask) are all issued before any is used, so a CTA waits on L2 about twice per row instead of
// once per group.
constexpr int kNormGroups = 4;

template <int M>
__device__ bool norm_prologue(const GemvArgs& a, const PipeSmem& sm, uint32_t& cphase, float* xres,
                              int KP, int ctid, int lane, int warp, bool write_h) {
  constexpr int NJ = kNormGroups;
  constexpr int STEP = kConsumerWarps * 32;
  const int K = a.K;
  const int K4 = K >> 2, KP4 = KP >> 2;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool g_vec = (reinterpret_cast<uintptr_t>(a.gamma) & 15) == 0;
  for (int m = 0; m < M; ++m) {
    const float4* hc = reinterpret_cast<const float4*>(a.nHc + (size_t)m * a.n_ldh);
    const float4* hs = reinterpret_cast<const float4*>(a.nHs + (size_t)m * a.n_ldh);
    const float4* dc = a.nDc ? reinterpret_cast<const float4*>(a.nDc + (size_t)m * a.n_ldh) : nullptr;
    const float4* ds = a.nDs ? reinterpret_cast<const float4*>(a.nDs + (size_t)m * a.n_ldh) : nullptr;
    float4* oc = (write_h && a.nHout_c) ? reinterpret_cast<float4*>(a.nHout_c + (size_t)m * a.n_ldh) : nullptr;
    float4* os = (write_h && a.nHout_s) ? reinterpret_cast<float4*>(a.nHout_s + (size_t)m * a.n_ldh) : nullptr;
    float* xr = xres + (size_t)(m * 2) * KP;
    float4* xr4 = reinterpret_cast<float4*>(xr);
    float ss = 0.0f;
    for (int b = 0; b < K4; b += NJ * STEP) {
      float4 c[NJ], s[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = b + ctid + j * STEP;
        c[j] = (i < K4) ? hc[i] : z4;
        s[j] = (i < K4) ? hs[i] : z4;
      }
      if (dc) {
        float4 e[NJ], f[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int i = b + ctid + j * STEP;
          e[j] = (i < K4) ? dc[i] : z4;
          f[j] = (i < K4) ? ds[i] : z4;
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int i = b + ctid + j * STEP;
          c[j] = make_float4(__fadd_rn(e[j].x, c[j].x), __fadd_rn(e[j].y, c[j].y), __fadd_rn(e[j].z, c[j].z),
                             __fadd_rn(e[j].w, c[j].w));
          s[j] = make_float4(__fadd_rn(f[j].x, s[j].x), __fadd_rn(f[j].y, s[j].y), __fadd_rn(f[j].z, s[j].z),
                             __fadd_rn(f[j].w, s[j].w));
          if (oc && i < K4) {
            oc[i] = c[j];
            os[i] = s[j];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = b + ctid + j * STEP;
        if (i < K4) {
          const float4 x = make_float4(__fadd_rn(c[j].x, s[j].x), __fadd_rn(c[j].y, s[j].y),
                                       __fadd_rn(c[j].z, s[j].z), __fadd_rn(c[j].w, s[j].w));
          xr4[i] = x;
          ss = __fmaf_rn(x.x, x.x, ss);
          ss = __fmaf_rn(x.y, x.y, ss);
          ss = __fmaf_rn(x.z, x.z, ss);
          ss = __fmaf_rn(x.w, x.w, ss);
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) sm.red[warp] = ss;
    if (!consumer_sync(sm, cphase, lane)) return false;
    float sum_sq = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) sum_sq = __fadd_rn(sum_sq, sm.red[w]);
    const float mean_sq = __fdiv_rn(sum_sq, (float)K);
    float inv;
    if (a.nvariant == SHD_NL_GPU) {
      inv = rsqrtf(__fadd_rn(mean_sq, a.eps));
    } else {
      const float rms = __fsqrt_rn(__fadd_rn(mean_sq, a.eps));
      if (a.nvariant == SHD_NL_MPC)
        inv = (rms > 1e-6f && isfinite(rms)) ? __fdiv_rn(1.0f, rms) : 1.0f;
      else
        inv = __fdiv_rn(1.0f, rms);
    }
    const float* mk = a.nmask ? a.nmask + (size_t)m * a.n_ldmask : nullptr;
    const bool m_vec = (reinterpret_cast<uintptr_t>(mk) & 15) == 0;
    for (int b = 0; b < KP4; b += NJ * STEP) {
      float4 gv[NJ], mv[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = b + ctid + j * STEP;
        gv[j] = z4;
        mv[j] = z4;
        if (i < K4) {
          gv[j] = g_vec ? reinterpret_cast<const float4*>(a.gamma)[i]
                        : make_float4(a.gamma[4 * i], a.gamma[4 * i + 1], a.gamma[4 * i + 2], a.gamma[4 * i + 3]);
          if (mk)
            mv[j] = m_vec ? reinterpret_cast<const float4*>(mk)[i]
                          : make_float4(mk[4 * i], mk[4 * i + 1], mk[4 * i + 2], mk[4 * i + 3]);
        }
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = b + ctid + j * STEP;
        if (i >= KP4) continue;
        float4 xc = z4, xs = z4;
        if (i < K4) {
          const float4 x = xr4[i];
          float r0 = __fmul_rn(__fmul_rn(x.x, inv), gv[j].x);
          float r1 = __fmul_rn(__fmul_rn(x.y, inv), gv[j].y);
          float r2 = __fmul_rn(__fmul_rn(x.z, inv), gv[j].z);
          float r3 = __fmul_rn(__fmul_rn(x.w, inv), gv[j].w);
          if (a.nvariant == SHD_NL_MPC) {
            if (!isfinite(r0)) r0 = 0.0f;
            if (!isfinite(r1)) r1 = 0.0f;
            if (!isfinite(r2)) r2 = 0.0f;
            if (!isfinite(r3)) r3 = 0.0f;
          }
          xc = make_float4(__fsub_rn(r0, mv[j].x), __fsub_rn(r1, mv[j].y), __fsub_rn(r2, mv[j].z),
                           __fsub_rn(r3, mv[j].w));
          xs = mv[j];
        }
        xr4[i] = xc;
        reinterpret_cast<float4*>(xr + KP)[i] = xs;
      }
    }
    if (!consumer_sync(sm, cphase, lane)) return false;  // red reuse and xres visibility
  }
  return true;
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
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == kConsumerWarps) {
    if (lane == 0)
      gemv_producer<M, kChunkBf16, float>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC, u0, u1, !NORM, a.err);
    return;
  }

  const int ctid = threadIdx.x;  // 0..255 among consumers
  uint32_t cphase = 0;
  pdl_wait();  // activations, positions and scratch come from earlier kernels
  if constexpr (NORM) {
    if (!norm_prologue<M>(a, sm, cphase, xres, KP, ctid, lane, warp, g == 0)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
  }

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
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (USE2) {
      unsigned long long w2[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint4 q = wv[(warp * 4 + r) * 32 + lane];
        w2[r][0] = bf16pair(q.x);
        w2[r][1] = bf16pair(q.y);
        w2[r][2] = bf16pair(q.z);
        w2[r][3] = bf16pair(q.w);
      }
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int sh = 0; sh < 2; ++sh) {
          const float* xp = xbase + (size_t)(m * 2 + sh) * xstride;
          const float4 xa = okA ? *reinterpret_cast<const float4*>(xp + 4 * lane) : z4;
          const float4 xb = okB ? *reinterpret_cast<const float4*>(xp + 128 + 4 * lane) : z4;
          const unsigned long long x0 = pack2(xa.x, xa.y), x1 = pack2(xa.z, xa.w);
          const unsigned long long x2 = pack2(xb.x, xb.y), x3 = pack2(xb.z, xb.w);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            unsigned long long& A = acc2[(r * 2 + sh) * M + m];
            fma2(A, w2[r][0], x0);
            fma2(A, w2[r][1], x1);
            fma2(A, w2[r][2], x2);
            fma2(A, w2[r][3], x3);
          }
        }
    } else {
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
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int sh = 0; sh < 2; ++sh) {
          const float* xp = xbase + (size_t)(m * 2 + sh) * xstride;
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

    // ---- this CTA's contribution to tile ct is complete ----
    if constexpr (USE2) {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        acc[j] = sum2(acc2[j]);
        acc2[j] = 0ull;
      }
    }
    int base, cnt;
    unsigned dup;
    warp_reduce_scatter<float, VP>(acc, lane, base, cnt, dup);
    if ((lane & dup) == 0) {
#pragma unroll
      for (int j = 0; j < VP; ++j)
        if (j < cnt && base + j < V) tsum[warp * V + base + j] = acc[j];
    }
#pragma unroll
    for (int j = 0; j < VP; ++j) acc[j] = 0.f;

    const bool full_tile = ((long long)ct * a.nKC >= u0) && (cc == a.nKC - 1);
    if (!consumer_sync(sm, cphase, lane)) {
      if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
      sm.flags[0] = 1;
      return;
    }
    if (!full_tile) {
      const int r = split_tile_fixup<float>(sm, cphase, tsum, a.partials, a.counters, TSUM, U, G, g, ct,
                                            a.nKC, first_tile, ctid, lane);
      if (r < 0) {
        if (lane == 0) atomicOr(a.err, SHD_DEVERR_TIMEOUT_FULL);
        sm.flags[0] = 1;
        return;
      }
      if (r == 0) continue;
    }
    epilogue_f32<M, EPI>(a, ct, tsum, ctid, a.err);
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
    if (lane == 0) gemv_producer<M, kChunkI32, int32_t>(sm, a.W, a.Xc, a.Xs, a.ldx, a.K, a.nKC, u0, u1, true, a.err);
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
      const int r = split_tile_fixup<long long>(sm, cphase, tsum, a.partials, a.counters, TSUM, U, G, g, ct,
                                                a.nKC, first_tile, ctid, lane);
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

// Two CTAs per SM (one streams while the other is in its prologue, split-tile exchange or
// epilogue) when at least 4 stages fit in half the shared memory and M <= 2 keeps the registers
// under the two-CTA limit; otherwise one CTA per SM.
template <int M, int EPI, bool NORM>
static int launch_f32_t(shd_ctx* ctx, const shd_weight* w, GemvArgs a) {
  static unsigned attr1 = 0, attr2 = 0;
  const int stage = kBlockBytes + (NORM ? 0 : M * 2 * kChunkBf16 * 4);
  const size_t xres = NORM ? (size_t)M * 2 * w->nKC * kChunkBf16 * 4 : 0;
  const long long U = (long long)w->nT * w->nKC;
  const long long s2 = ((long long)kSmemPerCta2 - kTailBytes - (long long)xres) / stage;
  if constexpr (M <= 2) {
    if (s2 >= 4) {
      const int rc = set_smem_attr(ctx, gemv_f32_kernel<M, EPI, NORM, 2>, attr2);
      if (rc) return rc;
      a.nstages = (int)std::min<long long>(kMaxStages, s2);
      const size_t smem = (size_t)a.nstages * stage + xres + kTailBytes;
      const int G = (int)std::min<long long>(U, 2LL * ctx->num_sms);
      SHD_CHECK_CUDA(ctx, launch_pdl(gemv_f32_kernel<M, EPI, NORM, 2>, dim3(G), dim3(kGemvThreads), smem, ctx->stream, a));
      ctx->launches++;
      return SHD_OK;
    }
  }
  (void)attr2;
  const int rc = set_smem_attr(ctx, gemv_f32_kernel<M, EPI, NORM, 1>, attr1);
  if (rc) return rc;
  const long long avail = (long long)kSmemLimit - kTailBytes - (long long)xres;
  a.nstages = (int)std::min<long long>(kMaxStages, avail / stage);
  if (a.nstages < 2) return shd_fail(ctx, SHD_ERR_ARG, "gemv: activation vector too long for the fused norm");
  const size_t smem = (size_t)a.nstages * stage + xres + kTailBytes;
  const int G = (int)std::min<long long>(U, ctx->num_sms);
  SHD_CHECK_CUDA(ctx, launch_pdl(gemv_f32_kernel<M, EPI, NORM, 1>, dim3(G), dim3(kGemvThreads), smem, ctx->stream, a));
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

int launch_gemv_f32(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs a, bool norm) {
  a.W = reinterpret_cast<const uint8_t*>(w->d_tiles);
  a.N = w->N;
  a.K = (w->K + 3) / 4 * 4;  // x extent copied per row (rows padded to 16 bytes)
  a.nT = w->nT;
  a.nKC = w->nKC;
  a.partials = ctx->d_partials;
  a.counters = ctx->d_counters;
  a.err = ctx->d_err;
  if (w->nT > ctx->n_counters - 8192) return shd_fail(ctx, SHD_ERR_ARG, "gemv: too many row tiles");
  if (norm) {
    if (w->K % 4 != 0) return shd_fail(ctx, SHD_ERR_ARG, "gemv: fused norm needs in_features % 4 == 0");
    a.K = w->K;
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
  if (w->nT > ctx->n_counters - 8192) return shd_fail(ctx, SHD_ERR_ARG, "gemv: too many row tiles");
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
