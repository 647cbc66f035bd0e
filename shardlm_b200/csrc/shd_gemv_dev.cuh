// Device building blocks of the dual-share GEMV kernels (shd_gemv.cu): stream-K bookkeeping, the
// consumer-group barrier, the split-tile fixup, the f32 epilogues, the fused RMSNorm prologue and
// the per-block multiply-accumulate. Activations written by other CTAs of the same grid are read
// with L2-coherent loads (__ldcg), so no CTA sees a stale L1 line.
#pragma once

#include <algorithm>

#include "shd_gemv.cuh"

namespace shd {

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

// push_epoch: the exchange call this launch pushes (read by the kernel before it released its
// dependents, see gemv_f32_kernel).
template <int M, int EPI>
__device__ void epilogue_f32(const GemvArgs& a, int t, const float* tsum, int ctid, int* err,
                             unsigned push_epoch = 0) {
  if constexpr (EPI == EPI_STORE) {
    if (a.tp_peer[0]) {
      // push the tile to every rank: consecutive threads take consecutive rows of one (peer, share,
      // row m), so each warp writes 256 contiguous bytes of one peer's slot.
      const unsigned epoch = push_epoch;
      const unsigned long long tag = (unsigned long long)epoch << 32;
      const int W = a.tp_world;
      for (int idx = ctid; idx < kTileRows * M * 2 * W; idx += kConsumerWarps * 32) {
        const int r = idx % kTileRows;
        const int m = (idx / kTileRows) % M;
        const int sh = (idx / (kTileRows * M)) & 1;
        const int q = idx / (kTileRows * M * 2);
        const int n = t * kTileRows + r;
        if (n >= a.N) continue;
        float y = tsum[(r * 2 + sh) * M + m];
        if (sh == 1 && a.bias) y = __fadd_rn(y, a.bias[n]);
        if (a.Rc) y = __fadd_rn(y, __ldcg((sh ? a.Rs : a.Rc) + (size_t)m * a.ldr + n));
        unsigned long long* dst = p2p_slot(a.tp_peer[q], (int)(epoch & 1u), W, a.tp_me) +
                                  ((size_t)sh * M + m) * a.ldy + n;
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(tag | __float_as_uint(y)) : "memory");
      }
      return;
    }
    for (int idx = ctid; idx < kTileRows * M; idx += kConsumerWarps * 32) {
      const int r = idx % kTileRows, m = idx / kTileRows;
      const int n = t * kTileRows + r;
      if (n >= a.N) continue;
      float yc = tsum[(r * 2 + 0) * M + m];
      float ys = tsum[(r * 2 + 1) * M + m];
      if (a.bias) ys = __fadd_rn(ys, a.bias[n]);
      if (a.Rc) {
        yc = __fadd_rn(yc, __ldcg(a.Rc + (size_t)m * a.ldr + n));
        ys = __fadd_rn(ys, __ldcg(a.Rs + (size_t)m * a.ldr + n));
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

__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ int ld_relaxed_s32(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Partial-tile exchange of stream-K, finished by the tile's owner: the CTA holding the tile's first
// K chunks. Ranges are contiguous in (tile, chunk) order, so the owner reaches its part of the tile
// at the END of its range while every other contributor (later CTAs) has its part at the START of
// its range. Contributors store their partial (one slot per CTA: a CTA contributes to at most one
// tile it does not own, its first) and publish it with a release increment of the tile's counter,
// without waiting. The owner waits (bounded) until all of them have published, resets the counter,
// and sums the partials in CTA order (its own first), so results do not depend on timing.
// Returns 1 when this CTA must run the tile's epilogue, 0 when the owner will, -1 on a timeout.
template <typename T>
__device__ int split_tile_close(const PipeSmem& sm, uint32_t& cphase, T* tsum, T* partials,
                                int* counters, int tsum_len, long long U, int G, int g, int t,
                                int nKC, long long u0, long long u1, int ctid, int lane,
                                const volatile unsigned long long* abort_flag = nullptr) {
  const long long tb = (long long)t * nKC, te = tb + nKC;
  if (tb < u0) {  // a later contributor: publish and move on
    T* part = partials + (size_t)g * tsum_len;
    for (int k = ctid; k < tsum_len; k += kConsumerWarps * 32) part[k] = tsum[k];
    if (!consumer_sync(sm, cphase, lane)) return -1;
    // the release increment orders every thread's partial store before the count: the stores are
    // ordered before it by the barrier (release/acquire at CTA scope) and release is cumulative
    if (ctid == 0) red_release_add(&counters[t], 1);
    return 0;
  }
  (void)u1;
  const int gl = unit_owner(U, G, te - 1);
  const int need = gl - g;
  if (ctid == 0) {
    bool ok = true;
    if (ld_relaxed_s32(&counters[t]) < need) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_relaxed_s32(&counters[t]) < need) {
        if ((abort_flag && *abort_flag) || globaltimer_ns() - t0 > SHD_WAIT_LIMIT_NS) {
          ok = false;
          break;
        }
      }
    }
    if (ok) {
      fence_acq_rel_gpu();  // acquire side of the contributors' releases
      counters[t] = 0;
    }
    sm.flags[1] = ok ? 1 : 0;
  }
  if (!consumer_sync(sm, cphase, lane)) return -1;
  if (!sm.flags[1]) return -1;
  if (need > 0) {
    // loads of a batch of contributors are all in flight before the in-order sum consumes them
    constexpr int B = 8;
    for (int k = ctid; k < tsum_len; k += kConsumerWarps * 32) {
      T sum = tsum[k];
      for (int g0 = g + 1; g0 <= gl; g0 += B) {
        T v[B];
#pragma unroll
        for (int j = 0; j < B; ++j) v[j] = (g0 + j <= gl) ? __ldcg(partials + (size_t)(g0 + j) * tsum_len + k) : T(0);
#pragma unroll
        for (int j = 0; j < B; ++j)
          if (g0 + j <= gl) sum = sum + v[j];
      }
      tsum[k] = sum;
    }
    if (!consumer_sync(sm, cphase, lane)) return -1;
  }
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

// The norm's gamma for this thread's first kNormGroups float4 groups, loaded before the wait on
// the previous kernel: gamma is a weight (written by copies, never by a kernel of the step), so
// its round trip overlaps the previous kernel instead of following the sum of squares.
struct NormGamma {
  float4 g[kNormGroups];
};

__device__ __forceinline__ void norm_gamma_preload(const GemvArgs& a, int ctid, NormGamma& ng) {
  constexpr int STEP = kConsumerWarps * 32;
  const int K4 = a.K >> 2;
  const bool g_vec = (reinterpret_cast<uintptr_t>(a.gamma) & 15) == 0;
#pragma unroll
  for (int j = 0; j < kNormGroups; ++j) {
    const int i = ctid + j * STEP;
    ng.g[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < K4)
      ng.g[j] = g_vec ? __ldg(reinterpret_cast<const float4*>(a.gamma) + i)
                      : make_float4(a.gamma[4 * i], a.gamma[4 * i + 1], a.gamma[4 * i + 2], a.gamma[4 * i + 3]);
  }
}

template <int M>
__device__ bool norm_prologue(const GemvArgs& a, const PipeSmem& sm, uint32_t& cphase, float* xres,
                              int KP, int ctid, int lane, int warp, bool write_h,
                              const NormGamma* pre = nullptr) {
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
        c[j] = (i < K4) ? __ldcg(hc + i) : z4;
        s[j] = (i < K4) ? __ldcg(hs + i) : z4;
      }
      if (dc) {
        float4 e[NJ], f[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int i = b + ctid + j * STEP;
          e[j] = (i < K4) ? __ldcg(dc + i) : z4;
          f[j] = (i < K4) ? __ldcg(ds + i) : z4;
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
          if (pre && b == 0)
            gv[j] = pre->g[j];
          else
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

// Multiply-accumulate one 16 KB weight block (32 rows x 256 columns, bf16) into this warp's
// accumulators for both shares of M rows. Warp w owns tile rows 4w..4w+3; lane l owns columns
// {4l..4l+3, 128+4l..128+4l+3}. x rows are at xbase + (m * 2 + share) * xstride; okA/okB mask the
// two column groups at a ragged K tail. Packed f32x2 accumulators (acc2) serve M <= 4.
template <int M, int V, int VP>
__device__ __forceinline__ void mac_block(const uint4* wv, const float* xbase, int xstride, bool okA,
                                          bool okB, int warp, int lane,
                                          unsigned long long (&acc2)[(M <= 4) ? V : 1],
                                          float (&acc)[VP]) {
  constexpr bool USE2 = (M <= 4);
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
}

// End of this CTA's contribution to a tile: fold the packed accumulators, reduce over the warp
// and write the warp's rows into tsum[(row * 2 + share) * M + m]; accumulators restart at zero.
template <int M, int V, int VP>
__device__ __forceinline__ void tile_reduce(unsigned long long (&acc2)[(M <= 4) ? V : 1], float (&acc)[VP],
                                            float* tsum, int warp, int lane) {
  constexpr bool USE2 = (M <= 4);
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
}

}  // namespace shd
