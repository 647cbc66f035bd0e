// Tensor-core dual-share linear for many rows (prefill chunks, batched decode): tcgen05 on sm_100a.
//
// The shares are f32 and the weights exact bf16 (the reference's f32 weights are bf16 upcasts,
// crates/v2/server/src/secure_weights.rs:432-440). Every f32 share value splits exactly into three
// bf16 terms, x = x0 + x1 + x2 (x0 = bf16(x), x1 = bf16(x - x0), x2 = x - x0 - x1: 8 + 8 + 8
// significand bits, the exponent range of bf16 is that of f32), and a bf16 x bf16 product is exact in
// f32. So Y = X W^T is computed as sum_i X_i W^T on the bf16 tensor cores with f32 accumulation in
// tensor memory: the only rounding is that of the f32 accumulation, as in an f32 GEMM.
//
// Kernel (one CTA per SM, persistent over output tiles of 128 weight rows x NT token rows):
//  * warp 4 (one lane) loads per 64-wide K block the weight tile with one 4-D TMA copy straight out
//    of the 16 KB tiled weight blocks (128 rows = 4 consecutive 32-row tiles, 64 of the 256 columns
//    of one chunk, 128-byte swizzle) and the six activation planes (client/server x three bf16
//    terms) with one 3-D TMA copy, into an S-stage mbarrier ring;
//  * warp 5 allocates tensor memory (two accumulator buffers, each [client | server] x NT f32
//    columns) and one lane issues tcgen05.mma (M = 128, N = NT, K = 16, bf16 x bf16 -> f32): per
//    16-wide K step, three MMAs per share accumulate the three terms; tcgen05.commit frees the ring
//    stage and, after the last K block, hands the accumulator to the epilogue;
//  * warps 0-3 (tensor memory lanes 0-127 = the tile's 128 weight rows) read the accumulators with
//    tcgen05.ld and apply the epilogue of the layer (store + bias + residual, q/k/v with RoPE and the
//    KV-cache write, gate/up with SwiGLU and reshare), one thread per weight row.
//
// The weight blocks keep the GEMV layout, whose 256 columns of a chunk are stored permuted (lane l
// of a row holds columns 4l..4l+3 and 128+4l..128+4l+3); the split kernel writes the activation
// planes in the same permuted column order, so the MMA's K sum pairs the right terms.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "shd_gemv_dev.cuh"
#include "shd_tc.cuh"
#include "shd_tcgen05.cuh"

namespace shd {
namespace {

constexpr int kTcBM = 128;          // weight rows per tile
constexpr int kTcBK = 64;           // K per ring stage (one 128-byte swizzle row of bf16)
constexpr int kTcThreads = 192;     // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int kTcSmemLimit = 232448 - 1024;
constexpr int kTcABytes = kTcBM * kTcBK * 2;  // 16 KB

// Instruction descriptor of this kernel's MMAs: M = 128 weight rows, N = nt.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int nt) { return idesc_bf16_f32_mn(kTcBM, nt); }

// ---------------------------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------------------------
struct TcArgs {
  GemvArgs g;    // epilogue parameters (as for the GEMV epilogues) and N, K, nT, nKC, err
  int epi;
  int M;         // token rows
  int n_tok;     // token tiles (ceil(M / NT))
  int n_row;     // weight row tiles of 128 (ceil(nT / 4))
  int n_kb;      // K blocks of 64
  int ksplit;    // K ranges per output tile (> 1: partial sums to `ws`, epilogue in tc_reduce_kernel)
  int nstages;
  float* ws;     // [ksplit][n_tok * NT][n_row * 128][2] partial sums (ksplit > 1)
  PlaneOut out;  // EPI_GATEUP in the reduce kernel: the output as the next linear's planes
};

// Token tiles of up to 32 rows keep the three terms of a share side by side in tensor memory (one
// MMA with N = 3 NT per share, terms summed in order by the epilogue). From 64 rows the terms
// accumulate into one accumulator per share (three MMAs with N = NT): the weight tile is reused by
// twice or four times the tokens per shared-memory fill, which is what limits this kernel at prompt
// sizes (the operands stream from L2 at about 90 GB/s per SM); the sum then runs over 3 K products
// per output instead of K, and its f32 rounding bound is that of 3 K terms.
template <int NT>
struct TcSmem {
  static constexpr bool kFused = NT >= 64;
  static constexpr int kBBytes = 6 * NT * kTcBK * 2;
  static constexpr int kStage = kTcABytes + kBBytes;
  static constexpr int kN = kFused ? NT : 3 * NT;  // MMA N per share
  static constexpr int kBuf = 2 * kN;              // tensor-memory columns per accumulator buffer
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  if (mbar_wait_bounded(bar, parity)) return true;
  atomicOr(err, SHD_DEVERR_TIMEOUT_FULL);
  *abort_flag = 1;
  return false;
}

// The epilogue of one value: weight row n (tile order; 32 consecutive rows per warp, lane = n % 32),
// token row m. Every lane of the warp calls it together (RoPE and SwiGLU pair rows across lanes).
__device__ __forceinline__ void tc_epi_value(const TcArgs& ta, int n, int m, bool live, float yc, float ys,
                                             int lane) {
  const GemvArgs& a = ta.g;
  if (ta.epi == EPI_STORE) {
    if (live && n < a.N) {
      if (a.bias) ys = __fadd_rn(ys, a.bias[n]);
      if (a.Rc) {
        yc = __fadd_rn(yc, __ldcg(a.Rc + (size_t)m * a.ldr + n));
        ys = __fadd_rn(ys, __ldcg(a.Rs + (size_t)m * a.ldr + n));
      }
      a.Yc[(size_t)m * a.ldy + n] = yc;
      a.Ys[(size_t)m * a.ldy + n] = ys;
    }
  } else if (ta.epi == EPI_QKV) {
    // rows 2p, 2p+1 of the tile order are a RoPE pair: exchange with the neighbour lane
    if (a.bias && n < a.N) ys = __fadd_rn(ys, a.bias[n]);
    const float oc = __shfl_xor_sync(0xffffffffu, yc, 1);
    const float os = __shfl_xor_sync(0xffffffffu, ys, 1);
    if (!live || n >= a.N) return;
    const int np = n & ~1;  // first row of the pair
    const bool second = (n & 1) != 0;
    const float x0c = second ? oc : yc, x1c = second ? yc : oc;
    const float x0s = second ? os : ys, x1s = second ? ys : os;
    const int hd = a.head_dim, half = hd >> 1;
    const int head = np / hd;
    const int p = (np % hd) >> 1;
    const int n0 = head * hd + p, n1 = n0 + half;
    const int pos = a.pos ? a.pos[m] : 0;
    float oc_, os_;
    if (n0 < a.q_dim + a.kv_dim) {
      if (pos < 0 || pos >= a.rope_max_seq) {
        atomicOr(a.err, SHD_DEVERR_ARG);
        return;
      }
      // RopeFrequencies::apply_to_share (secure_attention.rs:84-121), no fused multiply-add
      const float cs = a.rope_cos[(size_t)pos * half + p];
      const float sn = a.rope_sin[(size_t)pos * half + p];
      if (!second) {
        oc_ = __fsub_rn(__fmul_rn(x0c, cs), __fmul_rn(x1c, sn));
        os_ = __fsub_rn(__fmul_rn(x0s, cs), __fmul_rn(x1s, sn));
      } else {
        oc_ = __fadd_rn(__fmul_rn(x0c, sn), __fmul_rn(x1c, cs));
        os_ = __fadd_rn(__fmul_rn(x0s, sn), __fmul_rn(x1s, cs));
      }
    } else {
      oc_ = second ? x1c : x0c;
      os_ = second ? x1s : x0s;
    }
    const int nn = second ? n1 : n0;
    if (a.Yc) {
      a.Yc[(size_t)m * a.ldy + nn] = oc_;
      a.Ys[(size_t)m * a.ldy + nn] = os_;
    }
    const float v = __fadd_rn(oc_, os_);
    if (n0 < a.q_dim) {
      if (a.Q) a.Q[(size_t)m * a.ldq + nn] = v;
    } else {
      const bool isk = n0 < a.q_dim + a.kv_dim;
      float* cache = isk ? a.Kcache : a.Vcache;
      const int off = isk ? (nn - a.q_dim) : (nn - a.q_dim - a.kv_dim);
      if (cache) {
        const int sq = a.seq ? a.seq[m] : 0;
        cache[(size_t)sq * a.kv_seq_stride + (size_t)pos * a.kv_dim + off] = v;
      }
    }
  } else if (ta.epi == EPI_LOGITS) {
    // logit shares (optional) and the greedy key of the reconstructed logit; the 32 lanes are 32
    // vocabulary rows of one token row, reduced in the warp before one atomic max (as the GEMV)
    unsigned long long key = 0ull;
    bool nan = false;
    if (live && n < a.N) {
      if (a.Yc) {
        a.Yc[(size_t)m * a.ldy + n] = yc;
        a.Ys[(size_t)m * a.ldy + n] = ys;
      }
      const float l = __fadd_rn(yc, ys);
      nan = isnan(l);
      key = argmax_key(l, n + a.idx_offset);
    }
    if (__any_sync(0xffffffffu, nan) && lane == 0) atomicOr(a.err, SHD_DEVERR_NONFINITE);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    if (lane == 0 && key != 0ull) atomicMax(&a.amax[m], key);
  } else {  // EPI_GATEUP: lanes 0-15 gate rows, 16-31 the matching up rows of the 32-row tile
    const float uc = __shfl_xor_sync(0xffffffffu, yc, 16);
    const float us = __shfl_xor_sync(0xffffffffu, ys, 16);
    if (!live || lane >= 16) return;
    const int I = a.N >> 1;
    const int i = (n >> 5) * 16 + lane;
    if (i >= I) return;
    const float gv = __fadd_rn(yc, ys);
    const float uv = __fadd_rn(uc, us);
    const float y = swiglu_variant(gv, uv, a.variant);
    const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + i] : 0.0f;
    if (ta.out.p) {
      planes_store(ta.out, m, i, __fsub_rn(y, mk), mk);
    } else {
      a.Yc[(size_t)m * a.ldy + i] = __fsub_rn(y, mk);
      a.Ys[(size_t)m * a.ldy + i] = mk;
    }
  }
}

// Epilogue of one accumulator buffer (columns: share, term, token; or share, token when the terms
// accumulate together): this thread owns weight row r = 32 warp + lane of the tile. Side-by-side
// terms of a share are summed in order.
template <int NT>
__device__ void tc_epilogue(const TcArgs& ta, uint32_t tacc, int row0, int tok0, int ks, int warp, int lane) {
  using L = TcSmem<NT>;
  constexpr int Q = L::kFused ? 2 : 6;
  const int r = warp * 32 + lane;
  const int n = row0 + r;  // row in tile order
  const uint32_t tl = tacc + ((uint32_t)(warp * 32) << 16);
  const int ntok = min(NT, ta.M - tok0);
  const int rows_all = ta.n_row * kTcBM;
  for (int c0 = 0; c0 < NT; c0 += 8) {
    float t[Q][8];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const uint32_t col = L::kFused ? (uint32_t)(q * L::kN + c0) : (uint32_t)((q / 3) * L::kN + (q % 3) * NT + c0);
      tmem_ld8(tl + col, t[q]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < Q; ++q) tmem_loaded(t[q]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = tok0 + c0 + j;
      const bool live = (c0 + j < ntok);
      float yc, ys;
      if constexpr (L::kFused) {
        yc = t[0][j];
        ys = t[1][j];
      } else {
        yc = __fadd_rn(__fadd_rn(t[0][j], t[1][j]), t[2][j]);
        ys = __fadd_rn(__fadd_rn(t[Q / 2][j], t[Q / 2 + 1][j]), t[Q / 2 + 2][j]);
      }
      if (ta.ksplit > 1) {
        float* w = ta.ws + (((size_t)ks * ta.n_tok * NT + (size_t)(tok0 + c0 + j)) * rows_all + n) * 2;
        w[0] = yc;
        w[1] = ys;
      } else {
        tc_epi_value(ta, n, m, live, yc, ys, lane);
      }
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_linear_kernel(const __grid_constant__ TcArgs ta, const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_x) {
  using L = TcSmem<NT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = ta.nstages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * L::kStage);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;      // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;  // [2] epilogue -> MMA
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kCols = 512;  // two buffers of 2 x 3 NT columns (NT <= 32)
  static_assert(2 * L::kBuf <= (int)kCols, "accumulators exceed tensor memory");
  const int tiles = ta.n_row * ta.n_tok * ta.ksplit;
  const int kb_per = ta.n_kb / ta.ksplit;  // the launcher makes ksplit divide n_kb

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 5) tmem_alloc(tmem_base, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_base;
  pdl_wait();  // activation planes and epilogue inputs come from earlier kernels

  // work item t: weight row tile rt, token tile tt, K range ks (token tile fastest: CTAs that run
  // together share the weight tile through L2)
  if (warp == 4) {
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      long long n = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok && !*abort_flag; t += gridDim.x) {
        const int tt = t % ta.n_tok, ks = (t / ta.n_tok) % ta.ksplit, rt = t / (ta.n_tok * ta.ksplit);
        for (int kb = ks * kb_per; kb < (ks + 1) * kb_per; ++kb, ++n) {
          if (n >= S && !tc_wait(&empty[s], ph ^ 1u, ta.g.err, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (size_t)s * L::kStage;
          mbar_arrive_expect_tx(&full[s], (uint32_t)L::kStage);
          // weights: columns (kb % 4) * 64 of chunk kb / 4, rows of 32-row tiles 4 rt .. 4 rt + 3
          tma_load_4d(st, &map_w, (kb & 3) * kTcBK, 0, kb >> 2, rt * 4, &full[s], pol_w);
          // activation planes: K block kb, token rows tt * NT .., all six planes
          tma_load_3d(st + kTcABytes, &map_x, kb * kTcBK, tt * NT, 0, &full[s], pol_x);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(L::kN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t use = (uint32_t)(it >> 1);  // uses of this buffer so far
        if (use > 0 && !tc_wait(&acc_empty[buf], (use - 1) & 1u, ta.g.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t dacc = tbase + (uint32_t)(buf * L::kBuf);
        bool ok = true;
        for (int kb = 0; kb < kb_per; ++kb) {
          if (!tc_wait(&full[s], ph, ta.g.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + (size_t)s * L::kStage;
          const uint64_t ad = smem_desc_sw128(st);
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k) {
            if constexpr (L::kFused) {
              // three MMAs per share (one per term plane, N = NT) into the share's accumulator
#pragma unroll
              for (int sh = 0; sh < 2; ++sh)
#pragma unroll
                for (int t = 0; t < 3; ++t) {
                  const uint64_t bd = smem_desc_sw128(st + kTcABytes + (size_t)(sh * 3 + t) * NT * kTcBK * 2);
                  tc_mma(dacc + (uint32_t)(sh * L::kN), ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                         (kb > 0 || k > 0 || t > 0) ? 1u : 0u);
                }
            } else if constexpr (NT == 8) {
              // 3 NT = 24 is no valid N for M = 128: the six planes (48 consecutive rows) go through
              // ONE MMA with N = 48, whose columns sh * 3 NT + term * NT + token are the layout the
              // two per-share MMAs of wider tiles produce
              const uint64_t bd = smem_desc_sw128(st + kTcABytes);
              tc_mma(dacc, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc_bf16_f32(6 * NT),
                     (kb > 0 || k > 0) ? 1u : 0u);
            } else {
#pragma unroll
              for (int sh = 0; sh < 2; ++sh) {
                // the share's three term planes are 3 NT consecutive rows: one MMA with N = 3 NT
                const uint64_t bd = smem_desc_sw128(st + kTcABytes + (size_t)sh * 3 * NT * kTcBK * 2);
                tc_mma(dacc + (uint32_t)(sh * L::kN), ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
              }
            }
          }
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      // every MMA issued has completed before the accumulators are released
      tc_commit(done);
      if (!mbar_wait_bounded(done, 0)) atomicOr(ta.g.err, SHD_DEVERR_TIMEOUT_DRAIN);
    }
  } else {
    // epilogue warps 0-3: tensor memory lanes 32 w .. 32 w + 31
    int it = 0;
    for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      if (!warp_wait(&acc_full[buf], use & 1u)) {
        if (lane == 0) atomicOr(ta.g.err, SHD_DEVERR_TIMEOUT_FULL);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int tt = t % ta.n_tok, ks = (t / ta.n_tok) % ta.ksplit, rt = t / (ta.n_tok * ta.ksplit);
      tc_epilogue<NT>(ta, tbase + (uint32_t)(buf * L::kBuf), rt * kTcBM, tt * NT, ks, warp, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  // the producer's copies in flight must land before the CTA leaves
  if (warp == 4 && lane == 0 && *abort_flag) {
    for (int s = 0; s < S; ++s) mbar_wait_bounded(&full[s], 0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tbase, kCols);
}

// Split-K reduction: CTA (row tile, token tile) of 128 x 4 threads, threadIdx.x = weight row,
// threadIdx.y = a quarter of the token tile's rows. Partial sums are added in split order, with the
// partials of up to 4 splits x NT/4 rows (both shares in one 8-byte load) in flight at once, then
// the epilogue (its pair exchanges stay within a warp: 32 consecutive weight rows).
constexpr int kTcReduceY = 4;

template <int NT>
__global__ void __launch_bounds__(kTcBM * kTcReduceY) tc_reduce_kernel(const __grid_constant__ TcArgs ta) {
  constexpr int JT = NT / kTcReduceY;
  constexpr int KQ = JT >= 16 ? 1 : 16 / JT;  // splits loaded together: >= 16 partial pairs in flight
  pdl_wait();
  const int rt = blockIdx.x, tt = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int n = rt * kTcBM + threadIdx.x;
  const int rows_all = ta.n_row * kTcBM;
  const int m0 = tt * NT + threadIdx.y * JT;
  float yc[JT], ys[JT];
  for (int ks0 = 0; ks0 < ta.ksplit; ks0 += KQ) {
    float2 p[KQ][JT];
#pragma unroll
    for (int q = 0; q < KQ; ++q)
#pragma unroll
      for (int j = 0; j < JT; ++j) {
        p[q][j] = make_float2(0.f, 0.f);
        if (ks0 + q < ta.ksplit)
          p[q][j] = __ldcg(reinterpret_cast<const float2*>(
              ta.ws + (((size_t)(ks0 + q) * ta.n_tok * NT + (size_t)(m0 + j)) * rows_all + n) * 2));
      }
#pragma unroll
    for (int q = 0; q < KQ; ++q)
#pragma unroll
      for (int j = 0; j < JT; ++j) {
        const int ks = ks0 + q;
        if (ks == 0) {
          yc[j] = p[q][j].x;
          ys[j] = p[q][j].y;
        } else if (ks < ta.ksplit) {
          yc[j] = __fadd_rn(yc[j], p[q][j].x);
          ys[j] = __fadd_rn(ys[j], p[q][j].y);
        }
      }
  }
#pragma unroll
  for (int j = 0; j < JT; ++j) tc_epi_value(ta, n, m0 + j, m0 + j < ta.M, yc[j], ys[j], lane);
}

// Split f32 shares into the six bf16 planes [share * 3 + term][Mp][KP], columns permuted as in the
// weight blocks (physical j of chunk c <- logical column c*256 + 4 (j/8) + (j%8 < 4 ? j%8 : 124 + j%8)),
// zero beyond K and beyond M.
__global__ void split_planes_kernel(const float* __restrict__ xc, const float* __restrict__ xs, int ldx, int M,
                                    int K, int Mp, int KP, uint16_t* __restrict__ out) {
  pdl_wait();  // the shares come from the previous kernel
  const size_t plane = (size_t)Mp * KP;
  const long long total = (long long)Mp * KP;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(idx / KP), j = (int)(idx % KP);
    const int c = j >> 8, jj = j & 255;
    const int l = jj >> 3, i = jj & 7;
    const int col = c * 256 + (i < 4 ? 4 * l + i : 128 + 4 * l + (i - 4));
    float v[2] = {0.f, 0.f};
    if (m < M && col < K) {
      v[0] = xc[(size_t)m * ldx + col];
      v[1] = xs[(size_t)m * ldx + col];
    }
#pragma unroll
    for (int sh = 0; sh < 2; ++sh) {
      const __nv_bfloat16 b0 = __float2bfloat16_rn(v[sh]);
      const float r1 = __fsub_rn(v[sh], __bfloat162float(b0));
      const __nv_bfloat16 b1 = __float2bfloat16_rn(r1);
      const float r2 = __fsub_rn(r1, __bfloat162float(b1));
      const __nv_bfloat16 b2 = __float2bfloat16_rn(r2);
      out[(size_t)(sh * 3 + 0) * plane + idx] = __bfloat16_as_ushort(b0);
      out[(size_t)(sh * 3 + 1) * plane + idx] = __bfloat16_as_ushort(b1);
      out[(size_t)(sh * 3 + 2) * plane + idx] = __bfloat16_as_ushort(b2);
    }
  }
}

// The same with 8 physical columns per thread (two float4 loads per share, one 16-byte store per
// plane): rows 16-byte aligned (ldx % 4 == 0, aligned bases) and K a multiple of 256.
__global__ void split_planes_vec_kernel(const float* __restrict__ xc, const float* __restrict__ xs, int ldx, int M,
                                        int Mp, int KP, uint16_t* __restrict__ out) {
  pdl_wait();  // the shares come from the previous kernel
  const size_t plane = (size_t)Mp * KP;
  const long long groups = (long long)Mp * (KP / 8);
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(g / (KP / 8)), j = (int)(g % (KP / 8)) * 8;
    const int c = j >> 8, l = (j & 255) >> 3;
    const int col0 = c * 256 + 4 * l, col1 = col0 + 128;  // physical j..j+3 <- col0.., j+4..j+7 <- col1..
    float v[2][8];
#pragma unroll
    for (int sh = 0; sh < 2; ++sh) {
      const float* x = sh ? xs : xc;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (m < M) {
        a = *reinterpret_cast<const float4*>(x + (size_t)m * ldx + col0);
        b = *reinterpret_cast<const float4*>(x + (size_t)m * ldx + col1);
      }
      v[sh][0] = a.x; v[sh][1] = a.y; v[sh][2] = a.z; v[sh][3] = a.w;
      v[sh][4] = b.x; v[sh][5] = b.y; v[sh][6] = b.z; v[sh][7] = b.w;
    }
    const size_t at = (size_t)m * KP + j;
#pragma unroll
    for (int sh = 0; sh < 2; ++sh) {
      uint16_t t[8][3];
#pragma unroll
      for (int i = 0; i < 8; ++i) split3(v[sh][i], t[i]);
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        uint4 pk;
        pk.x = (uint32_t)t[0][q] | ((uint32_t)t[1][q] << 16);
        pk.y = (uint32_t)t[2][q] | ((uint32_t)t[3][q] << 16);
        pk.z = (uint32_t)t[4][q] | ((uint32_t)t[5][q] << 16);
        pk.w = (uint32_t)t[6][q] | ((uint32_t)t[7][q] << 16);
        *reinterpret_cast<uint4*>(out + (size_t)(sh * 3 + q) * plane + at) = pk;
      }
    }
  }
}

// Logical column of physical plane column j (the weight blocks' column permutation).
__device__ __forceinline__ int plane_col(int j) {
  const int c = j >> 8, jj = j & 255;
  const int l = jj >> 3, i = jj & 7;
  return c * 256 + (i < 4 ? 4 * l + i : 128 + 4 * l + (i - 4));
}

// RMSNorm + reshare straight into the six bf16 planes (replaces the norm kernel + split_planes
// pair before a tensor-core linear). CTA (row m, slice): every CTA of a row reduces the whole row
// (same thread count and per-thread order as norm_reshare_kernel, so the same inverse RMS) into
// shared memory, then writes its slice of 256-column chunks of the planes and of h = D + H. Rows
// from M to Mp are zero.
constexpr int kNormBatch = 8;  // a 5120-wide row in one round of loads at 1024 threads

__global__ void norm_planes_kernel(const NormArgs a, int M, int Mp, int KP, int chunks_per_slice,
                                   uint16_t* __restrict__ out) {
  extern __shared__ float xrow[];  // [K] x = h_c + h_s of this row
  __shared__ float red[33];
  if (threadIdx.x == 0) pdl_trigger();
  const int m = blockIdx.x;
  const int K = a.n;
  const size_t plane = (size_t)Mp * KP;
  const int j0 = blockIdx.y * chunks_per_slice * 256, j1 = min(KP, j0 + chunks_per_slice * 256);
  const int T = blockDim.x, tid = threadIdx.x;
  // gamma of this thread's first column of the slice: a weight, loaded before the wait
  float g_first = 0.0f;
  if (j0 + tid < j1 && plane_col(j0 + tid) < K) g_first = __ldg(a.gamma + plane_col(j0 + tid));
  pdl_wait();  // the shares come from earlier kernels
  if (m >= M) {
    for (int j = j0 + tid; j < j1; j += T)
#pragma unroll
      for (int p = 0; p < 6; ++p) out[(size_t)p * plane + (size_t)m * KP + j] = 0;
    return;
  }
  const float* hc = a.Hc + (size_t)m * a.ldh;
  const float* hs = a.Hs + (size_t)m * a.ldh;
  const float* dc = a.Dc ? a.Dc + (size_t)m * a.ldh : nullptr;
  const float* ds = a.Ds ? a.Ds + (size_t)m * a.ldh : nullptr;
  float* oc = a.Hout_c ? a.Hout_c + (size_t)m * a.ldh : nullptr;
  float* os = a.Hout_s ? a.Hout_s + (size_t)m * a.ldh : nullptr;
  float sq = 0.0f;
  for (int b = tid; b < K; b += kNormBatch * T) {
    float c[kNormBatch], s[kNormBatch], e[kNormBatch], f[kNormBatch];
#pragma unroll
    for (int q = 0; q < kNormBatch; ++q) {
      const int i = b + q * T;
      c[q] = s[q] = e[q] = f[q] = 0.0f;
      if (i < K) {
        c[q] = __ldcg(hc + i);
        s[q] = __ldcg(hs + i);
        if (dc) {
          e[q] = __ldcg(dc + i);
          f[q] = __ldcg(ds + i);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kNormBatch; ++q) {
      const int i = b + q * T;
      if (i >= K) break;
      float cc = c[q], ss = s[q];
      if (dc) {
        // residual: sublayer output + residual stream, per share
        cc = __fadd_rn(e[q], cc);
        ss = __fadd_rn(f[q], ss);
        if (oc && i >= j0 && i < j1) {
          oc[i] = cc;
          os[i] = ss;
        }
      }
      const float x = __fadd_rn(cc, ss);
      xrow[i] = x;
      sq = __fmaf_rn(x, x, sq);
    }
  }
  // block sum (the norm kernel's reduction)
  {
    const int lane = tid & 31, warp = tid >> 5, nw = T >> 5;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    if (warp == 0) {
      float w = lane < nw ? red[lane] : 0.0f;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) w = __fadd_rn(w, __shfl_xor_sync(0xffffffffu, w, o));
      if (lane == 0) red[32] = w;
    }
    __syncthreads();
  }
  const float mean_sq = __fdiv_rn(red[32], (float)K);
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
  const float* mk = a.mask ? a.mask + (size_t)m * a.ldmask : nullptr;
  for (int j = j0 + tid; j < j1; j += T) {
    const int col = plane_col(j);
    float vc = 0.0f, vs = 0.0f;
    if (col < K) {
      const float gm = (j == j0 + tid) ? g_first : a.gamma[col];
      float r = __fmul_rn(__fmul_rn(xrow[col], inv), gm);
      if (a.variant == SHD_NL_MPC && !isfinite(r)) r = 0.0f;
      const float mv = mk ? mk[col] : 0.0f;
      vc = __fsub_rn(r, mv);
      vs = mv;
    }
    uint16_t bc[3], bs[3];
    split3(vc, bc);
    split3(vs, bs);
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      out[(size_t)t * plane + (size_t)m * KP + j] = bc[t];
      out[(size_t)(3 + t) * plane + (size_t)m * KP + j] = bs[t];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Weight tensor map: dims (innermost first) 256 columns, 32 rows, nKC chunks, nT tiles of the
// 16 KB-block layout; box 64 x 32 x 1 x 4 = a 128-row x 64-column tile.
int weight_map(shd_ctx* ctx, const shd_weight* w, CUtensorMap* map) {
  auto enc = encode_fn();
  if (!enc) return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "tensor-core linear: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {256, 32, (cuuint64_t)w->nKC, (cuuint64_t)w->nT};
  const cuuint64_t strides[3] = {512, (cuuint64_t)kBlockBytes, (cuuint64_t)w->nKC * kBlockBytes};
  const cuuint32_t box[4] = {kTcBK, 32, 1, 4};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, w->d_tiles, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return shd_fail(ctx, SHD_ERR_CUDA, "tensor-core linear: weight tensor map");
  return SHD_OK;
}

// Activation-plane tensor map: dims KP, Mp, 6 planes; box 64 x NT x 6.
int planes_map(shd_ctx* ctx, const uint16_t* planes, int Mp, int KP, int nt, CUtensorMap* map) {
  auto enc = encode_fn();
  if (!enc) return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "tensor-core linear: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)KP, (cuuint64_t)Mp, 6};
  const cuuint64_t strides[2] = {(cuuint64_t)KP * 2, (cuuint64_t)Mp * KP * 2};
  const cuuint32_t box[3] = {kTcBK, (cuuint32_t)nt, 6};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(planes), dims, strides,
                         box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return shd_fail(ctx, SHD_ERR_CUDA, "tensor-core linear: activation tensor map");
  return SHD_OK;
}

int ensure_buffer(shd_ctx* ctx, void** buf, size_t* have, size_t elems) {
  if (*have >= elems) return SHD_OK;
  if (*buf) {
    SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));  // earlier launches may still read it
    cudaFree(*buf);
  }
  *buf = nullptr;
  *have = 0;
  SHD_CHECK_CUDA(ctx, cudaMalloc(buf, elems * 2));
  *have = elems;
  return SHD_OK;
}

// The planes this linear computes and reads; and the planes a producer writes for the linear after
// it (tc_input_planes), in a second buffer so that the producer's writes never meet its own reads.
int ensure_planes(shd_ctx* ctx, size_t elems) {
  return ensure_buffer(ctx, &ctx->d_tc_planes, &ctx->tc_planes_elems, elems);
}
int ensure_next_planes(shd_ctx* ctx, size_t elems) {
  return ensure_buffer(ctx, &ctx->d_tc_planes_next, &ctx->tc_planes_next_elems, elems);
}

template <int NT>
int launch_tc_t(shd_ctx* ctx, const TcArgs& ta, const CUtensorMap& mw, const CUtensorMap& mx) {
  static unsigned attr_devices = 0;
  const int S = std::min(10, (kTcSmemLimit - 1024 - 256) / TcSmem<NT>::kStage);  // barriers: 256-byte tail
  if (S < 2) return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "tensor-core linear: token tile too wide");
  const size_t smem = 1024 + (size_t)S * TcSmem<NT>::kStage + 256;
  if (!(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(tc_linear_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kTcSmemLimit));
    attr_devices |= 1u << (ctx->device & 31);
  }
  TcArgs a = ta;
  a.nstages = S;
  const int tiles = a.n_row * a.n_tok * a.ksplit;
  const int grid = std::min(tiles, ctx->num_sms);
  SHD_CHECK_CUDA(ctx, launch_pdl(tc_linear_kernel<NT>, dim3(grid), dim3(kTcThreads), smem, ctx->stream, a, mw, mx));
  ctx->launches++;
  if (a.ksplit > 1) {
    SHD_CHECK_CUDA(ctx, launch_pdl(tc_reduce_kernel<NT>, dim3(a.n_row, a.n_tok), dim3(kTcBM, kTcReduceY), 0,
                                   ctx->stream, a));
    ctx->launches++;
  }
  return SHD_OK;
}

int ensure_ws(shd_ctx* ctx, size_t floats) {
  if (ctx->tc_ws_floats >= floats) return SHD_OK;
  if (ctx->d_tc_ws) cudaFree(ctx->d_tc_ws);
  ctx->d_tc_ws = nullptr;
  ctx->tc_ws_floats = 0;
  SHD_CHECK_CUDA(ctx, cudaMalloc(&ctx->d_tc_ws, floats * 4));
  ctx->tc_ws_floats = floats;
  return SHD_OK;
}

}  // namespace

int tc_token_tile(int M) { return M <= 8 ? 8 : (M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128))); }

PlaneOut tc_input_planes(shd_ctx* ctx, const shd_weight* w, int M) {
  PlaneOut o{};
  if (M <= 0 || w->kind != WK_BF16 || !tc_preferred(w, M)) return o;
  if (M % tc_token_tile(M) != 0 || w->K % kChunkBf16 != 0) return o;
  const int KP = w->nKC * kChunkBf16;
  if (ensure_next_planes(ctx, (size_t)6 * M * KP) != SHD_OK) return o;
  o.p = reinterpret_cast<uint16_t*>(ctx->d_tc_planes_next);
  o.Mp = M;
  o.KP = KP;
  return o;
}

int launch_linear_tc(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs g, const NormArgs* norm,
                     bool planes_ready, const PlaneOut* out_planes, bool* wrote_out) {
  if (wrote_out) *wrote_out = false;
  if (w->kind != WK_BF16) return shd_fail(ctx, SHD_ERR_ARG, "tensor-core linear: need a bf16 weight");
  if (M <= 0) return SHD_OK;
  int rc = gemv_prepare(ctx, w, g, false);
  if (rc) return rc;
  const int nt = tc_token_tile(M);
  const int n_tok = (M + nt - 1) / nt;
  const int Mp = n_tok * nt;
  const int KP = w->nKC * kChunkBf16;
  // planes written by the producer of this linear's input (tc_input_planes) are read where it wrote
  // them; otherwise this launch computes its planes into the context's own buffer
  if (!planes_ready && (rc = ensure_planes(ctx, (size_t)6 * Mp * KP))) return rc;
  uint16_t* planes = reinterpret_cast<uint16_t*>(planes_ready ? ctx->d_tc_planes_next : ctx->d_tc_planes);
  if (planes_ready) {
    if (Mp != M || KP != w->K || ctx->tc_planes_next_elems < (size_t)6 * Mp * KP)
      return shd_fail(ctx, SHD_ERR_ARG, "tensor-core linear: planes written for another shape");
  } else if (norm) {
    if (norm->n != w->K) return shd_fail(ctx, SHD_ERR_ARG, "tensor-core linear: norm width != in_features");
    // every CTA of a row reloads the whole row for its sum: with few rows, slices of one column per
    // thread (at least one 256-column chunk) keep the SMs busy; with a row per SM or more (prompt
    // chunks), one CTA per row writes all its planes and the row is read once
    const int n_chunks = w->nKC;
    const int threads = norm->n >= 4096 ? 1024 : (norm->n >= 1024 ? 512 : 128);  // as launch_norm
    const int cps = Mp >= ctx->num_sms ? n_chunks : std::max(1, threads / 256);
    const int slices = (n_chunks + cps - 1) / cps;
    const size_t smem = (size_t)norm->n * 4;
    static unsigned attr_devices = 0;
    if (smem > 48 * 1024 && !(attr_devices & (1u << (ctx->device & 31)))) {
      SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(norm_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      attr_devices |= 1u << (ctx->device & 31);
    }
    if (smem > 200 * 1024) return shd_fail(ctx, SHD_ERR_ARG, "tensor-core linear: norm row too long");
    SHD_CHECK_CUDA(ctx, launch_pdl(norm_planes_kernel, dim3(Mp, slices), dim3(threads), smem, ctx->stream, *norm, M, Mp,
                                   KP, cps, planes));
    ctx->launches++;
  } else if (g.ldx % 4 == 0 && w->K % kChunkBf16 == 0 && shd_aligned16(g.Xc) && shd_aligned16(g.Xs)) {
    const long long groups = (long long)Mp * (KP / 8);
    const int blocks = (int)std::min<long long>((groups + 255) / 256, 8LL * ctx->num_sms);
    SHD_CHECK_CUDA(ctx, launch_pdl(split_planes_vec_kernel, dim3(blocks), dim3(256), 0, ctx->stream, g.Xc, g.Xs,
                                   g.ldx, M, Mp, KP, planes));
    ctx->launches++;
  } else {
    const long long total = (long long)Mp * KP;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 4LL * ctx->num_sms);
    SHD_CHECK_CUDA(ctx, launch_pdl(split_planes_kernel, dim3(blocks), dim3(256), 0, ctx->stream, g.Xc, g.Xs, g.ldx, M,
                                   w->K, Mp, KP, planes));
    ctx->launches++;
  }
  if (!w->tmap) {
    auto* m = new (std::align_val_t(64)) CUtensorMap;
    rc = weight_map(ctx, w, m);
    if (rc) {
      ::operator delete(m, std::align_val_t(64));
      return rc;
    }
    const_cast<shd_weight*>(w)->tmap = m;
  }
  alignas(64) CUtensorMap mx;
  if ((rc = planes_map(ctx, planes, Mp, KP, nt, &mx))) return rc;
  TcArgs ta{};
  ta.g = g;
  ta.epi = epi;
  ta.M = M;
  ta.n_tok = n_tok;
  ta.n_row = (w->nT + 3) / 4;
  ta.n_kb = w->nKC * (kChunkBf16 / kTcBK);
  // split K to balance the SMs: work items (row tile, token tile, K range) go round-robin to one CTA
  // per SM, so d splits take about ceil(items * d / SMs) / d full-K item times, plus the reduce
  // kernel (a launch and the partial sums through L2). Model: an item streams its weights at about
  // 45 GB/s per SM, the reduce costs 6 us plus its partials at 2 TB/s. Take the cheapest d (a
  // divisor of the K blocks keeping at least 8 blocks per split), the smallest on ties.
  ta.ksplit = 1;
  {
    const int items = ta.n_row * n_tok;
    const int sms = ctx->num_sms;
    const double item_us = (double)kTcBM * ta.n_kb * kTcBK * 2 / 45.0e3;
    double best = (double)((items + sms - 1) / sms) * item_us;
    for (int d = 2; d <= 16; ++d) {
      if (ta.n_kb % d != 0 || ta.n_kb / d < 8) continue;
      const double partial_bytes = (double)d * n_tok * nt * ta.n_row * kTcBM * 8;
      const double cost = (double)((items * d + sms - 1) / sms) / d * item_us + 6.0 + partial_bytes / 2.0e6;
      if (cost < best - 1e-9) {
        best = cost;
        ta.ksplit = d;
      }
    }
  }
  if (ta.ksplit > 1) {
    if ((rc = ensure_ws(ctx, (size_t)ta.ksplit * n_tok * nt * ta.n_row * kTcBM * 2))) return rc;
    ta.ws = ctx->d_tc_ws;
  }
  // the SwiGLU output as the next linear's planes, from the epilogue (in the reduce kernel when K is
  // split); they go to the second plane buffer, so this launch's own planes stay intact
  if (out_planes && out_planes->p && epi == EPI_GATEUP && out_planes->p != planes) {
    ta.out = *out_planes;
    if (wrote_out) *wrote_out = true;
  }
  const CUtensorMap& mw = *static_cast<const CUtensorMap*>(w->tmap);
  if (nt == 8) return launch_tc_t<8>(ctx, ta, mw, mx);
  if (nt == 16) return launch_tc_t<16>(ctx, ta, mw, mx);
  if (nt == 32) return launch_tc_t<32>(ctx, ta, mw, mx);
  if (nt == 64) return launch_tc_t<64>(ctx, ta, mw, mx);
  return launch_tc_t<128>(ctx, ta, mw, mx);
}

void free_weight_map(shd_weight* w) {
  if (w && w->tmap) {
    ::operator delete(static_cast<CUtensorMap*>(w->tmap), std::align_val_t(64));
    w->tmap = nullptr;
  }
}

}  // namespace shd
