// Prefill attention on the tensor cores (tcgen05, sm_100a): secure_attention_approx /
// compute_mpc_attention_on_shares (crates/v2/sharing/src/secure_nonlinear.rs:287-333,
// crates/v2/server/src/routes/secure_inference_mpc.rs:568-663) for a block of consecutive prompt
// positions of one sequence, followed by the reshare. The reference computes this position by
// position on the CPU; the plaintext analogue of the tiling is its flash_attention_kernel
// (crates/v2/core/src/kernel.rs:562-657).
//
// One CTA per (128 query rows, query head). Q, K and V are the reconstructed f32 values; every f32
// operand is split exactly into three bf16 terms (x = x0 + x1 + x2, shd_planes.cuh split3), and a
// dot product of two split values is the sum of the six term products with i + j <= 2 (the three
// dropped ones are below 2^-24 of the total, under f32 rounding). bf16 x bf16 products are exact and
// the tensor core accumulates in f32, so scores and weighted sums keep f32 accuracy:
//   S = sum_(i+j<=2) Q_i K_j^T      M = 128 queries, N = 64 positions, K = 128 head dims
//   O_tile = sum_(i+j<=2) P_i V_j   M = 128 queries, N = 128 head dims, K = 64 positions
// Eight worker warps load and split the K and V tiles into 128-byte-swizzled K-major shared-memory
// planes (V transposed so that positions are K); warps w and w + 4 share query rows 32 (w % 4) ..
// + 31 (their tensor-memory lanes) and split each row's columns in halves: they read the scores
// from tensor memory, run the online softmax (running max exchanged through shared memory, the
// reference's +-40 clamp applied to s - max for the approximate variant, masked positions weigh
// exactly 0), write the weights' planes, and keep half the output row in registers (O = O * alpha
// + O_tile). Warp 0 also owns tensor memory (S: 64 columns, O_tile: 128 columns) and thread 0
// issues the MMAs, each group committed to an mbarrier the warps wait on (bounded, as every wait in
// this library).
#include <cuda_bf16.h>

#include <cmath>

#include "shd_nonlinear.cuh"
#include "shd_planes.cuh"
#include "shd_tcgen05.cuh"

namespace shd {
namespace {

constexpr int kFQ = 128;          // query rows per CTA
constexpr int kFKV = 64;          // positions per K/V tile
constexpr int kFHD = 128;         // head_dim
constexpr int kFWorkers = 8;      // worker warps: warp w serves query rows 32 (w % 4) .. + 31 (its
                                  // tensor-memory lanes) and half w / 4 of the columns
constexpr int kFThreads = 32 * kFWorkers;  // warp 0 also owns tensor memory, thread 0 issues the MMAs
constexpr uint32_t kFCols = 256;  // S at columns [0, 64), O_tile at [64, 192)
constexpr uint32_t kFColO = 64;

// shared-memory plan (bytes from a 1024-aligned base)
constexpr uint32_t kQOff = 0;                          // Q   [3 terms][2 K blocks][128 rows][128 B]
constexpr uint32_t kKVOff = 3 * 2 * kFQ * 128;         // K   [3][2][64 rows][128 B]  (or)  V^T [3][128 rows][128 B]
constexpr uint32_t kPOff = kKVOff + 3 * kFHD * 128;    // P   [3][128 rows][128 B]
constexpr uint32_t kRedOff = kPOff + 3 * kFQ * 128;    // [2 halves][128 rows] f32: row maxima / sums
constexpr uint32_t kBarOff = kRedOff + 2 * kFQ * 4;    // s_full, pv_full, done, tmem base, abort
constexpr size_t kFSmem = kBarOff + 64 + 1024;         // + alignment slack

// the six kept term pairs (i, j), i + j <= 2
__device__ __forceinline__ int pair_a(int p) { return (p == 2 || p == 4) ? 1 : (p == 5 ? 2 : 0); }
__device__ __forceinline__ int pair_b(int p) { return (p == 1 || p == 4) ? 1 : (p == 3 ? 2 : 0); }

struct FlashArgs {
  AttnArgs a;  // Q, K/V cache, groups, pos (pos[0] = position of row 0), seq, variant, mask, out
  int M;       // query rows (consecutive positions pos[0] .. pos[0] + M - 1 of slot seq[0])
};

// Warp-uniform bounded wait (the tensor-memory loads that follow are warp-collective).
__device__ __forceinline__ bool flash_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
  if (!ok) {
    if ((threadIdx.x & 31) == 0) atomicOr(err, SHD_DEVERR_TIMEOUT_FULL);
    *abort_flag = 1;
  }
  return ok;
}

// The two worker warps of one lane quarter (warps q and q + 4) exchange row values through shared
// memory: named barrier 1 + q over their 64 threads.
__device__ __forceinline__ void pair_sync(int quarter) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}

// rows [0, nrows) x 128 f32 columns of `src` (row stride ld) -> three K-major 128-byte-swizzled bf16
// planes at dst + t * plane_bytes, K blocks of 64 columns nrows * 128 bytes apart. Rows at or past
// `valid` are zero. Worker warp w takes rows w, w + 8, ...; lane l columns 4l .. 4l + 3. The loads
// of 4 rows are issued before any is used (one memory latency per 4 rows, not per row).
__device__ __forceinline__ void split_rows_kmajor(uint8_t* dst, uint32_t plane_bytes, const float* src,
                                                  size_t ld, int nrows, int valid, int warp, int lane) {
  constexpr int G = 4;
  const int kb = lane >> 4, e = (4 * lane) & 63;
  for (int r0 = warp; r0 < nrows; r0 += kFWorkers * G) {
    float4 v[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int r = r0 + g * kFWorkers;
      v[g] = (r < valid && r < nrows) ? *reinterpret_cast<const float4*>(src + (size_t)r * ld + 4 * lane)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int r = r0 + g * kFWorkers;
      if (r >= nrows) continue;
      uint16_t b[4][3];
      split3(v[g].x, b[0]);
      split3(v[g].y, b[1]);
      split3(v[g].z, b[2]);
      split3(v[g].w, b[3]);
      const uint32_t off = (uint32_t)kb * (uint32_t)nrows * 128u + sw128_offset(r, e);
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        uint2 pk;
        pk.x = (uint32_t)b[0][t] | ((uint32_t)b[1][t] << 16);
        pk.y = (uint32_t)b[2][t] | ((uint32_t)b[3][t] << 16);
        *reinterpret_cast<uint2*>(dst + (size_t)t * plane_bytes + off) = pk;
      }
    }
  }
}

// V rows [0, 64) (positions) x 128 dims -> three planes of V^T: [128 dims][64 positions] K-major,
// 128-byte swizzle. Lane l takes positions 2l, 2l + 1 (one 4-byte store per dim and term, the 32
// lanes of a warp filling one 128-byte row); worker warp w takes dims 16w .. 16w + 15.
__device__ __forceinline__ void split_v_transposed(uint8_t* dst, const float* V, size_t ld, int valid, int warp,
                                                   int lane) {
  const int p0 = 2 * lane;
  const float* r0 = V + (size_t)p0 * ld + 16 * warp;
  const float* r1 = r0 + ld;
  const bool v0ok = p0 < valid, v1ok = p0 + 1 < valid;
  float4 a[4], b[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    a[q] = v0ok ? *reinterpret_cast<const float4*>(r0 + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
    b[q] = v1ok ? *reinterpret_cast<const float4*>(r1 + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float av[4] = {a[q].x, a[q].y, a[q].z, a[q].w}, bv[4] = {b[q].x, b[q].y, b[q].z, b[q].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = 16 * warp + 4 * q + j;
      uint16_t sa[3], sb[3];
      split3(av[j], sa);
      split3(bv[j], sb);
      const uint32_t off = sw128_offset(d, p0);
#pragma unroll
      for (int t = 0; t < 3; ++t)
        *reinterpret_cast<uint32_t*>(dst + (size_t)t * (kFHD * 128) + off) = (uint32_t)sa[t] | ((uint32_t)sb[t] << 16);
    }
  }
}

__global__ void __launch_bounds__(kFThreads, 1) flash_prefill_kernel(const __grid_constant__ FlashArgs fa) {
  const AttnArgs& a = fa.a;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + kRedOff);
  uint64_t* s_full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* pv_full = s_full + 1;
  uint64_t* done = s_full + 2;
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(s_full + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool worker = true;  // every warp works; thread 0 also issues the MMAs
  const int quarter = warp & 3, half = (warp >> 2) & 1;
  const int row = 32 * quarter + lane;  // query row of this worker thread (tensor-memory lane)

  if (tid == 0) {
    mbar_init(s_full, 1);
    mbar_init(pv_full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (tid == 0) pdl_trigger();
  pdl_wait();  // queries, the block's K/V rows and the positions come from the q/k/v kernel
  if (warp == 0) tmem_alloc(tmem_base, kFCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_base;

  // this CTA: query head hq (local), rows q0 .. q0 + 127 of the block
  const int hq = blockIdx.y, q0 = blockIdx.x * kFQ;
  int kvh = 0;
  for (int g = 0; g < a.n_groups; ++g) {
    const int4 gr = a.groups[g];
    if (hq >= gr.y && hq < gr.y + gr.z) kvh = gr.x;
  }
  const int pos0 = __ldcg(a.pos);
  const int sq = a.seq ? __ldcg(a.seq) : 0;
  const int rows = min(kFQ, fa.M - q0);                  // live query rows of this CTA
  const int kv_len = pos0 + q0 + rows;                   // positions the last live row attends to
  const float* K = a.Kcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * kFHD;
  const float* V = a.Vcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * kFHD;
  const bool mpc = a.variant == SHD_NL_MPC;
  const int my_pos = pos0 + q0 + row;
  const int n_tiles = (kv_len + kFKV - 1) / kFKV;
  const int sc0 = half * (kFKV / 2);   // this thread's score columns [sc0, sc0 + 32)
  const int oc0 = half * (kFHD / 2);   // this thread's output columns [oc0, oc0 + 64)

  // Q planes, once
  if (worker)
    split_rows_kmajor(smem + kQOff, 2 * kFQ * 128, a.Q + (size_t)q0 * a.ldq + (size_t)hq * kFHD, (size_t)a.ldq,
                      kFQ, rows, warp, lane);

  float o[kFHD / 2];
#pragma unroll
  for (int d = 0; d < kFHD / 2; ++d) o[d] = 0.0f;
  float m_run = -INFINITY, l_half = 0.0f;  // running max (same in both halves), this half's sum
  const uint32_t t_row = tbase + ((uint32_t)(quarter * 32) << 16);  // this warp's tensor-memory lanes

  for (int j = 0; j < n_tiles; ++j) {
    const int t0 = j * kFKV;
    const int nvalid = min(kFKV, kv_len - t0);
    if (worker) {
      split_rows_kmajor(smem + kKVOff, 2 * kFKV * 128, K + (size_t)t0 * a.kvd, (size_t)a.kvd, kFKV, nvalid, warp,
                        lane);
      fence_proxy_async_smem();
    }
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16_f32_mn(kFQ, kFKV);
#pragma unroll
      for (int p = 0; p < 6; ++p) {
        const int ta = pair_a(p), tb = pair_b(p);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t ad = smem_desc_sw128(smem + kQOff + (size_t)(ta * 2 + kb) * kFQ * 128);
          const uint64_t bd = smem_desc_sw128(smem + kKVOff + (size_t)(tb * 2 + kb) * kFKV * 128);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tbase, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (p > 0 || kb > 0 || k > 0) ? 1u : 0u);
        }
      }
      tc_commit(s_full);
    }
    float alpha = 0.0f;
    if (worker) {
      // both warps of a pair meet at the exchange whatever their waits returned (no unbounded wait)
      const bool ok = flash_wait(s_full, (uint32_t)(j & 1), a.err, abort_flag);
      // this half's 32 scores of the row, loaded once (four loads, one wait); its maximum over the
      // tile's valid positions, then the row's through the pair exchange
      float sv[kFKV / 2];
      float tmax = -INFINITY;
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < kFKV / 2; c0 += 8) {
          float s8[8];
          tmem_ld8(t_row + (uint32_t)(sc0 + c0), s8);
#pragma unroll
          for (int i = 0; i < 8; ++i) sv[c0 + i] = s8[i];
        }
        tmem_wait_ld();
#pragma unroll
        for (int c0 = 0; c0 < kFKV / 2; c0 += 8) tmem_loaded(*reinterpret_cast<float(*)[8]>(&sv[c0]));
#pragma unroll
        for (int c = 0; c < kFKV / 2; ++c) {
          sv[c] = __fmul_rn(sv[c], a.scale);
          if (t0 + sc0 + c <= my_pos) tmax = fmaxf(tmax, sv[c]);
        }
      }
      red[half * kFQ + row] = tmax;
      pair_sync(quarter);
      if (ok) {
        tmax = fmaxf(tmax, red[(half ^ 1) * kFQ + row]);
        const float mnew = fmaxf(m_run, tmax);
        // weights, this half's sum, and their three bf16 planes (columns sc0 .. of P's row)
        float tsum = 0.0f;
#pragma unroll
        for (int c0 = 0; c0 < kFKV / 2; c0 += 8) {
          uint16_t b[8][3];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float pe = 0.0f;
            if (t0 + sc0 + c0 + i <= my_pos) {
              float x = __fsub_rn(sv[c0 + i], mnew);
              if (!mpc) x = fminf(fmaxf(x, -40.0f), 40.0f);
              pe = expf(x);
            }
            tsum = __fadd_rn(tsum, pe);
            split3(pe, b[i]);
          }
#pragma unroll
          for (int t = 0; t < 3; ++t) {
            uint4 pk;
            pk.x = (uint32_t)b[0][t] | ((uint32_t)b[1][t] << 16);
            pk.y = (uint32_t)b[2][t] | ((uint32_t)b[3][t] << 16);
            pk.z = (uint32_t)b[4][t] | ((uint32_t)b[5][t] << 16);
            pk.w = (uint32_t)b[6][t] | ((uint32_t)b[7][t] << 16);
            *reinterpret_cast<uint4*>(smem + kPOff + (size_t)t * kFQ * 128 + sw128_offset(row, sc0 + c0)) = pk;
          }
        }
        alpha = (m_run == -INFINITY) ? 0.0f : expf(__fsub_rn(m_run, mnew));
        l_half = __fmaf_rn(l_half, alpha, tsum);
        m_run = mnew;
        tc_fence_before();
        // the S MMAs have read the K planes: the same buffer takes V^T
        split_v_transposed(smem + kKVOff, V + (size_t)t0 * a.kvd, (size_t)a.kvd, nvalid, warp, lane);
        fence_proxy_async_smem();
      }
    }
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16_f32_mn(kFQ, kFHD);
#pragma unroll
      for (int p = 0; p < 6; ++p) {
        const uint64_t ad = smem_desc_sw128(smem + kPOff + (size_t)pair_a(p) * kFQ * 128);
        const uint64_t bd = smem_desc_sw128(smem + kKVOff + (size_t)pair_b(p) * kFHD * 128);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma(tbase + kFColO, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (p > 0 || k > 0) ? 1u : 0u);
      }
      tc_commit(pv_full);
    }
    if (worker) {
      if (flash_wait(pv_full, (uint32_t)(j & 1), a.err, abort_flag)) {
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < kFHD / 2; c0 += 32) {
          float pv[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u) tmem_ld8(t_row + kFColO + (uint32_t)(oc0 + c0 + 8 * u), pv[u]);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 4; ++u) tmem_loaded(pv[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 8; ++i) o[c0 + 8 * u + i] = __fmaf_rn(o[c0 + 8 * u + i], alpha, pv[u][i]);
        }
        tc_fence_before();
      }
    }
  }

  // output row: O / L, reshared as (y - mask, mask); L = the two halves' sums
  __syncthreads();  // every thread reads the same abort flag before the pair exchange
  if (worker && !*abort_flag) {
    red[half * kFQ + row] = l_half;
    pair_sync(quarter);
    const float l_run = __fadd_rn(red[row], red[kFQ + row]);
    if (row < rows) {
      const int m = q0 + row;
      float* oc = a.Oc + (size_t)m * a.ldo + (size_t)hq * kFHD + oc0;
      float* os = a.Os + (size_t)m * a.ldo + (size_t)hq * kFHD + oc0;
      const float* mk = a.mask ? a.mask + (size_t)m * a.ldmask + (size_t)hq * kFHD + oc0 : nullptr;
      if (mpc && !(l_run > 1e-10f && isfinite(l_run))) {
        // compute_mpc_attention_on_shares: weights 1/seq_len when the sum is not usable
        const float invk = __fdiv_rn(1.0f, (float)(my_pos + 1));
        for (int d = 0; d < kFHD / 2; ++d) {
          float u = 0.0f;
          for (int t = 0; t <= my_pos; ++t) u = __fmaf_rn(invk, V[(size_t)t * a.kvd + oc0 + d], u);
          const float mv = mk ? mk[d] : 0.0f;
          oc[d] = __fsub_rn(u, mv);
          os[d] = mv;
        }
      } else {
#pragma unroll
        for (int d = 0; d < kFHD / 2; d += 4) {
          float4 y, mv = make_float4(0.f, 0.f, 0.f, 0.f);
          if (mk) mv = *reinterpret_cast<const float4*>(mk + d);
          y.x = __fsub_rn(__fdiv_rn(o[d], l_run), mv.x);
          y.y = __fsub_rn(__fdiv_rn(o[d + 1], l_run), mv.y);
          y.z = __fsub_rn(__fdiv_rn(o[d + 2], l_run), mv.z);
          y.w = __fsub_rn(__fdiv_rn(o[d + 3], l_run), mv.w);
          *reinterpret_cast<float4*>(oc + d) = y;
          *reinterpret_cast<float4*>(os + d) = mv;
        }
      }
    }
  }
  // every MMA issued has completed before tensor memory is released
  if (tid == 0) {
    tc_commit(done);
    if (!mbar_wait_bounded(done, 0)) atomicOr(a.err, SHD_DEVERR_TIMEOUT_DRAIN);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, kFCols);
}

}  // namespace

bool flash_prefill_supported(const AttnArgs& a, int M) {
  const bool rows16 = (a.ldq % 4 == 0) && (a.kvd % 4 == 0) && (a.ldo % 4 == 0) && (!a.mask || a.ldmask % 4 == 0);
  const bool ptr16 = shd_aligned16(a.Q) && shd_aligned16(a.Kcache) && shd_aligned16(a.Vcache) &&
                     shd_aligned16(a.Oc) && shd_aligned16(a.Os) && (!a.mask || shd_aligned16(a.mask)) &&
                     a.kv_seq_stride % 4 == 0;
  return a.head_dim == kFHD && M >= 1 && rows16 && ptr16;
}

// Rows m = 0 .. M-1 are positions pos[0] + m of slot seq[0] (a prompt block), each attending to
// positions [0, pos[0] + m]; the block's own K/V rows are in the cache before the launch.
int launch_flash_prefill(shd_ctx* ctx, const AttnArgs& a, int M) {
  if (!flash_prefill_supported(a, M)) return shd_fail(ctx, SHD_ERR_UNSUPPORTED, "flash prefill: head_dim must be 128");
  const int n_q = a.ldq / kFHD;  // local query heads
  static unsigned attr_devices = 0;
  if (!(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kFSmem));
    attr_devices |= 1u << (ctx->device & 31);
  }
  FlashArgs fa{};
  fa.a = a;
  fa.M = M;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M + kFQ - 1) / kFQ, n_q, 1);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = kFSmem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SHD_CHECK_CUDA(ctx, cudaLaunchKernelEx(&cfg, flash_prefill_kernel, fa));
  ctx->launches++;
  return SHD_OK;
}

}  // namespace shd
