// Decode attention over the device-resident reconstructed KV cache (secure_attention_approx,
// crates/v2/sharing/src/secure_nonlinear.rs:287-333, and compute_mpc_attention_on_shares,
// crates/v2/server/src/routes/secure_inference_mpc.rs:568-663), followed by the reshare.
//
// Split-K flash decode: CTA (split, head, row) scores its slice of positions (one warp per
// position, lanes over head_dim), forms exp(s - local max) and the weighted V sum, and writes a
// partial (max, sum, acc[head_dim]). The last CTA of a (row, head) to arrive combines the splits in
// split order -- deterministic -- and writes (out - mask, mask).
#include <algorithm>
#include <cmath>
#include <vector>

#include "shd_nonlinear.cuh"

namespace shd {

__global__ void attn_decode_kernel(const AttnArgs a) {
  extern __shared__ float sm[];  // q[head_dim] | scores[chunk_max] | red[34]
  const int hd = a.head_dim;
  const int sp = blockIdx.x, h = blockIdx.y, m = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int chunk_max = (int)((a.kv_seq_stride / a.kvd + a.nsplit - 1) / a.nsplit);
  float* q = sm;
  float* sc = sm + hd;
  float* red = sc + chunk_max;
  __shared__ int last_flag;

  if (tid == 0) pdl_trigger();
  pdl_wait();  // positions, queries and the cache come from earlier kernels
  const int p = a.pos[m];
  const int kv_len = p + 1;
  const int sq = a.seq ? a.seq[m] : 0;
  const int kvh = a.kv_head_of[h];
  const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
  const int t0 = min(sp * chunk, kv_len), t1 = min(t0 + chunk, kv_len);
  const float* K = a.Kcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * hd;
  const float* V = a.Vcache + (size_t)sq * a.kv_seq_stride + (size_t)kvh * hd;
  const bool mpc = a.variant == SHD_NL_MPC;

  for (int d = tid; d < hd; d += blockDim.x) q[d] = a.Q[(size_t)m * a.ldq + (size_t)h * hd + d];
  __syncthreads();

  // scores: one warp per position, lanes stride head_dim; score = (q.k) * scale
  for (int t = t0 + warp; t < t1; t += nw) {
    const float* kr = K + (size_t)t * a.kvd;
    float s = 0.0f;
    for (int d = lane; d < hd; d += 32) s = __fmaf_rn(q[d], kr[d], s);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) sc[t - t0] = __fmul_rn(s, a.scale);
  }
  __syncthreads();

  // local max
  float mx = -INFINITY;
  for (int t = t0 + tid; t < t1; t += blockDim.x) mx = fmaxf(mx, sc[t - t0]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int w = 0; w < nw; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();

  // weights and their sum (fixed tree)
  float l = 0.0f;
  for (int t = t0 + tid; t < t1; t += blockDim.x) {
    float x = __fsub_rn(sc[t - t0], mx);
    if (!mpc) x = fminf(fmaxf(x, -40.0f), 40.0f);
    const float e = expf(x);
    sc[t - t0] = e;
    l = __fadd_rn(l, e);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = 0.0f;
  for (int w = 0; w < nw; ++w) l = __fadd_rn(l, red[w]);

  // weighted V sum, one thread per dimension
  float* part = a.partials + (((size_t)m * a.H + h) * a.nsplit + sp) * (hd + 2);
  for (int d = tid; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int t = t0; t < t1; ++t) acc = __fmaf_rn(sc[t - t0], V[(size_t)t * a.kvd + d], acc);
    part[2 + d] = acc;
  }
  if (tid == 0) {
    part[0] = (t0 < t1) ? mx : -INFINITY;
    part[1] = l;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&a.counters[m * a.H + h], 1);
    last_flag = (old == a.nsplit - 1);
    if (last_flag) a.counters[m * a.H + h] = 0;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();

  const float* base = a.partials + ((size_t)m * a.H + h) * a.nsplit * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, __ldcg(base + (size_t)s * (hd + 2)));
  float L = 0.0f;
  for (int s = 0; s < a.nsplit; ++s) {
    const float ms = __ldcg(base + (size_t)s * (hd + 2));
    if (ms == -INFINITY) continue;
    L = __fadd_rn(L, __fmul_rn(__ldcg(base + (size_t)s * (hd + 2) + 1), expf(__fsub_rn(ms, M))));
  }
  const bool uniform = mpc && !(L > 1e-10f && isfinite(L));
  for (int d = tid; d < hd; d += blockDim.x) {
    float out;
    if (uniform) {
      // compute_mpc_attention_on_shares: 1/seq_len weights when the sum is not usable
      float acc = 0.0f;
      for (int t = 0; t < kv_len; ++t) acc = __fmaf_rn(__fdiv_rn(1.0f, (float)kv_len), V[(size_t)t * a.kvd + d], acc);
      out = acc;
    } else {
      float acc = 0.0f;
      for (int s = 0; s < a.nsplit; ++s) {
        const float ms = __ldcg(base + (size_t)s * (hd + 2));
        if (ms == -INFINITY) continue;
        acc = __fadd_rn(acc, __fmul_rn(__ldcg(base + (size_t)s * (hd + 2) + 2 + d), expf(__fsub_rn(ms, M))));
      }
      out = __fdiv_rn(acc, L);
    }
    const size_t o = (size_t)m * a.ldo + (size_t)h * hd + d;
    const float mk = a.mask ? a.mask[(size_t)m * a.ldmask + (size_t)h * hd + d] : 0.0f;
    a.Oc[o] = __fsub_rn(out, mk);
    a.Os[o] = mk;
  }
}

int ensure_attn_scratch(shd_ctx* ctx, size_t floats);

int launch_attention(shd_ctx* ctx, const AttnArgs& a, int M) {
  const int T = (int)(a.kv_seq_stride / a.kvd);
  const int chunk_max = (T + a.nsplit - 1) / a.nsplit;
  const size_t smem = (size_t)(a.head_dim + chunk_max + 34) * 4;
  if (smem > 200 * 1024) return shd_fail(ctx, SHD_ERR_ARG, "attention: too few splits for this cache length");
  static unsigned attr_devices = 0;
  if (smem > 48 * 1024 && !(attr_devices & (1u << (ctx->device & 31)))) {
    SHD_CHECK_CUDA(ctx, cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_devices |= 1u << (ctx->device & 31);
  }
  const int threads = std::max(64, std::min(256, a.head_dim));
  dim3 grid(a.nsplit, a.H, M);
  SHD_CHECK_CUDA(ctx, launch_pdl(attn_decode_kernel, grid, dim3(threads), smem, ctx->stream, a));
  ctx->launches++;
  return SHD_OK;
}

}  // namespace shd

using namespace shd;

// Scratch for split partials and (row, head) counters, grown outside any stream capture.
int shd::ensure_attn_scratch(shd_ctx* ctx, size_t floats) {
  if (floats <= ctx->attn_part_floats) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  cudaFree(ctx->d_attn_part);
  ctx->d_attn_part = nullptr;
  ctx->attn_part_floats = 0;
  SHD_CHECK_CUDA(ctx, cudaMalloc(&ctx->d_attn_part, floats * 4));
  ctx->attn_part_floats = floats;
  return SHD_OK;
}

// Choose the split count: enough CTAs to cover the SMs twice, chunks of at least 16 positions.
int shd_attn_splits(int num_sms, int H, int M, int max_len) {
  int ns = (2 * num_sms + H * M - 1) / (H * M);
  ns = std::max(1, std::min(ns, 64));
  ns = std::min(ns, std::max(1, (max_len + 15) / 16));
  while ((max_len + ns - 1) / ns > 16384) ++ns;
  return ns;
}

extern "C" int shd_attn_decode(shd_ctx* ctx, const float* q, const float* k_cache,
                               const float* v_cache, int kv_capacity, int H, int Hkv, int head_dim,
                               const int32_t* pos_host, int M, int variant, const float* mask,
                               float* out_c, float* out_s) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, q && k_cache && v_cache && pos_host && out_c && out_s, "shd_attn_decode: null pointer");
  SHD_REQUIRE(ctx, H > 0 && Hkv > 0 && H % Hkv == 0, "shd_attn_decode: num_heads must be a multiple of num_kv_heads");
  SHD_REQUIRE(ctx, head_dim > 0 && head_dim % 32 == 0 && head_dim <= 256, "shd_attn_decode: head_dim must be a multiple of 32, <= 256");
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_attn_decode: unknown variant");
  SHD_REQUIRE(ctx, M > 0 && kv_capacity > 0, "shd_attn_decode: bad shape");
  int maxp = 0;
  for (int i = 0; i < M; ++i) {
    SHD_REQUIRE(ctx, pos_host[i] >= 0 && pos_host[i] < kv_capacity, "shd_attn_decode: position outside the cache");
    maxp = std::max(maxp, (int)pos_host[i]);
  }
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const int ns = shd_attn_splits(ctx->num_sms, H, M, maxp + 1);
  const size_t part = (size_t)M * H * ns * (head_dim + 2);
  int rc = ensure_attn_scratch(ctx, part);
  if (rc) return rc;
  // small per-call staging: positions and the q-head -> kv-head map
  int* d_meta = nullptr;
  SHD_CHECK_CUDA(ctx, cudaMallocAsync(&d_meta, (size_t)(M + H) * 4, ctx->stream));
  std::vector<int> meta(M + H);
  for (int i = 0; i < M; ++i) meta[i] = pos_host[i];
  for (int h = 0; h < H; ++h) meta[M + h] = h / (H / Hkv);
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(d_meta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
  AttnArgs a{};
  a.Q = q;
  a.ldq = H * head_dim;
  a.Kcache = k_cache;
  a.Vcache = v_cache;
  a.kvd = Hkv * head_dim;
  a.kv_seq_stride = (int64_t)kv_capacity * a.kvd;
  a.kv_head_of = d_meta + M;
  a.H = H;
  a.head_dim = head_dim;
  a.pos = d_meta;
  a.seq = nullptr;
  a.variant = variant;
  a.scale = 1.0f / sqrtf((float)head_dim);
  a.mask = mask;
  a.ldmask = H * head_dim;
  a.Oc = out_c;
  a.Os = out_s;
  a.ldo = H * head_dim;
  a.nsplit = ns;
  a.partials = ctx->d_attn_part;
  a.counters = ctx->d_counters + (ctx->n_counters - 8192);
  a.err = ctx->d_err;
  SHD_REQUIRE(ctx, M * H <= 8192, "shd_attn_decode: too many (row, head) pairs");
  rc = launch_attention(ctx, a, M);
  cudaFreeAsync(d_meta, ctx->stream);
  // the host vector must outlive the async copy
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return shd_cuda_fail(ctx, e, "shd_attn_decode");
  return rc;
}
