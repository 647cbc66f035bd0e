// Reconstruct-compute-reshare kernels (RMSNorm, SwiGLU, SiLU), share-wise RoPE, embedding share
// generation and the client's greedy argmax. Block reductions use a fixed tree, so results do not
// depend on scheduling.
#include <cmath>
#include <vector>

#include "shd_nonlinear.cuh"

namespace shd {

// ---- block-wide deterministic sum (blockDim.x multiple of 32, <= 1024) ----
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // red may still be read from a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < nw ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) w = __fadd_rn(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) red[32] = w;
  }
  __syncthreads();
  return red[32];
}

// One CTA per token row. h = H (+ D) per share (residual add, written to Hout when given), then
// x = h_c + h_s, y = x * inv_rms * gamma, reshare (y - mask, mask).
__global__ void norm_reshare_kernel(NormArgs a) {
  __shared__ float red[33];
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const float* hc = a.Hc + (size_t)m * a.ldh;
  const float* hs = a.Hs + (size_t)m * a.ldh;
  const float* dc = a.Dc ? a.Dc + (size_t)m * a.ldh : nullptr;
  const float* ds = a.Ds ? a.Ds + (size_t)m * a.ldh : nullptr;
  float* oc = a.Hout_c ? a.Hout_c + (size_t)m * a.ldh : nullptr;
  float* os = a.Hout_s ? a.Hout_s + (size_t)m * a.ldh : nullptr;
  float sq = 0.0f;
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    float c = hc[i], s = hs[i];
    if (dc) {
      // residual: sublayer output + residual stream (o + h, down + h), per share
      c = __fadd_rn(dc[i], c);
      s = __fadd_rn(ds[i], s);
      if (oc) {
        oc[i] = c;
        os[i] = s;
      }
    }
    const float x = __fadd_rn(c, s);
    sq = __fmaf_rn(x, x, sq);
  }
  const float sum_sq = block_sum(sq, red);
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
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    float c = hc[i], s = hs[i];
    if (dc) {
      c = __fadd_rn(dc[i], c);
      s = __fadd_rn(ds[i], s);
    }
    const float x = __fadd_rn(c, s);
    float r = __fmul_rn(__fmul_rn(x, inv), a.gamma[i]);
    if (a.variant == SHD_NL_MPC && !isfinite(r)) r = 0.0f;
    const float mv = mk ? mk[i] : 0.0f;
    xc[i] = __fsub_rn(r, mv);
    xs[i] = mv;
  }
}

int launch_norm(shd_ctx* ctx, const NormArgs& a, int M) {
  const int threads = a.n >= 4096 ? 1024 : (a.n >= 1024 ? 512 : 128);
  SHD_CHECK_CUDA(ctx, launch_pdl(norm_reshare_kernel, dim3(M), dim3(threads), 0, ctx->stream, a));
  ctx->launches++;
  return SHD_OK;
}

__device__ __forceinline__ float silu_v(float g, int variant) {
  if (variant == SHD_NL_APPROX) {
    const float gc = fminf(fmaxf(g, -20.0f), 20.0f);
    return __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gc))));
  } else if (variant == SHD_NL_GPU) {
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  }
  if (!isfinite(g)) return 0.0f;
  return __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
}

__global__ void swiglu_reshare_kernel(const float* gc, const float* gs, const float* uc,
                                      const float* us, int variant, const float* mask, float* yc,
                                      float* ys, long long n, int silu_only) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float g = __fadd_rn(gc[i], gs[i]);
    float r = silu_v(g, variant);
    if (!silu_only) {
      const float u = __fadd_rn(uc[i], us[i]);
      if (variant == SHD_NL_MPC) {
        if (!(isfinite(r) && isfinite(u))) {
          r = 0.0f;
        } else {
          r = __fmul_rn(r, u);
          if (!isfinite(r)) r = 0.0f;
        }
      } else {
        r = __fmul_rn(r, u);
      }
    }
    const float mv = mask ? mask[i] : 0.0f;
    yc[i] = __fsub_rn(r, mv);
    ys[i] = mv;
  }
}

// In-place RoPE on both shares of [M][n_heads * head_dim] rows at positions pos[m].
__global__ void rope_shares_kernel(float* xc, float* xs, int M, int n_heads, int head_dim,
                                   const int* pos, int pos_scalar, const float* cos_t,
                                   const float* sin_t, int max_seq, int* err) {
  const int half = head_dim / 2;
  const long long n = (long long)M * n_heads * half;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < n;
       v += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(v % half);
    const long long hm = v / half;
    const int h = (int)(hm % n_heads), m = (int)(hm / n_heads);
    const int p = pos ? pos[m] : pos_scalar + m;
    if (p < 0 || p >= max_seq) {
      atomicOr(err, SHD_DEVERR_ARG);
      continue;
    }
    const float c = cos_t[(size_t)p * half + i], s = sin_t[(size_t)p * half + i];
    const size_t o = ((size_t)m * n_heads + h) * head_dim + i;
    const float x0c = xc[o], x1c = xc[o + half], x0s = xs[o], x1s = xs[o + half];
    xc[o] = __fsub_rn(__fmul_rn(x0c, c), __fmul_rn(x1c, s));
    xc[o + half] = __fadd_rn(__fmul_rn(x0c, s), __fmul_rn(x1c, c));
    xs[o] = __fsub_rn(__fmul_rn(x0s, c), __fmul_rn(x1s, s));
    xs[o + half] = __fadd_rn(__fmul_rn(x0s, s), __fmul_rn(x1s, c));
  }
}

// Embedding shares: server share s_k = unit(word(seed, 7, counter * hidden + k)), client e - s.
// Also (optionally) zeroes the sublayer-output rows D and resets the argmax keys for a new step.
__global__ void embed_shares_kernel(EmbedArgs a) {
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();  // tokens and positions come from the previous step
  const int m = blockIdx.y;
  const int tok = a.tokens[m];
  if (tok < 0 || tok >= a.vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, SHD_DEVERR_ARG);
    return;
  }
  const uint64_t counter = (a.slot_counter ? ((uint64_t)m << 32) : a.counter_base) +
                           (uint64_t)(a.pos ? a.pos[m] : m);
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < a.hidden; k += gridDim.x * blockDim.x) {
    const float e = __uint_as_float((uint32_t)a.table[(size_t)tok * a.hidden + k] << 16);
    const float s = u32_to_unit_f32(philox_word(a.seed, 7, counter * (uint64_t)a.hidden + (uint64_t)k));
    a.Hc[(size_t)m * a.ldh + k] = __fsub_rn(e, s);
    a.Hs[(size_t)m * a.ldh + k] = s;
    if (a.Dc) {
      a.Dc[(size_t)m * a.ldh + k] = 0.0f;
      a.Ds[(size_t)m * a.ldh + k] = 0.0f;
    }
  }
  if (a.amax && blockIdx.x == 0 && threadIdx.x == 0) a.amax[m] = 0ull;
}

int launch_embed(shd_ctx* ctx, const EmbedArgs& a, int M) {
  dim3 grid((a.hidden + 255) / 256, M);
  SHD_CHECK_CUDA(ctx, launch_pdl(embed_shares_kernel, grid, dim3(256), 0, ctx->stream, a));
  ctx->launches++;
  return SHD_OK;
}

__device__ __forceinline__ unsigned long long amax_key(float v, int idx) {
  if (v == 0.0f) v = 0.0f;
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned)idx;
}

// Greedy sample of reconstructed logits: one CTA per row; last index among equal maxima.
__global__ void argmax_kernel(const float* lc, const float* ls, int V, int ld, int* out, int* err) {
  __shared__ unsigned long long red[32];
  const int m = blockIdx.x;
  unsigned long long best = 0ull;
  bool nan = false;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = __fadd_rn(lc[(size_t)m * ld + i], ls[(size_t)m * ld + i]);
    nan |= isnan(v);
    const unsigned long long k = amax_key(v, i);
    best = k > best ? k : best;
  }
  if (__any_sync(0xffffffffu, nan) && (threadIdx.x & 31) == 0) atomicOr(err, SHD_DEVERR_NONFINITE);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
      b = t > b ? t : b;
    }
    if (threadIdx.x == 0) out[m] = (int)(b & 0xffffffffu);
  }
}

__global__ void keys_to_tokens_kernel(const unsigned long long* keys, int* tokens, int M) {
  const int m = threadIdx.x;
  if (m < M) tokens[m] = (int)(keys[m] & 0xffffffffu);
}

int launch_keys_to_tokens(shd_ctx* ctx, const unsigned long long* keys, int* tokens, int M) {
  keys_to_tokens_kernel<<<1, 32, 0, ctx->stream>>>(keys, tokens, M);
  SHD_CHECK_LAUNCH(ctx, "keys_to_tokens_kernel");
  return SHD_OK;
}

}  // namespace shd

using namespace shd;

static int ew_grid(shd_ctx* ctx, long long n) {
  long long g = (n + 255) / 256;
  if (g > (long long)ctx->num_sms * 8) g = (long long)ctx->num_sms * 8;
  return (int)(g < 1 ? 1 : g);
}

// RopeFrequencies::new (crates/v2/sharing/src/secure_attention.rs:42-63) on the host with libm's
// powf/cosf/sinf, exactly as the reference computes its table, then uploaded.
int shd::build_rope_table(shd_ctx* ctx, int head_dim, int max_seq, float theta, float** cos_out,
                          float** sin_out) {
  const int half = head_dim / 2;
  std::vector<float> inv(half), c((size_t)max_seq * half), s((size_t)max_seq * half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < half; ++i) {
      c[(size_t)p * half + i] = cosf((float)p * inv[i]);
      s[(size_t)p * half + i] = sinf((float)p * inv[i]);
    }
  float *dc = nullptr, *ds = nullptr;
  cudaError_t e = cudaMalloc(&dc, c.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ds, s.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(dc, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(ds, s.data(), s.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(dc);
    cudaFree(ds);
    return shd_cuda_fail(ctx, e, "RoPE table");
  }
  *cos_out = dc;
  *sin_out = ds;
  return SHD_OK;
}

// The context's table serves shd_rope_shares; it is replaced on every call.
int shd::shd_build_rope(shd_ctx* ctx, int head_dim, int max_seq, float theta) {
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  cudaFree(ctx->d_rope_cos);
  cudaFree(ctx->d_rope_sin);
  ctx->d_rope_cos = ctx->d_rope_sin = nullptr;
  ctx->rope_head_dim = ctx->rope_max_seq = 0;
  const int rc = build_rope_table(ctx, head_dim, max_seq, theta, &ctx->d_rope_cos, &ctx->d_rope_sin);
  if (rc) return rc;
  ctx->rope_head_dim = head_dim;
  ctx->rope_max_seq = max_seq;
  ctx->rope_theta = theta;
  return SHD_OK;
}

extern "C" int shd_rope_init(shd_ctx* ctx, int head_dim, int max_seq, float theta) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, head_dim > 0 && head_dim % 2 == 0, "shd_rope_init: head_dim must be even");
  SHD_REQUIRE(ctx, max_seq > 0, "shd_rope_init: max_seq <= 0");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  return shd_build_rope(ctx, head_dim, max_seq, theta);
}

extern "C" int shd_rope_shares(shd_ctx* ctx, float* xc, float* xs, int M, int n_heads, int head_dim,
                               int pos) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, xc && xs, "shd_rope_shares: null share");
  SHD_REQUIRE(ctx, ctx->d_rope_cos && ctx->rope_head_dim == head_dim,
              "shd_rope_shares: call shd_rope_init with this head_dim first");
  SHD_REQUIRE(ctx, pos >= 0 && pos + M <= ctx->rope_max_seq,
              "shd_rope_shares: position exceeds max_seq_len of the RoPE table");
  if (M <= 0) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const long long n = (long long)M * n_heads * (head_dim / 2);
  rope_shares_kernel<<<ew_grid(ctx, n), 256, 0, ctx->stream>>>(
      xc, xs, M, n_heads, head_dim, nullptr, pos, ctx->d_rope_cos, ctx->d_rope_sin, ctx->rope_max_seq,
      ctx->d_err);
  SHD_CHECK_LAUNCH(ctx, "rope_shares_kernel");
  return SHD_OK;
}

extern "C" int shd_rmsnorm_reshare(shd_ctx* ctx, const float* xc, const float* xs, const float* gamma,
                                   float eps, int variant, const float* mask, float* yc, float* ys,
                                   int M, int n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_rmsnorm_reshare: unknown variant");
  SHD_REQUIRE(ctx, n > 0 && M >= 0, "shd_rmsnorm_reshare: bad shape");
  if (M == 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && gamma && yc && ys, "shd_rmsnorm_reshare: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  NormArgs a{};
  a.Hc = xc;
  a.Hs = xs;
  a.ldh = n;
  a.gamma = gamma;
  a.eps = eps;
  a.variant = variant;
  a.mask = mask;
  a.ldmask = n;
  a.Xc = yc;
  a.Xs = ys;
  a.ldx = n;
  a.n = n;
  return launch_norm(ctx, a, M);
}

extern "C" int shd_swiglu_reshare(shd_ctx* ctx, const float* gc, const float* gs, const float* uc,
                                  const float* us, int variant, const float* mask, float* yc,
                                  float* ys, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_swiglu_reshare: unknown variant");
  if (n <= 0) return SHD_OK;
  SHD_REQUIRE(ctx, gc && gs && uc && us && yc && ys, "shd_swiglu_reshare: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  swiglu_reshare_kernel<<<ew_grid(ctx, n), 256, 0, ctx->stream>>>(gc, gs, uc, us, variant, mask, yc, ys, n, 0);
  SHD_CHECK_LAUNCH(ctx, "swiglu_reshare_kernel");
  return SHD_OK;
}

extern "C" int shd_silu_reshare(shd_ctx* ctx, const float* xc, const float* xs, int variant,
                                const float* mask, float* yc, float* ys, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, variant >= 0 && variant <= 2, "shd_silu_reshare: unknown variant");
  if (n <= 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && yc && ys, "shd_silu_reshare: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  swiglu_reshare_kernel<<<ew_grid(ctx, n), 256, 0, ctx->stream>>>(xc, xs, nullptr, nullptr, variant, mask, yc, ys, n, 1);
  SHD_CHECK_LAUNCH(ctx, "swiglu_reshare_kernel");
  return SHD_OK;
}

extern "C" int shd_embed_shares(shd_ctx* ctx, const uint16_t* table, int vocab, int hidden,
                                const int32_t* tokens, int M, uint64_t seed, uint64_t counter,
                                float* hc, float* hs) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, table && tokens && hc && hs, "shd_embed_shares: null pointer");
  SHD_REQUIRE(ctx, vocab > 0 && hidden > 0 && M >= 0, "shd_embed_shares: bad shape");
  if (M == 0) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  EmbedArgs a{};
  a.table = table;
  a.vocab = vocab;
  a.hidden = hidden;
  a.tokens = tokens;
  a.seed = seed;
  a.counter_base = counter;
  a.Hc = hc;
  a.Hs = hs;
  a.ldh = hidden;
  a.err = ctx->d_err;
  return launch_embed(ctx, a, M);
}

extern "C" int shd_argmax_reconstruct(shd_ctx* ctx, const float* lc, const float* ls, int V, int M,
                                      int32_t* tokens) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, lc && ls && tokens && V > 0 && M >= 0, "shd_argmax_reconstruct: bad argument");
  if (M == 0) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  argmax_kernel<<<M, 1024, 0, ctx->stream>>>(lc, ls, V, V, tokens, ctx->d_err);
  SHD_CHECK_LAUNCH(ctx, "argmax_kernel");
  return SHD_OK;
}
