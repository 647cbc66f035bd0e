// Client-side encoding and seeded share generation of the v1 ring path, and the session-keyed
// embedding shares of get_embeddings_direct, on the device.
//
//  * Fixed::from_f64 / FixedVector::from_f64_slice (crates/fixed_point/src/fixed.rs:30-49,
//    vector.rs:22-29): raw = round(v * 2^scale), half away from zero; values beyond i32 are an
//    Overflow / Underflow error for the first such element; NaN encodes as 0 (Rust's saturating
//    `f64 as i32`).
//  * Share::random_seeded / SharePair::from_plaintext_seeded (crates/sharing/src/share.rs:44-54,
//    116-135): server share = ChaCha20Rng::seed_from_u64(seed).next_u32() as i32, in order;
//    client share = x wrapping_sub server.
//  * get_embeddings_direct (crates/v2/server/src/routes/secure_inference.rs:387-460): one
//    ChaCha20Rng::from_seed(session id || 16 zero bytes) per request; token t's element k takes
//    keystream word t * hidden + k; s = (word >> 8) * 2^-24 (rand 0.8.5 Standard f32), c = e - s.
//
// ChaCha20Rng (rand_chacha 0.3.1) is the ChaCha20 block function of D. J. Bernstein ("ChaCha, a
// variant of Salsa20", 2008) keyed by the 32-byte seed, 64-bit block counter in state words 12-13
// from 0, stream id 0 in words 14-15, next_u32 = the keystream's little-endian words in order.
// Counter-based: one thread computes one 64-byte block (16 words) independently.
// seed_from_u64 (rand_core 0.6.4) fills the seed with eight PCG32 (XSH-RR) outputs, each taken
// after advancing the state; it runs on the host.
#include <cmath>
#include <cstring>
#include <string>

#include "shd_common.cuh"

namespace {

struct ChaChaKey {
  uint32_t w[8];
};

__device__ __forceinline__ uint32_t rotl(uint32_t v, int c) { return __funnelshift_l(v, v, c); }

__device__ __forceinline__ void quarter(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  a += b; d = rotl(d ^ a, 16);
  c += d; b = rotl(b ^ c, 12);
  a += b; d = rotl(d ^ a, 8);
  c += d; b = rotl(b ^ c, 7);
}

// Keystream block `blk` (stream 0) into out[16].
__device__ __forceinline__ void chacha20_block(const ChaChaKey& k, uint64_t blk, uint32_t out[16]) {
  uint32_t x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    k.w[0], k.w[1], k.w[2], k.w[3], k.w[4], k.w[5], k.w[6], k.w[7],
                    (uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = x[i];
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    quarter(x[0], x[4], x[8], x[12]);
    quarter(x[1], x[5], x[9], x[13]);
    quarter(x[2], x[6], x[10], x[14]);
    quarter(x[3], x[7], x[11], x[15]);
    quarter(x[0], x[5], x[10], x[15]);
    quarter(x[1], x[6], x[11], x[12]);
    quarter(x[2], x[7], x[8], x[13]);
    quarter(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] += x[i];
}

ChaChaKey key_from_bytes(const uint8_t b[32]) {
  ChaChaKey k;
  for (int i = 0; i < 8; ++i)
    k.w[i] = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) | ((uint32_t)b[4 * i + 2] << 16) |
             ((uint32_t)b[4 * i + 3] << 24);
  return k;
}

// rand_core 0.6.4 SeedableRng::seed_from_u64: eight PCG32 outputs, state advanced before each.
void seed_from_u64(uint64_t state, uint8_t seed[32]) {
  const uint64_t MUL = 6364136223846793005ull, INC = 11634580027462260723ull;
  for (int c = 0; c < 8; ++c) {
    state = state * MUL + INC;
    const uint32_t xorshifted = (uint32_t)(((state >> 18) ^ state) >> 27);
    const uint32_t rot = (uint32_t)(state >> 59);
    const uint32_t x = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
    for (int b = 0; b < 4; ++b) seed[4 * c + b] = (uint8_t)(x >> (8 * b));
  }
}

int grid_blocks(int64_t items, int threads) {
  const int64_t g = (items + threads - 1) / threads;
  return (int)(g < 1 ? 1 : (g > (1 << 30) ? (1 << 30) : g));
}

// One thread per 16-element block of the share vector.
__global__ void ring_share_kernel(const int32_t* __restrict__ x, int64_t n, ChaChaKey key,
                                  int32_t* __restrict__ xc, int32_t* __restrict__ xs) {
  const int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t i0 = blk * 16;
  if (i0 >= n) return;
  uint32_t w[16];
  chacha20_block(key, (uint64_t)blk, w);
  if (i0 + 16 <= n && (((uintptr_t)(x + i0) | (uintptr_t)(xc + i0) | (uintptr_t)(xs + i0)) & 15u) == 0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int4 xv = reinterpret_cast<const int4*>(x + i0)[v];
      int4 s, c;
      s.x = (int)w[4 * v]; s.y = (int)w[4 * v + 1]; s.z = (int)w[4 * v + 2]; s.w = (int)w[4 * v + 3];
      c.x = (int)((uint32_t)xv.x - w[4 * v]);
      c.y = (int)((uint32_t)xv.y - w[4 * v + 1]);
      c.z = (int)((uint32_t)xv.z - w[4 * v + 2]);
      c.w = (int)((uint32_t)xv.w - w[4 * v + 3]);
      reinterpret_cast<int4*>(xs + i0)[v] = s;
      reinterpret_cast<int4*>(xc + i0)[v] = c;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (i0 + j < n) {
      xs[i0 + j] = (int32_t)w[j];
      xc[i0 + j] = (int32_t)((uint32_t)x[i0 + j] - w[j]);
    }
}

// Fixed::from_f64 per element; the first failing element (lowest index) is recorded as
// index * 4 + kind (1 overflow, 2 underflow) with an atomic minimum.
__global__ void fixed_encode_kernel(const double* __restrict__ x, int64_t n, double factor,
                                    int32_t* __restrict__ out, unsigned long long* first_err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double scaled = x[i] * factor;  // power of two: exact
    int kind = 0;
    if (scaled > 2147483647.0) kind = 1;
    else if (scaled < -2147483648.0) kind = 2;
    if (kind) {
      atomicMin(first_err, (unsigned long long)i * 4ull + (unsigned long long)kind);
      out[i] = 0;
    } else {
      out[i] = isnan(scaled) ? 0 : (int32_t)round(scaled);  // round: half away from zero
    }
  }
}

// get_embeddings_direct: one thread per 16 keystream words of the request's token x hidden stream.
__global__ void embed_session_kernel(const uint16_t* __restrict__ table, int vocab, int hidden,
                                     const int32_t* __restrict__ tokens, int n_tokens, ChaChaKey key,
                                     float* __restrict__ hc, float* __restrict__ hs, int* err) {
  const int64_t total = (int64_t)n_tokens * hidden;
  const int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t i0 = blk * 16;
  if (i0 >= total) return;
  uint32_t w[16];
  chacha20_block(key, (uint64_t)blk, w);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int64_t i = i0 + j;
    if (i >= total) break;
    const int t = (int)(i / hidden), k = (int)(i % hidden);
    const int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
      atomicOr(err, SHD_DEVERR_ARG);
      continue;
    }
    const float s = (float)(w[j] >> 8) * 5.9604644775390625e-08f;  // exact: 24-bit integer * 2^-24
    const float e = __uint_as_float((uint32_t)table[(size_t)tok * hidden + k] << 16);
    hs[i] = s;
    hc[i] = __fsub_rn(e, s);
  }
}

}  // namespace

extern "C" int shd_fixed_from_f64(shd_ctx* ctx, const double* x, int64_t n, int scale, int32_t* out) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_fixed_from_f64: n < 0");
  SHD_REQUIRE(ctx, scale >= 0 && scale <= 30, "shd_fixed_from_f64: InvalidScale (scale must be 0..30)");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, x && out, "shd_fixed_from_f64: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  if (!ctx->d_scratch64) SHD_CHECK_CUDA(ctx, cudaMalloc(&ctx->d_scratch64, 8));
  SHD_CHECK_CUDA(ctx, cudaMemsetAsync(ctx->d_scratch64, 0xff, 8, ctx->stream));
  const int threads = 256;
  int grid = grid_blocks(n, threads);
  if (grid > ctx->num_sms * 8) grid = ctx->num_sms * 8;
  fixed_encode_kernel<<<grid, threads, 0, ctx->stream>>>(x, n, (double)(1ull << scale), out,
                                                          ctx->d_scratch64);
  SHD_CHECK_LAUNCH(ctx, "fixed_encode_kernel");
  unsigned long long first = 0;
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(&first, ctx->d_scratch64, 8, cudaMemcpyDeviceToHost, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (first != ~0ull) {
    const int64_t idx = (int64_t)(first >> 2);
    double v = 0.0;
    SHD_CHECK_CUDA(ctx, cudaMemcpy(&v, x + idx, 8, cudaMemcpyDeviceToHost));
    char buf[160];
    snprintf(buf, sizeof(buf), "shd_fixed_from_f64: %s { value: %.17g } at element %lld",
             (first & 3) == 1 ? "Overflow" : "Underflow", v, (long long)idx);
    return shd_fail(ctx, SHD_ERR_ARG, buf);
  }
  return SHD_OK;
}

extern "C" int shd_ring_share_seeded(shd_ctx* ctx, const int32_t* x, int64_t n, uint64_t seed,
                                     int32_t* xc, int32_t* xs) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_ring_share_seeded: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, x && xc && xs, "shd_ring_share_seeded: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  uint8_t s[32];
  seed_from_u64(seed, s);
  const int64_t blocks = (n + 15) / 16;
  ring_share_kernel<<<grid_blocks(blocks, 128), 128, 0, ctx->stream>>>(x, n, key_from_bytes(s), xc, xs);
  SHD_CHECK_LAUNCH(ctx, "ring_share_kernel");
  return SHD_OK;
}

extern "C" int shd_embed_shares_session(shd_ctx* ctx, const uint16_t* table, int vocab, int hidden,
                                        const int32_t* tokens, int n_tokens, const uint8_t* session_id16,
                                        float* hc, float* hs) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n_tokens >= 0 && hidden > 0 && vocab > 0, "shd_embed_shares_session: bad sizes");
  if (n_tokens == 0) return SHD_OK;
  SHD_REQUIRE(ctx, table && tokens && session_id16 && hc && hs, "shd_embed_shares_session: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  uint8_t s[32] = {};
  std::memcpy(s, session_id16, 16);
  const int64_t blocks = ((int64_t)n_tokens * hidden + 15) / 16;
  embed_session_kernel<<<grid_blocks(blocks, 128), 128, 0, ctx->stream>>>(
      table, vocab, hidden, tokens, n_tokens, key_from_bytes(s), hc, hs, ctx->d_err);
  SHD_CHECK_LAUNCH(ctx, "embed_session_kernel");
  return SHD_OK;
}
