// ORACLE -- test infrastructure only. A CPU restatement of the ShardLM reference's share arithmetic
// (Rust, crates/v2 and crates/{fixed_point,sharing}), used by tests/, by __graft_entry__.smoke()
// as the checker, and by bench.py's cpu_baseline leg / --impl reference arm as the timed CPU
// path. The product (libshardlm_cuda.so) never links or calls this code.
//
// Parity pinning: the reference is Rust and no Rust toolchain exists here, so it cannot be run.
// This restatement is pinned against the reference's own known-answer tests, restated in
// tests/test_oracle_golden.py from tests/golden/reference_known_answers.json.
//
// Build: g++ -O2 -std=c++17 -ffp-contract=off -fno-fast-math -pthread -shared -fPIC.
// Rust neither contracts a*b+c into an FMA nor reassociates float sums; neither does this file.
// f32::exp / sqrt / powf / sin / cos on Linux are the libm calls used here.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <thread>

#define ORC_API extern "C" __attribute__((visibility("default")))

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

static int g_threads = 1;
ORC_API void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
ORC_API int orc_max_threads() {
  const unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

// Run fn(tid, nth) on g_threads threads (the calling thread is tid 0).
template <typename F>
static void parallel_run(F fn) {
  const int nth = g_threads;
  if (nth <= 1) {
    fn(0, 1);
    return;
  }
  std::vector<std::thread> ts;
  ts.reserve(nth - 1);
  for (int t = 1; t < nth; ++t) ts.emplace_back(fn, t, nth);
  fn(0, nth);
  for (auto& t : ts) t.join();
}

// ------------------------------------------------------------------------------------------------
// f32 share-wise linear: SecureLinear::matmul + forward_secure
// (crates/v2/sharing/src/secure_linear.rs:57-117). out[j] += x_i * W[i*out + j] with i outer,
// each share on its own; bias added to the server share only. Weights [in][out]; values are exact
// bf16 upcasts (crates/v2/server/src/secure_weights.rs:432-440), so a bf16 [in][out] array gives
// identical results. Columns are split over threads; each column's summation order is unchanged.
// ------------------------------------------------------------------------------------------------
template <typename WT>
static void linear_core(const WT* w, const float* bias, int in, int out, const float* xc,
                        const float* xs, float* yc, float* ys, int M) {
  parallel_run([&](int tid, int nth) {
    const int per = ((out + nth - 1) / nth + 15) / 16 * 16;
    const int j0 = tid * per, j1 = (j0 + per < out) ? j0 + per : out;
    if (j0 < j1) {
      const int nj = j1 - j0;
      std::vector<float> acc((size_t)2 * M * nj, 0.0f);
      for (int i = 0; i < in; ++i) {
        const WT* row = w + (size_t)i * out + j0;
        for (int m = 0; m < M; ++m) {
          const float xi_c = xc[(size_t)m * in + i];
          const float xi_s = xs[(size_t)m * in + i];
          float* ac = acc.data() + (size_t)(2 * m) * nj;
          float* as = ac + nj;
          for (int j = 0; j < nj; ++j) {
            float wv;
            if constexpr (sizeof(WT) == 2) wv = bf16_to_f32(row[j]);
            else wv = row[j];
            ac[j] += xi_c * wv;
            as[j] += xi_s * wv;
          }
        }
      }
      for (int m = 0; m < M; ++m)
        for (int j = 0; j < nj; ++j) {
          float c = acc[(size_t)(2 * m) * nj + j];
          float s = acc[(size_t)(2 * m + 1) * nj + j];
          if (bias) s += bias[j0 + j];
          yc[(size_t)m * out + j0 + j] = c;
          ys[(size_t)m * out + j0 + j] = s;
        }
    }
  });
}

ORC_API void orc_linear_f32(const float* w_in_out, const float* bias, int in, int out,
                            const float* xc, const float* xs, float* yc, float* ys, int M) {
  linear_core<float>(w_in_out, bias, in, out, xc, xs, yc, ys, M);
}

ORC_API void orc_linear_bf16(const uint16_t* w_in_out, const float* bias, int in, int out,
                             const float* xc, const float* xs, float* yc, float* ys, int M) {
  linear_core<uint16_t>(w_in_out, bias, in, out, xc, xs, yc, ys, M);
}

// Sum_i |x_i| |W_ij| per output, in f64: the scale of the rounding error of any summation order.
ORC_API void orc_linear_abs_bf16(const uint16_t* w_in_out, int in, int out, const float* x,
                                 double* y) {
  for (int j = 0; j < out; ++j) y[j] = 0.0;
  for (int i = 0; i < in; ++i) {
    const double xi = std::fabs((double)x[i]);
    const uint16_t* row = w_in_out + (size_t)i * out;
    for (int j = 0; j < out; ++j) y[j] += xi * std::fabs((double)bf16_to_f32(row[j]));
  }
}

// ------------------------------------------------------------------------------------------------
// v1 ring linear: LinearServer::multiply_vector + handle_request (crates/sharing/src/linear.rs:
// 230-274). acc_j = sum_i (i64)x_i * (i64)W_ij (wrapping, i outer), y_j = (i32)(acc_j >> scale),
// server share += bias (wrapping).
// ------------------------------------------------------------------------------------------------
ORC_API void orc_linear_ring(const int32_t* w_in_out, const int32_t* bias, int in, int out,
                             const int32_t* xc, const int32_t* xs, int32_t* yc, int32_t* ys, int M,
                             int scale) {
  std::vector<uint64_t> ac(out), as(out);
  for (int m = 0; m < M; ++m) {
    std::fill(ac.begin(), ac.end(), 0);
    std::fill(as.begin(), as.end(), 0);
    for (int i = 0; i < in; ++i) {
      const int64_t xi_c = xc[(size_t)m * in + i], xi_s = xs[(size_t)m * in + i];
      const int32_t* row = w_in_out + (size_t)i * out;
      for (int j = 0; j < out; ++j) {
        ac[j] += (uint64_t)(xi_c * (int64_t)row[j]);
        as[j] += (uint64_t)(xi_s * (int64_t)row[j]);
      }
    }
    for (int j = 0; j < out; ++j) {
      yc[(size_t)m * out + j] = (int32_t)((int64_t)ac[j] >> scale);
      int32_t s = (int32_t)((int64_t)as[j] >> scale);
      if (bias) s = (int32_t)((uint32_t)s + (uint32_t)bias[j]);
      ys[(size_t)m * out + j] = s;
    }
  }
}

// plaintext_linear (crates/sharing/src/linear.rs:323-363): the same on the reconstructed input.
ORC_API void orc_plaintext_linear_ring(const int32_t* w_in_out, const int32_t* bias, int in, int out,
                                       const int32_t* x, int32_t* y, int scale) {
  std::vector<uint64_t> acc(out, 0);
  for (int i = 0; i < in; ++i) {
    const int64_t xi = x[i];
    for (int j = 0; j < out; ++j) acc[j] += (uint64_t)(xi * (int64_t)w_in_out[(size_t)i * out + j]);
  }
  for (int j = 0; j < out; ++j) {
    int32_t r = (int32_t)((int64_t)acc[j] >> scale);
    if (bias) r = (int32_t)((uint32_t)r + (uint32_t)bias[j]);
    y[j] = r;
  }
}

// Fixed::from_f64 (crates/fixed_point/src/fixed.rs:30-49): round(v * 2^scale) with round half away
// from zero; returns 0 ok, 1 overflow, 2 underflow, 3 invalid scale.
ORC_API int orc_fixed_from_f64(double v, int scale, int32_t* out) {
  if (scale > 30) return 3;
  const double scaled = v * (double)(1ull << scale);
  if (scaled > 2147483647.0) return 1;
  if (scaled < -2147483648.0) return 2;
  // Rust's `f64 as i32` saturates and maps NaN to 0
  *out = std::isnan(scaled) ? 0 : (int32_t)std::round(scaled);
  return 0;
}

// Fixed::mul (fixed.rs:109-132): (i64 a * i64 b) >> scale, overflow -> status 1.
ORC_API int orc_fixed_mul(int32_t a, int32_t b, int scale, int32_t* out) {
  const int64_t r = ((int64_t)a * (int64_t)b) >> scale;
  if (r > 2147483647LL || r < -2147483648LL) return 1;
  *out = (int32_t)r;
  return 0;
}

// ------------------------------------------------------------------------------------------------
// Beaver multiply, f32: secure_multiply_mpc (crates/v2/sharing/src/beaver.rs:167-197).
// ------------------------------------------------------------------------------------------------
ORC_API void orc_beaver_f32(const float* xc, const float* xs, const float* yc, const float* ys,
                            const float* ac, const float* as, const float* bc, const float* bs,
                            const float* cc, const float* cs, float* d_out, float* e_out, float* zc,
                            float* zs, int64_t n) {
  parallel_run([&](int tid, int nth) {
  const int64_t i0 = n * tid / nth, i1 = n * (tid + 1) / nth;
  for (int64_t i = i0; i < i1; ++i) {
    const float d_client = xc[i] - ac[i];
    const float d_server = xs[i] - as[i];
    const float e_client = yc[i] - bc[i];
    const float e_server = ys[i] - bs[i];
    const float d = d_client + d_server;
    const float e = e_client + e_server;
    zc[i] = cc[i] + ac[i] * e + d * bc[i] + d * e;
    zs[i] = cs[i] + as[i] * e + d * bs[i];
    if (d_out) d_out[i] = d;
    if (e_out) e_out[i] = e;
  }
  });
}

// Z_2^32 Beaver with Fixed's wrapping add/sub and wrapping multiply; optional SecureML truncation.
ORC_API void orc_beaver_ring(const uint32_t* xc, const uint32_t* xs, const uint32_t* yc,
                             const uint32_t* ys, const uint32_t* ac, const uint32_t* as,
                             const uint32_t* bc, const uint32_t* bs, const uint32_t* cc,
                             const uint32_t* cs, uint32_t* d_out, uint32_t* e_out, uint32_t* zc,
                             uint32_t* zs, int64_t n, int f) {
  parallel_run([&](int tid, int nth) {
  const int64_t i0 = n * tid / nth, i1 = n * (tid + 1) / nth;
  for (int64_t i = i0; i < i1; ++i) {
    const uint32_t d = (xc[i] - ac[i]) + (xs[i] - as[i]);
    const uint32_t e = (yc[i] - bc[i]) + (ys[i] - bs[i]);
    uint32_t z0 = cc[i] + ac[i] * e + d * bc[i] + d * e;
    uint32_t z1 = cs[i] + as[i] * e + d * bs[i];
    if (f > 0) {
      z0 = (uint32_t)((int32_t)z0 >> f);
      z1 = 0u - (uint32_t)((int32_t)(0u - z1) >> f);
    }
    zc[i] = z0;
    zs[i] = z1;
    if (d_out) d_out[i] = d;
    if (e_out) e_out[i] = e;
  }
  });
}

// ------------------------------------------------------------------------------------------------
// Counter-based generator (Philox4x32-10, Salmon et al. SC'11) -- the same construction the
// library uses for shares, masks and triples, so both sides see identical inputs.
// ------------------------------------------------------------------------------------------------
static inline void philox(uint64_t block, uint64_t stream, uint64_t seed, uint32_t out[4]) {
  uint32_t c0 = (uint32_t)block, c1 = (uint32_t)(block >> 32);
  uint32_t c2 = (uint32_t)stream, c3 = (uint32_t)(stream >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static inline uint32_t philox_word(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint32_t o[4];
  philox(idx >> 2, stream, seed, o);
  return o[idx & 3];
}

static inline float unit_f32(uint32_t u) { return (float)(u >> 8) * 5.9604644775390625e-08f; }
static inline float uniform_f32(uint32_t u, float lo, float hi) { return lo + unit_f32(u) * (hi - lo); }

ORC_API void orc_philox_words(uint64_t seed, uint64_t stream, uint64_t offset, uint32_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = philox_word(seed, stream, offset + (uint64_t)i);
}

ORC_API void orc_fill_uniform(uint64_t seed, uint64_t offset, float lo, float hi, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = uniform_f32(philox_word(seed, 0, offset + (uint64_t)i), lo, hi);
}

// Random-init weights for the CPU timing leg (not part of the reference): N(0, std) by Box-Muller
// over two counter words, rounded to bf16 (nearest, ties to even), on all oracle threads. Values
// only need the benchmark's distribution; nothing compares them with the GPU's own weights.
ORC_API void orc_fill_normal_bf16(uint64_t seed, uint64_t stream, float stdev, uint16_t* out, int64_t n) {
  const int64_t groups = (n + 3) / 4;  // four values (two Box-Muller pairs) per counter block
  parallel_run([&](int tid, int nth) {
    const int64_t per = (groups + nth - 1) / nth;
    const int64_t g0 = tid * per, g1 = g0 + per < groups ? g0 + per : groups;
    for (int64_t g = g0; g < g1; ++g) {
      uint32_t o[4];
      philox((uint64_t)g, stream, seed, o);
      float z[4];
      for (int p = 0; p < 2; ++p) {
        const float u1 = ((float)(o[2 * p] >> 8) + 1.0f) * 5.9604644775390625e-08f;  // (0, 1]
        const float u2 = (float)(o[2 * p + 1] >> 8) * 5.9604644775390625e-08f;
        const float r = sqrtf(-2.0f * logf(u1)) * stdev, t = 6.2831853071795865f * u2;
        z[2 * p] = r * cosf(t);
        z[2 * p + 1] = r * sinf(t);
      }
      for (int k = 0; k < 4 && 4 * g + k < n; ++k) {
        uint32_t u;
        std::memcpy(&u, &z[k], 4);
        out[4 * g + k] = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
      }
    }
  });
}

// BeaverTriple::random (beaver.rs:44-68) restated over the counter generator.
ORC_API void orc_triples_f32(uint64_t seed, uint64_t offset, int64_t n, float* a, float* b, float* c,
                             float* ac, float* as, float* bc, float* bs, float* cc, float* cs) {
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t k = offset + (uint64_t)i;
    const float av = uniform_f32(philox_word(seed, 0, k), -1.0f, 1.0f);
    const float bv = uniform_f32(philox_word(seed, 1, k), -1.0f, 1.0f);
    const float cv = av * bv;
    const float a_s = uniform_f32(philox_word(seed, 2, k), -10.0f, 10.0f);
    const float b_s = uniform_f32(philox_word(seed, 3, k), -10.0f, 10.0f);
    const float c_s = uniform_f32(philox_word(seed, 4, k), -10.0f, 10.0f);
    if (a) a[i] = av;
    if (b) b[i] = bv;
    if (c) c[i] = cv;
    if (as) as[i] = a_s;
    if (bs) bs[i] = b_s;
    if (cs) cs[i] = c_s;
    if (ac) ac[i] = av - a_s;
    if (bc) bc[i] = bv - b_s;
    if (cc) cc[i] = cv - c_s;
  }
}

ORC_API void orc_triples_ring(uint64_t seed, uint64_t offset, int64_t n, uint32_t* ac, uint32_t* as,
                              uint32_t* bc, uint32_t* bs, uint32_t* cc, uint32_t* cs) {
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t k = offset + (uint64_t)i;
    const uint32_t av = philox_word(seed, 0, k), bv = philox_word(seed, 1, k);
    const uint32_t cv = av * bv;
    const uint32_t a_s = philox_word(seed, 2, k), b_s = philox_word(seed, 3, k), c_s = philox_word(seed, 4, k);
    if (as) as[i] = a_s;
    if (bs) bs[i] = b_s;
    if (cs) cs[i] = c_s;
    if (ac) ac[i] = av - a_s;
    if (bc) bc[i] = bv - b_s;
    if (cc) cc[i] = cv - c_s;
  }
}

// Embedding share generation (get_embeddings_direct, crates/v2/server/src/routes/
// secure_inference.rs:427-447: server share uniform [0,1), client share = e - s) restated over the
// counter generator: s_k = unit(word(seed, stream 7, counter * hidden + k)).
ORC_API void orc_embed_shares(const uint16_t* table, int hidden, int token, uint64_t seed,
                              uint64_t counter, float* hc, float* hs) {
  for (int k = 0; k < hidden; ++k) {
    const float e = bf16_to_f32(table[(size_t)token * hidden + k]);
    const float s = unit_f32(philox_word(seed, 7, counter * (uint64_t)hidden + (uint64_t)k));
    hs[k] = s;
    hc[k] = e - s;
  }
}

// ------------------------------------------------------------------------------------------------
// ChaCha20Rng (rand_chacha 0.3.1, a dependency pinned in the reference's Cargo.lock and absent
// here), restated from its published algorithm: the ChaCha20 block function (D. J. Bernstein,
// "ChaCha, a variant of Salsa20", 2008; 20 rounds = 10 column + diagonal double rounds) with the
// 32-byte seed as the key, a 64-bit block counter in words 12-13 starting at 0 and a 64-bit stream
// id (0) in words 14-15; next_u32 returns the keystream's little-endian 32-bit words in order.
// seed_from_u64 (rand_core 0.6.4, SeedableRng's default) expands a u64 into the 32-byte seed with
// eight PCG32 (XSH-RR, O'Neill 2014) outputs, advancing the state before each output.
// Used by Share::random_seeded (crates/sharing/src/share.rs:44-54) and get_embeddings_direct
// (crates/v2/server/src/routes/secure_inference.rs:387-460).
// ------------------------------------------------------------------------------------------------
static inline uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

static void chacha20_block(const uint32_t key[8], uint64_t counter, uint64_t stream, uint32_t out[16]) {
  uint32_t x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                    (uint32_t)counter, (uint32_t)(counter >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
  uint32_t in[16];
  std::memcpy(in, x, sizeof(in));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < 10; ++r) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + in[i];
}

static void key_words(const uint8_t seed[32], uint32_t key[8]) {
  for (int i = 0; i < 8; ++i)
    key[i] = (uint32_t)seed[4 * i] | ((uint32_t)seed[4 * i + 1] << 8) | ((uint32_t)seed[4 * i + 2] << 16) |
             ((uint32_t)seed[4 * i + 3] << 24);
}

ORC_API void orc_chacha20_words(const uint8_t seed[32], uint64_t word_offset, uint32_t* out, int64_t n) {
  uint32_t key[8], blk[16];
  key_words(seed, key);
  uint64_t cur = ~0ull;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t w = word_offset + (uint64_t)i;
    if (w / 16 != cur) {
      cur = w / 16;
      chacha20_block(key, cur, 0, blk);
    }
    out[i] = blk[w % 16];
  }
}

ORC_API void orc_seed_from_u64(uint64_t state, uint8_t seed[32]) {
  const uint64_t MUL = 6364136223846793005ull, INC = 11634580027462260723ull;
  for (int c = 0; c < 8; ++c) {
    state = state * MUL + INC;
    const uint32_t xorshifted = (uint32_t)(((state >> 18) ^ state) >> 27);
    const uint32_t rot = (uint32_t)(state >> 59);
    const uint32_t x = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
    for (int b = 0; b < 4; ++b) seed[4 * c + b] = (uint8_t)(x >> (8 * b));
  }
}

// Share::random_seeded + SharePair::from_plaintext_seeded (crates/sharing/src/share.rs:44-54,
// 116-135): server share = next_u32() as i32 from ChaCha20Rng::seed_from_u64(seed), client share =
// x wrapping_sub server.
ORC_API void orc_ring_share_seeded(const int32_t* x, int64_t n, uint64_t seed, int32_t* xc, int32_t* xs) {
  uint8_t key[32];
  orc_seed_from_u64(seed, key);
  std::vector<uint32_t> w((size_t)n);
  orc_chacha20_words(key, 0, w.data(), n);
  for (int64_t i = 0; i < n; ++i) {
    xs[i] = (int32_t)w[i];
    xc[i] = (int32_t)((uint32_t)x[i] - w[i]);
  }
}

// get_embeddings_direct (crates/v2/server/src/routes/secure_inference.rs:387-460): one ChaCha20Rng
// per request from seed = session id bytes || 16 zero bytes; for each token in order and each of
// its `hidden` elements, s = rng.gen::<f32>() (rand 0.8.5 Standard: (next_u32 >> 8) * 2^-24) and
// c = e - s with e the bf16 table value.
ORC_API void orc_embed_shares_chacha(const uint16_t* table, int hidden, const int32_t* tokens, int n_tokens,
                                     const uint8_t seed[32], float* hc, float* hs) {
  std::vector<uint32_t> w((size_t)n_tokens * hidden);
  orc_chacha20_words(seed, 0, w.data(), (int64_t)w.size());
  for (int t = 0; t < n_tokens; ++t)
    for (int k = 0; k < hidden; ++k) {
      const size_t i = (size_t)t * hidden + k;
      const float s = unit_f32(w[i]);
      hs[i] = s;
      hc[i] = bf16_to_f32(table[(size_t)tokens[t] * hidden + k]) - s;
    }
}

// OtFunctionTable::new (crates/v2/sharing/src/secure_nonlinear_ot.rs:44-72) for the functions of
// StandardOtTables::new (:554-575): kind 0 SiLU x * (1 / (1 + exp(-x))), 1 exp, 2 1/sqrt, 3 1/x;
// x_i = lo + i * step with step = (hi - lo) / (size - 1), all f32 as the Rust code.
ORC_API void orc_ot_table(int kind, float lo, float hi, int size, float* out) {
  const float step = (hi - lo) / (float)(size - 1);
  for (int i = 0; i < size; ++i) {
    const float x = lo + (float)i * step;
    float v;
    if (kind == 0) v = x * (1.0f / (1.0f + expf(-x)));
    else if (kind == 1) v = expf(x);
    else if (kind == 2) v = 1.0f / sqrtf(x);
    else v = 1.0f / x;
    out[i] = v;
  }
}

// OtFunctionTable::input_to_index: clamp, (x - min) / step rounded half away from zero, capped at
// size - 1; NaN -> 0 (Rust's saturating float-to-int cast).
ORC_API uint32_t orc_ot_input_to_index(float x, float lo, float hi, int size) {
  const float step = (hi - lo) / (float)(size - 1);
  if (std::isnan(x)) return 0;
  const float c = x < lo ? lo : (x > hi ? hi : x);
  const float r = std::round((c - lo) / step);
  long long idx = r < 0 ? 0 : (long long)r;
  return (uint32_t)(idx > size - 1 ? size - 1 : idx);
}
