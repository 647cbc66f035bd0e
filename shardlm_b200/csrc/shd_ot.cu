// V3-OT: the server's side of the function-table lookups on the GPU.
//
// In the V3-OT route (crates/v2/server/src/routes/secure_inference_ot.rs:504-600) the client sends
// batches of 1-of-N OT queries against the server's function tables (StandardOtTables: SiLU, exp,
// 1/sqrt, 1/x, crates/v2/sharing/src/secure_nonlinear_ot.rs:554-585), and the server answers each
// with IknpOtExtension::process_query (crates/ot/src/iknp.rs:495-572): per query entry j
//   item_key = SHA-256("IKNP-Item-Key-v2" || commitment || batch_seed || u32 j || u64 ctr)[0..16]
//   idx      = idx_enc ^ u32(PRF(item_key, 0, 4))          (an index >= table rows is an error)
//   row_key  = row_key_enc ^ PRF(item_key, 1, 16)
//   response_j = table[idx] ^ PRF(row_key, ctr * 1000 + j, row_bytes)
// with PRF(k, c, len) the AES-128 encryptions under k of the blocks (u64 c || u64 i), i = 0, 1, ...
// (little-endian), truncated to len. The reference runs the entries one by one on the CPU; here one
// GPU thread serves one entry: SHA-256 (FIPS 180-4) from the midstate of the query's common first
// block (computed once on the host), two AES-128 key expansions and the PRF blocks (FIPS-197,
// T-table formulation, tables in shared memory, generated on the host from the S-box's definition:
// multiplicative inverse in GF(2^8) followed by the affine map).
//
// The function tables themselves (OtFunctionTable::new, secure_nonlinear_ot.rs:44-72) are built on
// the host with the same f32 operations and libm calls as the reference's Rust (f32 exp and sqrt
// on Linux), so the table bytes are the reference's.
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "shd_common.cuh"

namespace {

// ------------------------------------------------------------------------------------------------
// Host-side constants, generated from their definitions
// ------------------------------------------------------------------------------------------------
struct AesTables {
  uint32_t te[4][256];
  uint8_t sbox[256];
};

uint8_t gf_mul(uint8_t a, uint8_t b) {
  uint8_t r = 0;
  while (b) {
    if (b & 1) r ^= a;
    a = (uint8_t)((a << 1) ^ ((a & 0x80) ? 0x1b : 0));
    b >>= 1;
  }
  return r;
}

const AesTables& aes_tables() {
  static AesTables t;
  static std::once_flag once;
  std::call_once(once, [] {
    for (int x = 0; x < 256; ++x) {
      uint8_t inv = 0;
      if (x)
        for (int y = 1; y < 256; ++y)
          if (gf_mul((uint8_t)x, (uint8_t)y) == 1) {
            inv = (uint8_t)y;
            break;
          }
      // affine map: b ^ rotl(b,1) ^ rotl(b,2) ^ rotl(b,3) ^ rotl(b,4) ^ 0x63
      uint8_t s = inv;
      for (int r = 1; r <= 4; ++r) s ^= (uint8_t)((inv << r) | (inv >> (8 - r)));
      t.sbox[x] = (uint8_t)(s ^ 0x63);
    }
    for (int x = 0; x < 256; ++x) {
      const uint8_t s = t.sbox[x];
      const uint32_t w = ((uint32_t)gf_mul(s, 2) << 24) | ((uint32_t)s << 16) | ((uint32_t)s << 8) | gf_mul(s, 3);
      t.te[0][x] = w;
      t.te[1][x] = (w >> 8) | (w << 24);
      t.te[2][x] = (w >> 16) | (w << 16);
      t.te[3][x] = (w >> 24) | (w << 8);
    }
  });
  return t;
}

// SHA-256 round constants and initial state: the first 32 bits of the fractional parts of the cube
// roots of the first 64 primes and of the square roots of the first 8 primes.
struct ShaConsts {
  uint32_t k[64];
  uint32_t h0[8];
};

uint32_t frac32(double v) {
  const double f = v - std::floor(v);
  return (uint32_t)std::floor(f * 4294967296.0);
}

const ShaConsts& sha_consts() {
  static ShaConsts c;
  static std::once_flag once;
  std::call_once(once, [] {
    int n = 0;
    for (int p = 2; n < 64; ++p) {
      bool prime = true;
      for (int d = 2; d * d <= p; ++d)
        if (p % d == 0) prime = false;
      if (!prime) continue;
      if (n < 8) c.h0[n] = frac32(std::sqrt((double)p));
      c.k[n] = frac32(std::cbrt((double)p));
      ++n;
    }
  });
  return c;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha256_block_host(uint32_t st[8], const uint8_t blk[64], const ShaConsts& c) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = ((uint32_t)blk[4 * i] << 24) | ((uint32_t)blk[4 * i + 1] << 16) | ((uint32_t)blk[4 * i + 2] << 8) | blk[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = st[0], b = st[1], cc = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
  for (int i = 0; i < 64; ++i) {
    const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + c.k[i] + w[i];
    const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & cc) ^ (b & cc));
    h = g; g = f; f = e; e = d + t1; d = cc; cc = b; b = a; a = t1 + t2;
  }
  st[0] += a; st[1] += b; st[2] += cc; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

// ------------------------------------------------------------------------------------------------
// Device side
// ------------------------------------------------------------------------------------------------
struct OtArgs {
  uint32_t mid[8];        // SHA-256 state after the common first 64 bytes of every item-key message
  uint8_t tail16[16];     // batch_seed[16..32): the first bytes of the second block
  uint64_t ctr;
  const uint8_t* entries;  // [m][20]: idx_enc (u32 LE) || row_key_enc (16)
  int m;
  const uint8_t* table;    // [rows][row_bytes]
  int rows, row_bytes;
  uint8_t* out;            // [m][row_bytes]
  unsigned int* first_bad;  // lowest entry index whose idx is out of range (atomic min)
  const uint32_t* k;       // SHA-256 round constants [64]
  const uint32_t* te;      // AES T-tables [4][256]
  const uint8_t* sbox;     // [256]
};

__device__ __forceinline__ uint32_t drotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

__device__ void sha256_compress(uint32_t st[8], const uint32_t w_in[16], const uint32_t* K) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = w_in[i];
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll 4
  for (int i = 0; i < 64; ++i) {
    uint32_t wi;
    if (i < 16) {
      wi = w[i];
    } else {
      const uint32_t w15 = w[(i - 15) & 15], w2 = w[(i - 2) & 15];
      const uint32_t s0 = drotr(w15, 7) ^ drotr(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = drotr(w2, 17) ^ drotr(w2, 19) ^ (w2 >> 10);
      wi = w[i & 15] + s0 + w[(i - 7) & 15] + s1;
      w[i & 15] = wi;
    }
    const uint32_t t1 = h + (drotr(e, 6) ^ drotr(e, 11) ^ drotr(e, 25)) + ((e & f) ^ (~e & g)) + K[i] + wi;
    const uint32_t t2 = (drotr(a, 2) ^ drotr(a, 13) ^ drotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

struct AesSmem {
  uint32_t te[4][256];
  uint8_t sbox[256];
  uint32_t k[64];
};

__device__ __forceinline__ uint32_t sub_word(const AesSmem& S, uint32_t w) {
  return ((uint32_t)S.sbox[w >> 24] << 24) | ((uint32_t)S.sbox[(w >> 16) & 0xff] << 16) |
         ((uint32_t)S.sbox[(w >> 8) & 0xff] << 8) | S.sbox[w & 0xff];
}

// AES-128 key expansion: key bytes -> 44 big-endian round-key words.
__device__ void aes_expand(const AesSmem& S, const uint8_t key[16], uint32_t rk[44]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    rk[i] = ((uint32_t)key[4 * i] << 24) | ((uint32_t)key[4 * i + 1] << 16) | ((uint32_t)key[4 * i + 2] << 8) | key[4 * i + 3];
  uint32_t rcon = 0x01;
#pragma unroll
  for (int i = 4; i < 44; ++i) {
    uint32_t t = rk[i - 1];
    if ((i & 3) == 0) {
      t = sub_word(S, (t << 8) | (t >> 24)) ^ (rcon << 24);
      rcon = (rcon << 1) ^ ((rcon & 0x80) ? 0x11b : 0);
    }
    rk[i] = rk[i - 4] ^ t;
  }
}

// Encrypt the block (u64 c || u64 i, little-endian) under rk; out = the 16 ciphertext bytes.
__device__ void aes_encrypt_ctr(const AesSmem& S, const uint32_t rk[44], uint64_t c, uint64_t i, uint8_t out[16]) {
  uint8_t in[16];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    in[b] = (uint8_t)(c >> (8 * b));
    in[8 + b] = (uint8_t)(i >> (8 * b));
  }
  uint32_t s[4];
#pragma unroll
  for (int w = 0; w < 4; ++w)
    s[w] = (((uint32_t)in[4 * w] << 24) | ((uint32_t)in[4 * w + 1] << 16) | ((uint32_t)in[4 * w + 2] << 8) | in[4 * w + 3]) ^ rk[w];
#pragma unroll
  for (int r = 1; r < 10; ++r) {
    uint32_t t[4];
#pragma unroll
    for (int w = 0; w < 4; ++w)
      t[w] = S.te[0][s[w] >> 24] ^ S.te[1][(s[(w + 1) & 3] >> 16) & 0xff] ^ S.te[2][(s[(w + 2) & 3] >> 8) & 0xff] ^
             S.te[3][s[(w + 3) & 3] & 0xff] ^ rk[4 * r + w];
#pragma unroll
    for (int w = 0; w < 4; ++w) s[w] = t[w];
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t o = ((uint32_t)S.sbox[s[w] >> 24] << 24) ^ ((uint32_t)S.sbox[(s[(w + 1) & 3] >> 16) & 0xff] << 16) ^
                       ((uint32_t)S.sbox[(s[(w + 2) & 3] >> 8) & 0xff] << 8) ^ S.sbox[s[(w + 3) & 3] & 0xff] ^ rk[40 + w];
    out[4 * w] = (uint8_t)(o >> 24);
    out[4 * w + 1] = (uint8_t)(o >> 16);
    out[4 * w + 2] = (uint8_t)(o >> 8);
    out[4 * w + 3] = (uint8_t)o;
  }
}

constexpr int kOtThreads = 128;

__global__ void __launch_bounds__(kOtThreads) ot_process_kernel(const __grid_constant__ OtArgs a) {
  __shared__ AesSmem S;
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) (&S.te[0][0])[i] = a.te[i];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) S.sbox[i] = a.sbox[i];
  for (int i = threadIdx.x; i < 64; i += blockDim.x) S.k[i] = a.k[i];
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.m) return;
  // second SHA-256 block: batch_seed[16..32) || u32 j || u64 ctr || 0x80 || 0... || bit length 736
  uint8_t blk[64];
#pragma unroll
  for (int b = 0; b < 16; ++b) blk[b] = a.tail16[b];
#pragma unroll
  for (int b = 0; b < 4; ++b) blk[16 + b] = (uint8_t)((uint32_t)j >> (8 * b));
#pragma unroll
  for (int b = 0; b < 8; ++b) blk[20 + b] = (uint8_t)(a.ctr >> (8 * b));
  blk[28] = 0x80;
#pragma unroll
  for (int b = 29; b < 62; ++b) blk[b] = 0;
  blk[62] = (uint8_t)(736 >> 8);
  blk[63] = (uint8_t)(736 & 0xff);
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    w[i] = ((uint32_t)blk[4 * i] << 24) | ((uint32_t)blk[4 * i + 1] << 16) | ((uint32_t)blk[4 * i + 2] << 8) | blk[4 * i + 3];
  uint32_t st[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) st[i] = a.mid[i];
  sha256_compress(st, w, S.k);
  uint8_t item_key[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    item_key[4 * i] = (uint8_t)(st[i] >> 24);
    item_key[4 * i + 1] = (uint8_t)(st[i] >> 16);
    item_key[4 * i + 2] = (uint8_t)(st[i] >> 8);
    item_key[4 * i + 3] = (uint8_t)st[i];
  }
  uint32_t rk[44];
  aes_expand(S, item_key, rk);
  uint8_t m0[16], m1[16];
  aes_encrypt_ctr(S, rk, 0, 0, m0);
  aes_encrypt_ctr(S, rk, 1, 0, m1);
  const uint8_t* e = a.entries + (size_t)j * 20;
  const uint32_t idx_enc = (uint32_t)e[0] | ((uint32_t)e[1] << 8) | ((uint32_t)e[2] << 16) | ((uint32_t)e[3] << 24);
  const uint32_t idx = idx_enc ^ ((uint32_t)m0[0] | ((uint32_t)m0[1] << 8) | ((uint32_t)m0[2] << 16) | ((uint32_t)m0[3] << 24));
  uint8_t* out = a.out + (size_t)j * a.row_bytes;
  if (idx >= (uint32_t)a.rows) {
    atomicMin(a.first_bad, (unsigned int)j);
    for (int b = 0; b < a.row_bytes; ++b) out[b] = 0;
    return;
  }
  uint8_t row_key[16];
#pragma unroll
  for (int b = 0; b < 16; ++b) row_key[b] = e[4 + b] ^ m1[b];
  aes_expand(S, row_key, rk);
  const uint8_t* row = a.table + (size_t)idx * a.row_bytes;
  const uint64_t c = a.ctr * 1000ull + (uint64_t)j;
  for (int blkno = 0; blkno * 16 < a.row_bytes; ++blkno) {
    uint8_t mk[16];
    aes_encrypt_ctr(S, rk, c, (uint64_t)blkno, mk);
    const int n = min(16, a.row_bytes - 16 * blkno);
    for (int b = 0; b < n; ++b) out[16 * blkno + b] = row[16 * blkno + b] ^ mk[b];
  }
}

struct OtDeviceConsts {
  uint32_t* k = nullptr;
  uint32_t* te = nullptr;
  uint8_t* sbox = nullptr;
};

std::mutex g_ot_mu;
OtDeviceConsts g_ot_dev[64];

int ot_consts(shd_ctx* ctx, OtDeviceConsts* out) {
  const int dev = ctx->device;
  if (dev < 0 || dev >= 64) return shd_fail(ctx, SHD_ERR_ARG, "ot: device index");
  std::lock_guard<std::mutex> lock(g_ot_mu);
  OtDeviceConsts& c = g_ot_dev[dev];
  if (!c.k) {
    const ShaConsts& sc = sha_consts();
    const AesTables& at = aes_tables();
    void* p = nullptr;
    SHD_CHECK_CUDA(ctx, cudaMalloc(&p, 64 * 4 + 1024 * 4 + 256));
    uint8_t* base = static_cast<uint8_t*>(p);
    SHD_CHECK_CUDA(ctx, cudaMemcpy(base, sc.k, 64 * 4, cudaMemcpyHostToDevice));
    SHD_CHECK_CUDA(ctx, cudaMemcpy(base + 256, at.te, 1024 * 4, cudaMemcpyHostToDevice));
    SHD_CHECK_CUDA(ctx, cudaMemcpy(base + 256 + 4096, at.sbox, 256, cudaMemcpyHostToDevice));
    c.k = reinterpret_cast<uint32_t*>(base);
    c.te = reinterpret_cast<uint32_t*>(base + 256);
    c.sbox = base + 256 + 4096;
  }
  *out = c;
  return SHD_OK;
}

// OtFunctionTable::new: x_i = min + i * step, step = (max - min) / (size - 1), all in f32.
void build_table(int kind, float lo, float hi, int size, float* out) {
  const float step = (hi - lo) / (float)(size - 1);
  for (int i = 0; i < size; ++i) {
    const float x = lo + (float)i * step;
    float v;
    switch (kind) {
      case 0: v = x * (1.0f / (1.0f + expf(-x))); break;  // SiLU
      case 1: v = expf(x); break;
      case 2: v = 1.0f / sqrtf(x); break;
      default: v = 1.0f / x; break;
    }
    out[i] = v;
  }
}

}  // namespace

// StandardOtTables::new(size) (secure_nonlinear_ot.rs:554-575): [4][size] f32 on the device in the
// order silu [-8, 8], exp [-10, 0], rsqrt [0.01, 10], reciprocal [0.01, 100].
extern "C" int shd_ot_standard_tables(shd_ctx* ctx, int table_size, float* dev_out) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, table_size >= 2 && dev_out, "shd_ot_standard_tables: table_size >= 2 and an output buffer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  std::vector<float> t((size_t)4 * table_size);
  const float lo[4] = {-8.0f, -10.0f, 0.01f, 0.01f}, hi[4] = {8.0f, 0.0f, 10.0f, 100.0f};
  for (int k = 0; k < 4; ++k) build_table(k, lo[k], hi[k], table_size, t.data() + (size_t)k * table_size);
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(dev_out, t.data(), t.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SHD_OK;
}

extern "C" int shd_ot_process_query(shd_ctx* ctx, const uint8_t* commitment32, uint64_t ctr, const uint8_t* query,
                                    size_t query_len, const uint8_t* table_dev, size_t table_bytes, int row_bytes,
                                    uint8_t* response, size_t response_cap, size_t* response_len) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, commitment32 && query && table_dev && response_len, "shd_ot_process_query: null pointer");
  SHD_REQUIRE(ctx, row_bytes > 0 && table_bytes >= (size_t)row_bytes, "shd_ot_process_query: bad table");
  // InvalidMessageFormat: u16 m || batch_seed[32] || m x (u32 idx_enc || row_key_enc[16])
  if (query_len < 34) return shd_fail(ctx, SHD_ERR_ARG, "shd_ot_process_query: InvalidMessageFormat");
  const int m = (int)((uint32_t)query[0] | ((uint32_t)query[1] << 8));
  if (query_len != 34 + (size_t)m * 20) return shd_fail(ctx, SHD_ERR_ARG, "shd_ot_process_query: InvalidMessageFormat");
  const size_t need = (size_t)m * row_bytes;
  *response_len = need;
  if (m == 0) return SHD_OK;
  if (!response || response_cap < need)
    return shd_fail(ctx, SHD_ERR_ARG, "shd_ot_process_query: response needs " + std::to_string(need) + " bytes");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  OtDeviceConsts dc;
  int rc = ot_consts(ctx, &dc);
  if (rc) return rc;
  // the first 64 bytes of every item-key message: domain string || commitment || batch_seed[0..16)
  OtArgs a{};
  {
    const ShaConsts& sc = sha_consts();
    uint8_t blk[64];
    std::memcpy(blk, "IKNP-Item-Key-v2", 16);
    std::memcpy(blk + 16, commitment32, 32);
    std::memcpy(blk + 48, query + 2, 16);
    for (int i = 0; i < 8; ++i) a.mid[i] = sc.h0[i];
    sha256_block_host(a.mid, blk, sc);
    std::memcpy(a.tail16, query + 18, 16);
  }
  a.ctr = ctr;
  a.m = m;
  a.table = table_dev;
  a.rows = (int)(table_bytes / (size_t)row_bytes);
  a.row_bytes = row_bytes;
  a.k = dc.k;
  a.te = dc.te;
  a.sbox = dc.sbox;
  // staging: entries in, masked rows out, the error word
  uint8_t* d = nullptr;
  const size_t ent = (size_t)m * 20, outb = need, al = 256;
  const size_t bytes = (ent + al - 1) / al * al + (outb + al - 1) / al * al + al;
  {
    void* p = nullptr;
    const int src = shd_stage(ctx, bytes, &p);
    if (src) return src;
    d = static_cast<uint8_t*>(p);
  }
  uint8_t* d_ent = d;
  uint8_t* d_out = d + (ent + al - 1) / al * al;
  unsigned int* d_bad = reinterpret_cast<unsigned int*>(d_out + (outb + al - 1) / al * al);
  a.entries = d_ent;
  a.out = d_out;
  a.first_bad = d_bad;
  cudaError_t e = cudaMemcpyAsync(d_ent, query + 34, ent, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_bad, 0xff, 4, ctx->stream);
  if (e == cudaSuccess) {
    ot_process_kernel<<<(m + kOtThreads - 1) / kOtThreads, kOtThreads, 0, ctx->stream>>>(a);
    e = cudaGetLastError();
    ctx->launches++;
  }
  unsigned int bad = 0xffffffffu;
  if (e == cudaSuccess) e = cudaMemcpyAsync(response, d_out, outb, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&bad, d_bad, 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return shd_cuda_fail(ctx, e, "shd_ot_process_query");
  if (bad != 0xffffffffu) {
    // the reference stops at the first entry whose index is out of range
    return shd_fail(ctx, SHD_ERR_ARG, "shd_ot_process_query: InvalidIndex at entry " + std::to_string(bad) +
                                          " (max " + std::to_string(a.rows) + ")");
  }
  return SHD_OK;
}
