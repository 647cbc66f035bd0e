// Elementwise share kernels: reconstruct, reshare, per-share add, Beaver multiply (f32 and Z_2^32),
// triple and mask generation. All are HBM-bound streams; each thread handles 4 consecutive
// elements with 16-byte accesses when every pointer is 16-byte aligned, else one element.
#include "shd_common.cuh"

namespace {

constexpr int kEwThreads = 256;

int ew_grid(shd_ctx* ctx, long long items) {
  long long g = (items + kEwThreads - 1) / kEwThreads;
  const long long cap = (long long)ctx->num_sms * 8;  // 8 resident CTAs of 256 threads per SM
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

bool all_aligned16(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p && !shd_aligned16(p)) return false;
  return true;
}

// ---- f32 Beaver (crates/v2/sharing/src/beaver.rs:167-197), operation order kept exactly ----
struct BeaverF32 {
  __device__ __forceinline__ static void op(float xc, float xs, float yc, float ys, float ac, float as,
                                            float bc, float bs, float cc, float cs, float& d, float& e,
                                            float& zc, float& zs) {
    const float dc = __fsub_rn(xc, ac), ds = __fsub_rn(xs, as);
    const float ec = __fsub_rn(yc, bc), es = __fsub_rn(ys, bs);
    d = __fadd_rn(dc, ds);
    e = __fadd_rn(ec, es);
    // z_client = c_c + a_c*e + d*b_c + d*e ; z_server = c_s + a_s*e + d*b_s (left to right)
    zc = __fadd_rn(__fadd_rn(__fadd_rn(cc, __fmul_rn(ac, e)), __fmul_rn(d, bc)), __fmul_rn(d, e));
    zs = __fadd_rn(__fadd_rn(cs, __fmul_rn(as, e)), __fmul_rn(d, bs));
  }
};

__global__ void beaver_f32_vec4(const float4* __restrict__ xc, const float4* __restrict__ xs,
                                const float4* __restrict__ yc, const float4* __restrict__ ys,
                                const float4* __restrict__ ac, const float4* __restrict__ as,
                                const float4* __restrict__ bc, const float4* __restrict__ bs,
                                const float4* __restrict__ cc, const float4* __restrict__ cs,
                                float4* __restrict__ dout, float4* __restrict__ eout,
                                float4* __restrict__ zc, float4* __restrict__ zs, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 a0 = __ldcs(xc + i), a1 = __ldcs(xs + i), a2 = __ldcs(yc + i), a3 = __ldcs(ys + i);
    const float4 t0 = __ldcs(ac + i), t1 = __ldcs(as + i), t2 = __ldcs(bc + i), t3 = __ldcs(bs + i);
    const float4 t4 = __ldcs(cc + i), t5 = __ldcs(cs + i);
    float4 d, e, z0, z1;
    BeaverF32::op(a0.x, a1.x, a2.x, a3.x, t0.x, t1.x, t2.x, t3.x, t4.x, t5.x, d.x, e.x, z0.x, z1.x);
    BeaverF32::op(a0.y, a1.y, a2.y, a3.y, t0.y, t1.y, t2.y, t3.y, t4.y, t5.y, d.y, e.y, z0.y, z1.y);
    BeaverF32::op(a0.z, a1.z, a2.z, a3.z, t0.z, t1.z, t2.z, t3.z, t4.z, t5.z, d.z, e.z, z0.z, z1.z);
    BeaverF32::op(a0.w, a1.w, a2.w, a3.w, t0.w, t1.w, t2.w, t3.w, t4.w, t5.w, d.w, e.w, z0.w, z1.w);
    if (dout) __stcs(dout + i, d);
    if (eout) __stcs(eout + i, e);
    __stcs(zc + i, z0);
    __stcs(zs + i, z1);
  }
}

__global__ void beaver_f32_scalar(const float* __restrict__ xc, const float* __restrict__ xs,
                                  const float* __restrict__ yc, const float* __restrict__ ys,
                                  const float* __restrict__ ac, const float* __restrict__ as,
                                  const float* __restrict__ bc, const float* __restrict__ bs,
                                  const float* __restrict__ cc, const float* __restrict__ cs,
                                  float* __restrict__ dout, float* __restrict__ eout,
                                  float* __restrict__ zc, float* __restrict__ zs, long long i0,
                                  long long n) {
  for (long long i = i0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float d, e, z0, z1;
    BeaverF32::op(xc[i], xs[i], yc[i], ys[i], ac[i], as[i], bc[i], bs[i], cc[i], cs[i], d, e, z0, z1);
    if (dout) dout[i] = d;
    if (eout) eout[i] = e;
    zc[i] = z0;
    zs[i] = z1;
  }
}

// ---- Z_2^32 Beaver: wrapping arithmetic; optional SecureML local truncation ----
__device__ __forceinline__ void beaver_ring_op(uint32_t xc, uint32_t xs, uint32_t yc, uint32_t ys,
                                               uint32_t ac, uint32_t as, uint32_t bc, uint32_t bs,
                                               uint32_t cc, uint32_t cs, int f, uint32_t& d,
                                               uint32_t& e, uint32_t& zc, uint32_t& zs) {
  d = (xc - ac) + (xs - as);
  e = (yc - bc) + (ys - bs);
  zc = cc + ac * e + d * bc + d * e;
  zs = cs + as * e + d * bs;
  if (f > 0) {
    zc = (uint32_t)((int32_t)zc >> f);
    zs = 0u - (uint32_t)((int32_t)(0u - zs) >> f);
  }
}

__global__ void beaver_ring_vec4(const uint4* __restrict__ xc, const uint4* __restrict__ xs,
                                 const uint4* __restrict__ yc, const uint4* __restrict__ ys,
                                 const uint4* __restrict__ ac, const uint4* __restrict__ as,
                                 const uint4* __restrict__ bc, const uint4* __restrict__ bs,
                                 const uint4* __restrict__ cc, const uint4* __restrict__ cs,
                                 uint4* __restrict__ dout, uint4* __restrict__ eout,
                                 uint4* __restrict__ zc, uint4* __restrict__ zs, long long n4, int f) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const uint4 a0 = __ldcs(xc + i), a1 = __ldcs(xs + i), a2 = __ldcs(yc + i), a3 = __ldcs(ys + i);
    const uint4 t0 = __ldcs(ac + i), t1 = __ldcs(as + i), t2 = __ldcs(bc + i), t3 = __ldcs(bs + i);
    const uint4 t4 = __ldcs(cc + i), t5 = __ldcs(cs + i);
    uint4 d, e, z0, z1;
    beaver_ring_op(a0.x, a1.x, a2.x, a3.x, t0.x, t1.x, t2.x, t3.x, t4.x, t5.x, f, d.x, e.x, z0.x, z1.x);
    beaver_ring_op(a0.y, a1.y, a2.y, a3.y, t0.y, t1.y, t2.y, t3.y, t4.y, t5.y, f, d.y, e.y, z0.y, z1.y);
    beaver_ring_op(a0.z, a1.z, a2.z, a3.z, t0.z, t1.z, t2.z, t3.z, t4.z, t5.z, f, d.z, e.z, z0.z, z1.z);
    beaver_ring_op(a0.w, a1.w, a2.w, a3.w, t0.w, t1.w, t2.w, t3.w, t4.w, t5.w, f, d.w, e.w, z0.w, z1.w);
    if (dout) __stcs(dout + i, d);
    if (eout) __stcs(eout + i, e);
    __stcs(zc + i, z0);
    __stcs(zs + i, z1);
  }
}

__global__ void beaver_ring_scalar(const uint32_t* __restrict__ xc, const uint32_t* __restrict__ xs,
                                   const uint32_t* __restrict__ yc, const uint32_t* __restrict__ ys,
                                   const uint32_t* __restrict__ ac, const uint32_t* __restrict__ as,
                                   const uint32_t* __restrict__ bc, const uint32_t* __restrict__ bs,
                                   const uint32_t* __restrict__ cc, const uint32_t* __restrict__ cs,
                                   uint32_t* __restrict__ dout, uint32_t* __restrict__ eout,
                                   uint32_t* __restrict__ zc, uint32_t* __restrict__ zs, long long i0,
                                   long long n, int f) {
  for (long long i = i0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    uint32_t d, e, z0, z1;
    beaver_ring_op(xc[i], xs[i], yc[i], ys[i], ac[i], as[i], bc[i], bs[i], cc[i], cs[i], f, d, e, z0, z1);
    if (dout) dout[i] = d;
    if (eout) eout[i] = e;
    zc[i] = z0;
    zs[i] = z1;
  }
}

// ---- reconstruct / reshare / add ----
__global__ void reconstruct_kernel(const float* __restrict__ c, const float* __restrict__ s,
                                   float* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = __fadd_rn(c[i], s[i]);
}

__global__ void reshare_kernel(const float* __restrict__ y, const float* __restrict__ mask,
                               float* __restrict__ oc, float* __restrict__ os, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float m = mask ? mask[i] : 0.0f;
    const float v = y[i];
    oc[i] = __fsub_rn(v, m);
    os[i] = m;
  }
}

__global__ void add_shares_kernel(const float* __restrict__ ac, const float* __restrict__ as,
                                  const float* __restrict__ bc, const float* __restrict__ bs,
                                  float* __restrict__ yc, float* __restrict__ ys, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float c = __fadd_rn(ac[i], bc[i]);
    const float s = __fadd_rn(as[i], bs[i]);
    yc[i] = c;
    ys[i] = s;
  }
}

// ---- generators. Streams: 0 a, 1 b, 2 a_server, 3 b_server, 4 c_server (f32); ring the same ----
__global__ void triples_f32_kernel(uint64_t seed, uint64_t offset, long long n, float* a, float* b,
                                   float* c, float* ac, float* as, float* bc, float* bs, float* cc,
                                   float* cs) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const uint64_t k = offset + (uint64_t)i;
    const float av = uniform_f32(philox_word(seed, 0, k), -1.0f, 1.0f);
    const float bv = uniform_f32(philox_word(seed, 1, k), -1.0f, 1.0f);
    const float cv = __fmul_rn(av, bv);
    const float a_s = uniform_f32(philox_word(seed, 2, k), -10.0f, 10.0f);
    const float b_s = uniform_f32(philox_word(seed, 3, k), -10.0f, 10.0f);
    const float c_s = uniform_f32(philox_word(seed, 4, k), -10.0f, 10.0f);
    if (a) a[i] = av;
    if (b) b[i] = bv;
    if (c) c[i] = cv;
    if (as) as[i] = a_s;
    if (bs) bs[i] = b_s;
    if (cs) cs[i] = c_s;
    if (ac) ac[i] = __fsub_rn(av, a_s);
    if (bc) bc[i] = __fsub_rn(bv, b_s);
    if (cc) cc[i] = __fsub_rn(cv, c_s);
  }
}

__global__ void triples_ring_kernel(uint64_t seed, uint64_t offset, long long n, uint32_t* ac,
                                    uint32_t* as, uint32_t* bc, uint32_t* bs, uint32_t* cc,
                                    uint32_t* cs) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const uint64_t k = offset + (uint64_t)i;
    const uint32_t av = philox_word(seed, 0, k), bv = philox_word(seed, 1, k);
    const uint32_t cv = av * bv;
    const uint32_t a_s = philox_word(seed, 2, k), b_s = philox_word(seed, 3, k);
    const uint32_t c_s = philox_word(seed, 4, k);
    if (as) as[i] = a_s;
    if (bs) bs[i] = b_s;
    if (cs) cs[i] = c_s;
    if (ac) ac[i] = av - a_s;
    if (bc) bc[i] = bv - b_s;
    if (cc) cc[i] = cv - c_s;
  }
}

__global__ void fill_uniform_kernel(uint64_t seed, uint64_t offset, float lo, float hi, float* out,
                                    long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = uniform_f32(philox_word(seed, 0, offset + (uint64_t)i), lo, hi);
}

}  // namespace

extern "C" int shd_reconstruct_f32(shd_ctx* ctx, const float* c, const float* s, float* y, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_reconstruct_f32: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, c && s && y, "shd_reconstruct_f32: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  reconstruct_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(c, s, y, n);
  SHD_CHECK_LAUNCH(ctx, "reconstruct_kernel");
  return SHD_OK;
}

extern "C" int shd_reshare_f32(shd_ctx* ctx, const float* y, const float* mask, float* out_c,
                               float* out_s, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_reshare_f32: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, y && out_c && out_s, "shd_reshare_f32: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  reshare_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(y, mask, out_c, out_s, n);
  SHD_CHECK_LAUNCH(ctx, "reshare_kernel");
  return SHD_OK;
}

extern "C" int shd_add_shares(shd_ctx* ctx, const float* ac, const float* as, const float* bc,
                              const float* bs, float* yc, float* ys, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_add_shares: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, ac && as && bc && bs && yc && ys, "shd_add_shares: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  add_shares_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(ac, as, bc, bs, yc, ys, n);
  SHD_CHECK_LAUNCH(ctx, "add_shares_kernel");
  return SHD_OK;
}

extern "C" int shd_beaver_mul_f32(shd_ctx* ctx, const float* xc, const float* xs, const float* yc,
                                  const float* ys, const float* ac, const float* as, const float* bc,
                                  const float* bs, const float* cc, const float* cs, float* d_out,
                                  float* e_out, float* zc, float* zs, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_beaver_mul_f32: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && yc && ys && ac && as && bc && bs && cc && cs && zc && zs,
              "shd_beaver_mul_f32: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  long long done = 0;
  if (all_aligned16({xc, xs, yc, ys, ac, as, bc, bs, cc, cs, d_out, e_out, zc, zs}) && n >= 4) {
    const long long n4 = n / 4;
    beaver_f32_vec4<<<ew_grid(ctx, n4), kEwThreads, 0, ctx->stream>>>(
        (const float4*)xc, (const float4*)xs, (const float4*)yc, (const float4*)ys, (const float4*)ac,
        (const float4*)as, (const float4*)bc, (const float4*)bs, (const float4*)cc, (const float4*)cs,
        (float4*)d_out, (float4*)e_out, (float4*)zc, (float4*)zs, n4);
    SHD_CHECK_LAUNCH(ctx, "beaver_f32_vec4");
    done = n4 * 4;
  }
  if (done < n) {
    beaver_f32_scalar<<<ew_grid(ctx, n - done), kEwThreads, 0, ctx->stream>>>(
        xc, xs, yc, ys, ac, as, bc, bs, cc, cs, d_out, e_out, zc, zs, done, n);
    SHD_CHECK_LAUNCH(ctx, "beaver_f32_scalar");
  }
  return SHD_OK;
}

extern "C" int shd_beaver_mul_ring(shd_ctx* ctx, const uint32_t* xc, const uint32_t* xs,
                                   const uint32_t* yc, const uint32_t* ys, const uint32_t* ac,
                                   const uint32_t* as, const uint32_t* bc, const uint32_t* bs,
                                   const uint32_t* cc, const uint32_t* cs, uint32_t* d_out,
                                   uint32_t* e_out, uint32_t* zc, uint32_t* zs, int64_t n,
                                   int trunc_shift) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_beaver_mul_ring: n < 0");
  SHD_REQUIRE(ctx, trunc_shift >= 0 && trunc_shift < 32, "shd_beaver_mul_ring: trunc_shift outside 0..31");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, xc && xs && yc && ys && ac && as && bc && bs && cc && cs && zc && zs,
              "shd_beaver_mul_ring: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  long long done = 0;
  if (all_aligned16({xc, xs, yc, ys, ac, as, bc, bs, cc, cs, d_out, e_out, zc, zs}) && n >= 4) {
    const long long n4 = n / 4;
    beaver_ring_vec4<<<ew_grid(ctx, n4), kEwThreads, 0, ctx->stream>>>(
        (const uint4*)xc, (const uint4*)xs, (const uint4*)yc, (const uint4*)ys, (const uint4*)ac,
        (const uint4*)as, (const uint4*)bc, (const uint4*)bs, (const uint4*)cc, (const uint4*)cs,
        (uint4*)d_out, (uint4*)e_out, (uint4*)zc, (uint4*)zs, n4, trunc_shift);
    SHD_CHECK_LAUNCH(ctx, "beaver_ring_vec4");
    done = n4 * 4;
  }
  if (done < n) {
    beaver_ring_scalar<<<ew_grid(ctx, n - done), kEwThreads, 0, ctx->stream>>>(
        xc, xs, yc, ys, ac, as, bc, bs, cc, cs, d_out, e_out, zc, zs, done, n, trunc_shift);
    SHD_CHECK_LAUNCH(ctx, "beaver_ring_scalar");
  }
  return SHD_OK;
}

extern "C" int shd_beaver_triples_f32(shd_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n,
                                      float* a, float* b, float* c, float* ac, float* as, float* bc,
                                      float* bs, float* cc, float* cs) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_beaver_triples_f32: n < 0");
  if (n == 0) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  triples_f32_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(seed, offset, n, a, b, c, ac,
                                                                          as, bc, bs, cc, cs);
  SHD_CHECK_LAUNCH(ctx, "triples_f32_kernel");
  return SHD_OK;
}

extern "C" int shd_beaver_triples_ring(shd_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n,
                                       uint32_t* ac, uint32_t* as, uint32_t* bc, uint32_t* bs,
                                       uint32_t* cc, uint32_t* cs) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_beaver_triples_ring: n < 0");
  if (n == 0) return SHD_OK;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  triples_ring_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(seed, offset, n, ac, as, bc,
                                                                           bs, cc, cs);
  SHD_CHECK_LAUNCH(ctx, "triples_ring_kernel");
  return SHD_OK;
}

extern "C" int shd_fill_uniform_f32(shd_ctx* ctx, uint64_t seed, uint64_t offset, float lo, float hi,
                                    float* out, int64_t n) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, n >= 0, "shd_fill_uniform_f32: n < 0");
  if (n == 0) return SHD_OK;
  SHD_REQUIRE(ctx, out, "shd_fill_uniform_f32: null output");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  fill_uniform_kernel<<<ew_grid(ctx, n), kEwThreads, 0, ctx->stream>>>(seed, offset, lo, hi, out, n);
  SHD_CHECK_LAUNCH(ctx, "fill_uniform_kernel");
  return SHD_OK;
}
