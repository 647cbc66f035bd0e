// Context, error plumbing and weight tiling for libshardlm_cuda.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "shd_gemv.cuh"
#include "shd_tc.cuh"

using namespace shd;

int shd_fail(shd_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

int shd_cuda_fail(shd_ctx* ctx, cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return shd_fail(ctx, SHD_ERR_CUDA, m);
}

// Split-K partial storage: up to two CTAs per SM, 2 slots per CTA, a tile of 32 rows x 2 shares x
// 8 token rows, 8 bytes per value (the ring kernel accumulates in 64 bits).
static size_t partial_floats_for(int sms) { return (size_t)2 * sms * 2 * (kTileRows * 2 * 8) * 2; }

extern "C" int shd_init(int device, shd_ctx** out) {
  if (!out) return SHD_ERR_ARG;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return SHD_ERR_CUDA;
  }
  if (device < 0 || device >= ndev) return SHD_ERR_ARG;
  shd_ctx* ctx = new shd_ctx();
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) { delete ctx; return SHD_ERR_CUDA; }
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) { delete ctx; return SHD_ERR_CUDA; }
  if (prop.major != 10) {
    // The kernels are built for sm_100a only; there is no other code path.
    delete ctx;
    return SHD_ERR_UNSUPPORTED;
  }
  ctx->num_sms = prop.multiProcessorCount;
  ctx->partial_floats = partial_floats_for(ctx->num_sms);
  ctx->n_counters = 1 << 16;
  if ((e = cudaMalloc(&ctx->d_err, 16)) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  if ((e = cudaMalloc(&ctx->d_partials, ctx->partial_floats * 4)) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  if ((e = cudaMalloc(&ctx->d_counters, (size_t)ctx->n_counters * 4)) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  if ((e = cudaMemset(ctx->d_err, 0, 16)) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  if ((e = cudaMemset(ctx->d_counters, 0, (size_t)ctx->n_counters * 4)) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) { shd_destroy(ctx); return SHD_ERR_CUDA; }
  *out = ctx;
  return SHD_OK;
}

int shd_stage(shd_ctx* ctx, size_t bytes, void** out) {
  if (bytes > ctx->stage_bytes) {
    SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->d_stage);
    ctx->d_stage = nullptr;
    ctx->stage_bytes = 0;
    const size_t want = std::max<size_t>(bytes, 1 << 16);
    SHD_CHECK_CUDA(ctx, cudaMalloc(&ctx->d_stage, want));
    ctx->stage_bytes = want;
  }
  *out = ctx->d_stage;
  return SHD_OK;
}

extern "C" int shd_destroy(shd_ctx* ctx) {
  if (!ctx) return SHD_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_partials);
  cudaFree(ctx->d_counters);
  cudaFree(ctx->d_scratch64);
  cudaFree(ctx->d_stage);
  cudaFree(ctx->d_rope_cos);
  cudaFree(ctx->d_rope_sin);
  cudaFree(ctx->d_xpad);
  cudaFree(ctx->d_tc_planes);
  cudaFree(ctx->d_tc_planes_next);
  cudaFree(ctx->d_tc_ws);
  delete ctx;
  return SHD_OK;
}

extern "C" int shd_set_stream(shd_ctx* ctx, void* stream) {
  if (!ctx) return SHD_ERR_ARG;
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return SHD_OK;
}

extern "C" const char* shd_last_error(shd_ctx* ctx) {
  if (!ctx) return "null context";
  return ctx->last_error.c_str();
}

extern "C" int64_t shd_launch_count(shd_ctx* ctx) { return ctx ? ctx->launches : -1; }

// Waits on a device flag that nothing sets, for at most limit_ns of %globaltimer, then records a
// stage-fill timeout in the error word and returns, exactly as every pipeline wait does on expiry.
__global__ void wait_selftest_kernel(const int* flag, uint64_t limit_ns, int* err) {
  const uint64_t t0 = globaltimer_ns();
  while (*reinterpret_cast<const volatile int*>(flag) == 0) {
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicOr(err, SHD_DEVERR_TIMEOUT_FULL);
      return;
    }
  }
}

extern "C" int shd_wait_selftest(shd_ctx* ctx, int limit_ms) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_REQUIRE(ctx, limit_ms > 0 && limit_ms <= 2000, "shd_wait_selftest: limit_ms must be 1..2000");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  // the error word's allocation holds 4 ints; the last is a zero flag that no kernel ever sets
  const int* flag = ctx->d_err + 3;
  wait_selftest_kernel<<<1, 1, 0, ctx->stream>>>(flag, (uint64_t)limit_ms * 1000000ull, ctx->d_err);
  SHD_CHECK_LAUNCH(ctx, "wait_selftest_kernel");
  return SHD_OK;
}

extern "C" int shd_sync(shd_ctx* ctx) {
  if (!ctx) return SHD_ERR_ARG;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  int h = 0;
  SHD_CHECK_CUDA(ctx, cudaMemcpy(&h, ctx->d_err, 4, cudaMemcpyDeviceToHost));
  if (h == 0) return SHD_OK;
  // A kernel gave up: clear the word and the tile counters it may have left behind.
  SHD_CHECK_CUDA(ctx, cudaMemset(ctx->d_err, 0, 4));
  SHD_CHECK_CUDA(ctx, cudaMemset(ctx->d_counters, 0, (size_t)ctx->n_counters * 4));
  SHD_CHECK_CUDA(ctx, cudaDeviceSynchronize());
  char buf[160];
  snprintf(buf, sizeof buf, "device error word 0x%x (%s%s%s%s%s)", h,
           (h & SHD_DEVERR_TIMEOUT_FULL) ? "stage-fill timeout " : "",
           (h & SHD_DEVERR_TIMEOUT_EMPTY) ? "stage-drain timeout " : "",
           (h & SHD_DEVERR_TIMEOUT_DRAIN) ? "abort-drain timeout " : "",
           (h & SHD_DEVERR_NONFINITE) ? "non-finite logit " : "",
           (h & SHD_DEVERR_ARG) ? "index out of range" : "");
  if (h & (SHD_DEVERR_TIMEOUT_FULL | SHD_DEVERR_TIMEOUT_EMPTY | SHD_DEVERR_TIMEOUT_DRAIN))
    return shd_fail(ctx, SHD_ERR_TIMEOUT, buf);
  if (h & SHD_DEVERR_NONFINITE) return shd_fail(ctx, SHD_ERR_NUMERIC, buf);
  return shd_fail(ctx, SHD_ERR_ARG, buf);
}

// ------------------------------------------------------------------------------------------------
// Weight tiling
// ------------------------------------------------------------------------------------------------

// Source row of tile row r of tile t for a row order.
__device__ __forceinline__ int tiled_source_row(int rows, int head_dim, int np) {
  if (rows == SHD_ROWS_QKV) {
    // pair (p, p + head_dim/2) of each head stored adjacently
    const int head = np / head_dim, j = np % head_dim;
    return head * head_dim + ((j & 1) ? (j >> 1) + head_dim / 2 : (j >> 1));
  }
  return np;
}

// GATEUP: tile t rows 0..15 = gate rows 16t..16t+15, rows 16..31 = up rows 16t..16t+15.
__device__ __forceinline__ int gateup_source_row(int I, int np) {
  const int t = np / kTileRows, r = np % kTileRows;
  return (r < 16) ? (t * 16 + r) : (I + t * 16 + (r - 16));
}

// One thread per 8 bf16 (16 bytes) of the tiled output.
__global__ void tile_bf16_kernel(const uint16_t* __restrict__ src, int N, int K, int nT, int nKC,
                                 int rows, int head_dim, uint16_t* __restrict__ dst,
                                 const float* __restrict__ bias_src, float* __restrict__ bias_dst) {
  const long long total = (long long)nT * nKC * (kBlockBytes / 16);
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const long long blk = v / (kBlockBytes / 16);
    const int within = (int)(v % (kBlockBytes / 16));  // 0..1023
    const int r = within / 32, lane = within % 32;
    const int t = (int)(blk / nKC), c = (int)(blk % nKC);
    const int np = t * kTileRows + r;
    int n = -1;
    if (rows == SHD_ROWS_GATEUP) {
      if (np < N) n = gateup_source_row(N / 2, np);
    } else if (np < N) {
      n = tiled_source_row(rows, head_dim, np);
    }
    uint16_t out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = c * kChunkBf16 + ((j < 4) ? (4 * lane + j) : (128 + 4 * lane + j - 4));
      out[j] = (n >= 0 && col < K) ? src[(size_t)n * K + col] : (uint16_t)0;
    }
    uint4 pk;
    pk.x = (uint32_t)out[0] | ((uint32_t)out[1] << 16);
    pk.y = (uint32_t)out[2] | ((uint32_t)out[3] << 16);
    pk.z = (uint32_t)out[4] | ((uint32_t)out[5] << 16);
    pk.w = (uint32_t)out[6] | ((uint32_t)out[7] << 16);
    reinterpret_cast<uint4*>(dst)[v] = pk;
    if (bias_dst && c == 0 && lane == 0) bias_dst[np] = (n >= 0 && bias_src) ? bias_src[n] : 0.0f;
  }
}

// f32 [in][out] host layout -> bf16 [out][in]; flags values that are not exact bf16 upcasts.
__global__ void f32_in_out_to_bf16_kernel(const float* __restrict__ w, int in, int out,
                                          uint16_t* __restrict__ dst, int* __restrict__ lossy) {
  const long long total = (long long)in * out;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(v / out), j = (int)(v % out);
    const uint32_t b = __float_as_uint(w[v]);
    if (b & 0xffffu) atomicOr(lossy, 1);
    dst[(size_t)j * in + i] = (uint16_t)(b >> 16);
  }
}

// i32 [in][out] -> tiled [32 rows][128 cols] blocks (rows = output features).
__global__ void tile_i32_kernel(const int32_t* __restrict__ w, int in, int out, int nT, int nKC,
                                int32_t* __restrict__ dst) {
  const long long total = (long long)nT * nKC * (kBlockBytes / 4);
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const long long blk = v / (kBlockBytes / 4);
    const int within = (int)(v % (kBlockBytes / 4));  // 0..4095
    const int r = within / kChunkI32, col = within % kChunkI32;
    const int t = (int)(blk / nKC), c = (int)(blk % nKC);
    const int n = t * kTileRows + r, k = c * kChunkI32 + col;
    dst[v] = (n < out && k < in) ? w[(size_t)k * out + n] : 0;
  }
}

static int grid_for(long long work, int sms) {
  long long g = (work + 255) / 256;
  if (g > (long long)sms * 16) g = (long long)sms * 16;
  return (int)(g < 1 ? 1 : g);
}

extern "C" int shd_weight_from_bf16(shd_ctx* ctx, const uint16_t* w_out_in_dev, const float* bias_dev,
                                    int in_features, int out_features, int rows, int head_dim,
                                    shd_weight** out) {
  if (!ctx || !out) return SHD_ERR_ARG;
  *out = nullptr;
  SHD_REQUIRE(ctx, w_out_in_dev, "shd_weight_from_bf16: null weight");
  SHD_REQUIRE(ctx, in_features > 0 && out_features > 0, "shd_weight_from_bf16: empty shape");
  SHD_REQUIRE(ctx, rows == SHD_ROWS_PLAIN || rows == SHD_ROWS_QKV || rows == SHD_ROWS_GATEUP,
              "shd_weight_from_bf16: unknown row order");
  if (rows == SHD_ROWS_QKV)
    SHD_REQUIRE(ctx, head_dim > 0 && head_dim % 32 == 0 && out_features % head_dim == 0,
                "shd_weight_from_bf16: QKV rows need head_dim % 32 == 0 dividing out_features");
  if (rows == SHD_ROWS_GATEUP)
    SHD_REQUIRE(ctx, out_features % 32 == 0, "shd_weight_from_bf16: GATEUP needs intermediate % 16 == 0");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  shd_weight* w = new shd_weight();
  w->ctx = ctx;
  w->kind = WK_BF16;
  w->N = out_features;
  w->K = in_features;
  w->nT = (out_features + kTileRows - 1) / kTileRows;
  w->nKC = (in_features + kChunkBf16 - 1) / kChunkBf16;
  w->rows = rows;
  w->head_dim = head_dim;
  w->bytes = (int64_t)w->nT * w->nKC * kBlockBytes;
  cudaError_t e = cudaMalloc(&w->d_tiles, (size_t)w->bytes);
  if (e != cudaSuccess) { delete w; return shd_cuda_fail(ctx, e, "cudaMalloc(weight tiles)"); }
  if (bias_dev) {
    e = cudaMalloc(&w->d_bias, (size_t)w->nT * kTileRows * 4);
    if (e != cudaSuccess) { shd_weight_destroy(w); return shd_cuda_fail(ctx, e, "cudaMalloc(bias)"); }
  }
  const long long work = (long long)w->nT * w->nKC * (kBlockBytes / 16);
  tile_bf16_kernel<<<grid_for(work, ctx->num_sms), 256, 0, ctx->stream>>>(
      w_out_in_dev, out_features, in_features, w->nT, w->nKC, rows, head_dim,
      reinterpret_cast<uint16_t*>(w->d_tiles), bias_dev, w->d_bias);
  e = cudaGetLastError();
  if (e != cudaSuccess) { shd_weight_destroy(w); return shd_cuda_fail(ctx, e, "tile_bf16_kernel"); }
  ctx->launches++;
  // the tiles are complete when the call returns, so any stream may use the weight afterwards
  e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) { shd_weight_destroy(w); return shd_cuda_fail(ctx, e, "tile_bf16_kernel"); }
  *out = w;
  return SHD_OK;
}

extern "C" int shd_weight_upload_f32_as_bf16(shd_ctx* ctx, const float* w_in_out_host, int in_features,
                                             int out_features, shd_weight** out) {
  if (!ctx || !out) return SHD_ERR_ARG;
  *out = nullptr;
  SHD_REQUIRE(ctx, w_in_out_host, "shd_weight_upload_f32_as_bf16: null weight");
  SHD_REQUIRE(ctx, in_features > 0 && out_features > 0, "shd_weight_upload_f32_as_bf16: empty shape");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const size_t n = (size_t)in_features * out_features;
  float* d_f32 = nullptr;
  uint16_t* d_bf = nullptr;
  int* d_lossy = nullptr;
  int rc = SHD_OK;
  cudaError_t e;
  if ((e = cudaMalloc(&d_f32, n * 4)) != cudaSuccess) return shd_cuda_fail(ctx, e, "cudaMalloc(f32 staging)");
  if ((e = cudaMalloc(&d_bf, n * 2)) != cudaSuccess) { cudaFree(d_f32); return shd_cuda_fail(ctx, e, "cudaMalloc(bf16 staging)"); }
  if ((e = cudaMalloc(&d_lossy, 4)) != cudaSuccess) { cudaFree(d_f32); cudaFree(d_bf); return shd_cuda_fail(ctx, e, "cudaMalloc"); }
  int lossy = 0;
  e = cudaMemcpyAsync(d_f32, w_in_out_host, n * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_lossy, 0, 4, ctx->stream);
  if (e == cudaSuccess) {
    f32_in_out_to_bf16_kernel<<<grid_for((long long)n, ctx->num_sms), 256, 0, ctx->stream>>>(
        d_f32, in_features, out_features, d_bf, d_lossy);
    e = cudaGetLastError();
    ctx->launches++;
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&lossy, d_lossy, 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    rc = shd_cuda_fail(ctx, e, "shd_weight_upload_f32_as_bf16");
  } else if (lossy) {
    rc = shd_fail(ctx, SHD_ERR_UNSUPPORTED,
                  "shd_weight_upload_f32_as_bf16: weight has values that are not exact bf16 upcasts");
  } else {
    rc = shd_weight_from_bf16(ctx, d_bf, nullptr, in_features, out_features, SHD_ROWS_PLAIN, 0, out);
    if (rc == SHD_OK) {
      e = cudaStreamSynchronize(ctx->stream);
      if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "tiling");
    }
  }
  cudaFree(d_f32);
  cudaFree(d_bf);
  cudaFree(d_lossy);
  return rc;
}

extern "C" int shd_weight_upload_i32(shd_ctx* ctx, const int32_t* w_in_out_host, const int32_t* bias_host,
                                     int in_features, int out_features, shd_weight** out) {
  if (!ctx || !out) return SHD_ERR_ARG;
  *out = nullptr;
  SHD_REQUIRE(ctx, w_in_out_host, "shd_weight_upload_i32: null weight");
  SHD_REQUIRE(ctx, in_features > 0 && out_features > 0, "shd_weight_upload_i32: empty shape");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  shd_weight* w = new shd_weight();
  w->ctx = ctx;
  w->kind = WK_I32;
  w->N = out_features;
  w->K = in_features;
  w->nT = (out_features + kTileRows - 1) / kTileRows;
  w->nKC = (in_features + kChunkI32 - 1) / kChunkI32;
  w->bytes = (int64_t)w->nT * w->nKC * kBlockBytes;
  const size_t n = (size_t)in_features * out_features;
  int32_t* d_src = nullptr;
  cudaError_t e = cudaMalloc(&w->d_tiles, (size_t)w->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&d_src, n * 4);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_src, w_in_out_host, n * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess && bias_host) {
    e = cudaMalloc(&w->d_bias_i32, (size_t)out_features * 4);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(w->d_bias_i32, bias_host, (size_t)out_features * 4, cudaMemcpyHostToDevice, ctx->stream);
  }
  if (e == cudaSuccess) {
    const long long work = (long long)w->nT * w->nKC * (kBlockBytes / 4);
    tile_i32_kernel<<<grid_for(work, ctx->num_sms), 256, 0, ctx->stream>>>(
        d_src, in_features, out_features, w->nT, w->nKC, reinterpret_cast<int32_t*>(w->d_tiles));
    e = cudaGetLastError();
    ctx->launches++;
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFree(d_src);
  if (e != cudaSuccess) {
    shd_weight_destroy(w);
    return shd_cuda_fail(ctx, e, "shd_weight_upload_i32");
  }
  *out = w;
  return SHD_OK;
}

extern "C" int shd_weight_destroy(shd_weight* w) {
  if (!w) return SHD_OK;
  if (w->ctx) cudaSetDevice(w->ctx->device);
  cudaFree(w->d_tiles);
  cudaFree(w->d_bias);
  cudaFree(w->d_bias_i32);
  shd::free_weight_map(w);
  delete w;
  return SHD_OK;
}

extern "C" int64_t shd_weight_device_bytes(const shd_weight* w) { return w ? w->bytes : -1; }
