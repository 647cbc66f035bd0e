// Allocation-free variant of the dual-share f32 linear layer.
//
// Some callers cannot allocate device memory when they run a layer: code inside a region whose
// allocator is owned and frozen by a host framework (a serving engine that reserves the GPU's
// memory up front), or code that must not trigger an allocation mid-request. For them this entry
// point runs the same split-K GEMV as shd_linear_dual_f32 but takes its scratch -- split-tile
// partial sums, tile arrival counters and the error word -- from the file-scope device array below
// instead of the context's allocations. It calls no cudaMalloc, cudaFree or other allocating routine.
//
// Limits: at most kNaMaxTiles row tiles (out_features <= 262144), two CTAs per SM on at most 160
// SMs, rows 16-byte aligned (in_features % 4 == 0), M processed in groups of 8. The array occupies
// kNaScratchFloats * 4 bytes (about 1.3 MB) on every GPU that loads the library, until the process
// exits. Every call shares it and it keeps the last call's contents; the tile counters, which must
// start at zero, are cleared on the caller's stream at the start of each call. Calls that overlap
// on the GPU (different streams, or different host threads without ordering) race on it.
//
// Set-up: the first call on a device, with that device current, looks up the array's device
// address (cudaGetSymbolAddress; the host-side name is only a stand-in). With lazy module loading
// that lookup or the first launch may load the library's module and place the array in device
// memory, so make one call per device before the host framework freezes device memory and before
// any stream capture. Device-side wait timeouts set the array's error word, which this entry point
// does not read back: they are not reported.
#include <mutex>

#include "shd_gemv.cuh"

namespace {

constexpr int kNaMaxCtas = 2 * 160;   // two CTAs per SM, up to 160 SMs
constexpr int kNaMaxRowsPerLaunch = 8;
constexpr int kNaMaxTiles = 8192;     // row tiles of 32 outputs
constexpr size_t kNaPartialFloats =
    (size_t)kNaMaxCtas * 2 * shd::kTileRows * 2 * kNaMaxRowsPerLaunch;  // 2 slots per CTA
constexpr size_t kNaScratchFloats = kNaPartialFloats + kNaMaxTiles + 64;

}  // namespace

// [partials: kNaPartialFloats][counters: kNaMaxTiles ints][error word + padding: 64]
static __device__ __align__(256) float g_noalloc_scratch[kNaScratchFloats];

namespace {

struct DeviceScratch {
  float* base = nullptr;  // device address of g_noalloc_scratch on that device
  int sms = 0;
};

std::mutex g_mu;
DeviceScratch g_dev[64];

// Once per device, with the device current: the symbol's device address (the host-side name of
// the array is only a stand-in and must never be passed to a kernel) and the SM count.
int device_scratch(int dev, DeviceScratch* out) {
  if (dev < 0 || dev >= 64) return SHD_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dev[dev].base) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return SHD_ERR_CUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return SHD_ERR_CUDA;
    if (2 * sms > kNaMaxCtas) return SHD_ERR_UNSUPPORTED;
    g_dev[dev].base = static_cast<float*>(p);
    g_dev[dev].sms = sms;
  }
  *out = g_dev[dev];
  return SHD_OK;
}

}  // namespace

using namespace shd;

extern "C" int shd_linear_dual_f32_noalloc(const shd_weight* w, const float* bias, const float* xc,
                                           const float* xs, float* yc, float* ys, int M,
                                           const float* residual_c, const float* residual_s,
                                           void* stream) {
  if (!w || w->kind != WK_BF16 || w->rows != SHD_ROWS_PLAIN || !w->ctx) return SHD_ERR_ARG;
  if (M < 0) return SHD_ERR_ARG;
  if (M == 0) return SHD_OK;
  if (!xc || !xs || !yc || !ys) return SHD_ERR_ARG;
  if ((residual_c == nullptr) != (residual_s == nullptr)) return SHD_ERR_ARG;
  // no staging buffer can be allocated here: inputs must already be 16-byte aligned rows
  if (w->K % 4 != 0 || !shd_aligned16(xc) || !shd_aligned16(xs)) return SHD_ERR_ARG;
  if (w->nT > kNaMaxTiles) return SHD_ERR_ARG;  // out_features beyond the scratch maximum
  const int dev = w->ctx->device;
  if (cudaSetDevice(dev) != cudaSuccess) return SHD_ERR_CUDA;
  DeviceScratch ds;
  const int rc0 = device_scratch(dev, &ds);
  if (rc0) return rc0;
  float* partials = ds.base;
  int* counters = reinterpret_cast<int*>(ds.base + kNaPartialFloats);
  int* err = reinterpret_cast<int*>(ds.base + kNaPartialFloats + kNaMaxTiles);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counters, 0, (size_t)w->nT * sizeof(int), s) != cudaSuccess) return SHD_ERR_CUDA;
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) return SHD_ERR_CUDA;
  // a context on the stack that points at the static scratch (no device memory of its own)
  shd_ctx tmp;
  tmp.device = dev;
  tmp.stream = s;
  tmp.num_sms = ds.sms;
  tmp.d_partials = partials;
  tmp.partial_floats = kNaPartialFloats;
  tmp.d_counters = counters;
  tmp.n_counters = kNaMaxTiles;
  tmp.d_err = err;
  for (int m0 = 0; m0 < M;) {
    const int mm = (M - m0) >= kNaMaxRowsPerLaunch ? kNaMaxRowsPerLaunch : (M - m0);
    GemvArgs a{};
    a.Xc = xc + (size_t)m0 * w->K;
    a.Xs = xs + (size_t)m0 * w->K;
    a.ldx = w->K;
    a.bias = bias ? bias : w->d_bias;
    a.Rc = residual_c ? residual_c + (size_t)m0 * w->N : nullptr;
    a.Rs = residual_s ? residual_s + (size_t)m0 * w->N : nullptr;
    a.ldr = w->N;
    a.Yc = yc + (size_t)m0 * w->N;
    a.Ys = ys + (size_t)m0 * w->N;
    a.ldy = w->N;
    const int rc = launch_gemv_f32(&tmp, w, mm, EPI_STORE, a);
    if (rc) {
      w->ctx->last_error = tmp.last_error;  // readable through shd_last_error(weight's context)
      return rc;
    }
    m0 += mm;
  }
  return SHD_OK;
}
