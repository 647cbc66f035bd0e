// Tensor-core (tcgen05) dual-share linear for many token rows.
#pragma once

#include "shd_gemv.cuh"
#include "shd_nonlinear.cuh"
#include "shd_planes.cuh"

namespace shd {

// Whether M rows of a linear with weight w go to the tensor cores rather than the CUDA-core GEMV.
// The GEMV's arithmetic per weight byte grows with the rows. Measured on B200: from 5 rows the
// 16-row tensor-core tiles are at least as fast for every projection; at 3-4 rows only for the large
// ones (gate/up, down: >= 48 M weights), the small latency-bound ones (q/k/v, o) stay on the GEMV.
inline bool tc_preferred(const shd_weight* w, int M) {
  if (M >= 5) return true;
  return M >= 3 && (long long)w->N * w->K >= 48ll * 1024 * 1024;
}

// Token rows per output tile for M rows (8, 16 or 32).
int tc_token_tile(int M);

// The planes of a tensor-core linear of w over M rows, for the kernel producing its input to write
// instead of f32 shares: empty when the linear does not run on the tensor cores, or when M rows do
// not fill whole token tiles or in_features is not a multiple of 256 (padding would need zeroing).
// Sizes the shared planes buffer, so call it before enqueuing the producer.
PlaneOut tc_input_planes(shd_ctx* ctx, const shd_weight* w, int M);
// Y shares of M rows through the tensor cores with the epilogue `epi` (EPI_STORE, EPI_QKV,
// EPI_GATEUP or EPI_LOGITS; same GemvArgs fields as launch_gemv_f32 with staged activations
// Xc/Xs/ldx). With `norm`, the activations are instead reshare(RMSNorm(D + H)) of its fields
// (n = in_features; its Xc/Xs are not written), computed by the kernel that splits the bf16 planes.
// planes_ready: the planes were written by the producing kernel (tc_input_planes); out_planes
// (EPI_GATEUP): write the output as the next linear's planes when the epilogue runs in the split-K
// reduce kernel, i.e. after this linear has read its own planes; *wrote_out says whether it did.
int launch_linear_tc(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs g, const NormArgs* norm = nullptr,
                     bool planes_ready = false, const PlaneOut* out_planes = nullptr, bool* wrote_out = nullptr);
// Release the weight's cached tensor map.
void free_weight_map(shd_weight* w);

}  // namespace shd
