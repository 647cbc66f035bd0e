// Tensor-core (tcgen05) dual-share linear for many token rows.
#pragma once

#include "shd_gemv.cuh"
#include "shd_nonlinear.cuh"

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
// Y shares of M rows through the tensor cores with the epilogue `epi` (EPI_STORE, EPI_QKV,
// EPI_GATEUP or EPI_LOGITS; same GemvArgs fields as launch_gemv_f32 with staged activations
// Xc/Xs/ldx). With `norm`, the activations are instead reshare(RMSNorm(D + H)) of its fields
// (n = in_features; its Xc/Xs are not written), computed by the kernel that splits the bf16 planes.
int launch_linear_tc(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs g, const NormArgs* norm = nullptr);
// Release the weight's cached tensor map.
void free_weight_map(shd_weight* w);

}  // namespace shd
