// Tensor-core (tcgen05) dual-share linear for many token rows.
#pragma once

#include "shd_gemv.cuh"

namespace shd {

// Rows from which the tensor cores beat the CUDA-core GEMV (whose arithmetic per weight byte grows
// with the rows until it is no longer bandwidth-bound).
constexpr int kTcMinRows = 5;

// Token rows per output tile for M rows (16 or 32).
int tc_token_tile(int M);
// Y shares of M rows through the tensor cores with the epilogue `epi` (EPI_STORE, EPI_QKV or
// EPI_GATEUP; same GemvArgs fields as launch_gemv_f32 with staged activations Xc/Xs/ldx).
int launch_linear_tc(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs g);
// Release the weight's cached tensor map.
void free_weight_map(shd_weight* w);

}  // namespace shd
