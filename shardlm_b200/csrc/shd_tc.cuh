// Tensor-core (tcgen05) dual-share linear for many token rows.
#pragma once

#include "shd_gemv.cuh"

namespace shd {

// Token rows per output tile for M rows (8, 16, 32 or 64).
int tc_token_tile(int M);
// Y shares of M rows through the tensor cores with the epilogue `epi` (EPI_STORE, EPI_QKV or
// EPI_GATEUP; same GemvArgs fields as launch_gemv_f32 with staged activations Xc/Xs/ldx).
int launch_linear_tc(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs g);
// Release the weight's cached tensor map.
void free_weight_map(shd_weight* w);

}  // namespace shd
