// Internal interface of the dual-share GEMV family (used by the C ABI and by the model loop).
#pragma once

#include "shd_common.cuh"
#include "shd_p2p.cuh"

namespace shd {

constexpr int kTileRows = 32;          // weight rows per tile
constexpr int kChunkBf16 = 256;        // bf16 columns per chunk (16 KB block)
constexpr int kChunkI32 = 128;         // i32 columns per chunk (16 KB block)
constexpr int kBlockBytes = 16384;     // one tiled weight block = one pipeline stage of weights
constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;

enum WeightKind { WK_BF16 = 0, WK_I32 = 1 };

// Epilogues of the f32-share GEMV.
enum Epi {
  EPI_STORE = 0,   // yc = acc_c (+rc), ys = acc_s + bias (+rs)
  EPI_QKV = 1,     // bias, RoPE per share on q/k, reconstruct; q -> Q, k/v -> KV cache
  EPI_GATEUP = 2,  // reconstruct gate/up, SwiGLU, reshare (y - mask, mask)
  EPI_LOGITS = 3,  // logit shares out + fused greedy argmax (last index among equal maxima)
};

}  // namespace shd

struct shd_weight {
  shd_ctx* ctx = nullptr;
  int kind = shd::WK_BF16;
  int N = 0, K = 0;        // logical out, in
  int nT = 0, nKC = 0;     // tiles, chunks
  int rows = SHD_ROWS_PLAIN;
  int head_dim = 0;
  void* d_tiles = nullptr;  // nT * nKC blocks of 16 KB
  float* d_bias = nullptr;  // f32 bias in tile row order (nT*32), nullable
  int32_t* d_bias_i32 = nullptr;
  int64_t bytes = 0;
  void* tmap = nullptr;     // host copy of the TMA tensor map of the blocks (tensor-core path)
};

namespace shd {

struct GemvArgs {
  const uint8_t* W;
  int N, K, nT, nKC;
  const float* Xc;
  const float* Xs;
  int ldx;
  // EPI_STORE
  const float* bias;  // tile row order
  const float* Rc;
  const float* Rs;
  int ldr;
  float* Yc;
  float* Ys;
  int ldy;
  // EPI_QKV
  int q_dim, kv_dim, head_dim;
  const float* rope_cos;  // [max_seq][head_dim/2]
  const float* rope_sin;
  int rope_max_seq;
  const int* pos;  // [M] positions
  const int* seq;  // [M] sequence slots (nullable -> 0)
  float* Q;
  int ldq;
  float* Kcache;
  float* Vcache;
  int64_t kv_seq_stride;  // floats between sequence slots in the cache
  // EPI_GATEUP
  int variant;
  const float* mask;  // [M][N/2], nullable
  int ldmask;
  // EPI_LOGITS
  unsigned long long* amax;  // [M]
  int idx_offset;            // global index of local row 0 (vocabulary-parallel lm_head)
  // RMSNorm prologue (norm = true at launch): x = reshare(RMSNorm(D + H)) computed per CTA into
  // shared memory; Xc/Xs are then unused.
  const float* nHc;  // residual stream shares [M][n_ldh]
  const float* nHs;
  const float* nDc;  // sublayer output shares added first (nullable)
  const float* nDs;
  float* nHout_c;    // h = D + H written by CTA 0 (nullable)
  float* nHout_s;
  int n_ldh;
  const float* gamma;
  float eps;
  int nvariant;
  const float* nmask;  // reshare mask [M][n_ldmask] (nullable)
  int n_ldmask;
  // scratch
  float* partials;
  int* counters;
  int* err;
  int nstages;  // pipeline depth (set by the launcher)
  // Tensor-parallel push (EPI_STORE, when tp_peer[0] is set): every output value goes, as one
  // 8-byte {float bits, call epoch} store, into this rank's source slot of every rank's receive
  // buffer (shd_p2p.cuh) at its index in the packed [2][M][ldy] message, instead of to Yc/Ys; the
  // receive kernel of the same call sums the sources.
  uint8_t* tp_peer[8];
  int tp_me, tp_world;
  unsigned long long* trace;  // launch timeline slot (nullable; TraceField in shd_common.cuh)
};

// Launch shape of the f32-share GEMV (what launch_gemv_f32 will launch for these rows).
struct GemvPlan {
  int per_sm;     // CTAs per SM (1 or 2)
  int G;          // CTAs
  int nstages;    // pipeline stages of 16 KB weight blocks
  long long U;    // (tile, chunk) units, CTA g taking [U g / G, U (g + 1) / G)
  size_t smem;
};
GemvPlan gemv_plan(const shd_ctx* ctx, const shd_weight* w, int M, bool norm);

// Launch the f32-share GEMV for M rows with the given epilogue; `norm` selects the fused RMSNorm
// prologue (x from nHc/nHs/...) instead of staged activations (Xc/Xs).
int launch_gemv_f32(shd_ctx* ctx, const shd_weight* w, int M, int epi, GemvArgs a, bool norm = false);
// Fill the weight, shape and scratch fields of `a` for `w` (what launch_gemv_f32 adds before a
// launch; the tensor-core linear uses it for its split-K scratch too).
int gemv_prepare(shd_ctx* ctx, const shd_weight* w, GemvArgs& a, bool norm);

struct RingArgs {
  const uint8_t* W;
  int N, K, nT, nKC;
  const int32_t* Xc;
  const int32_t* Xs;
  int ldx;
  const int32_t* bias;  // nullable, [N]
  int32_t* Yc;
  int32_t* Ys;
  int ldy;
  int scale;
  long long* partials;
  int* counters;
  int* err;
};

int launch_gemv_ring(shd_ctx* ctx, const shd_weight* w, int M, RingArgs a);

}  // namespace shd
