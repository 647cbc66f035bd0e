// Whole-model secret-shared forward pass: the per-token layer loop of the reference
// (batched_full_forward_gpu / generate_token_gpu, crates/v2/server/src/routes/secure_inference.rs:
// 1553-1796; batched_prefill_gpu_v3, :2299-2632; mpc_prefill, routes/secure_inference_mpc.rs:
// 163-562), run entirely on the device:
//
//   h = H + D                      (residual of the previous sublayer, per share)
//   x = reshare(RMSNorm(h_c+h_s))  norm_reshare_kernel
//   q,k,v shares = x W_qkv^T + b   gemv EPI_QKV: one weight pass for both shares; RoPE per share;
//                                  q reconstructed, k/v reconstructed into the KV cache
//   a = reshare(attn(q, K, V))     attn_decode_kernel (split-K, deterministic combine)
//   D = a W_o^T                    gemv EPI_STORE            [TP: all-reduce D, both shares]
//   h' = h + D; x = norm(h')       norm_reshare_kernel
//   act = reshare(silu(g) u)       gemv EPI_GATEUP (gate/up interleaved per tile)
//   D = act W_down^T               gemv EPI_STORE            [TP: all-reduce D]
//   final norm, logits shares, greedy argmax (gemv EPI_LOGITS)  [TP: all-reduce max of keys]
//
// Activations are [2][M][width] per buffer (client rows, then server rows), so one collective
// covers both shares. Decode steps for all active slots are captured once into a CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "shd_gemv.cuh"
#include "shd_model.cuh"
#include "shd_tc.cuh"
#include "shd_nonlinear.cuh"

using namespace shd;


namespace {

constexpr int kMaxRows = 8;        // decode batch (sequence slots stepped together)
constexpr int kPrefillRows = 512;  // prompt positions per prefill chunk
constexpr int kAttnWideRows = 4;   // from this many rows, attention groups of up to 8 q heads
constexpr int kFlashRows = 16;     // prompt blocks of this many rows and more: tensor-core attention

// Decode bookkeeping after the logits: tokens = keys, history row, position advance. It does not
// release its dependents early: the next step's kernels all start after it has completed, so the
// positions it writes (and every K/V row of earlier steps) may be read before their own waits.
__global__ void finish_step_kernel(const unsigned long long* keys, int* tokens, int* pos, int* hist,
                                   int hist_cap, unsigned long long* step, int M) {
  pdl_wait();  // the argmax keys come from the lm_head kernel
  const int m = threadIdx.x;
  const unsigned long long s = *step;
  if (m < M) {
    const int tok = (int)(keys[m] & 0xffffffffu);
    tokens[m] = tok;
    hist[(size_t)(s % hist_cap) * M + m] = tok;
    pos[m] += 1;
  }
  __syncthreads();
  if (m == 0) *step = s + 1;
}

__global__ void concat_rows_kernel(const uint16_t* a, long long na, const uint16_t* b, long long nb,
                                   const uint16_t* c, long long nc, uint16_t* out) {
  const long long n = na + nb + nc;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = i < na ? a[i] : (i < na + nb ? b[i - na] : c[i - na - nb]);
}

__global__ void concat_f32_kernel(const float* a, int na, const float* b, int nb, const float* c,
                                  int nc, float* out) {
  const int n = na + nb + nc;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = i < na ? (a ? a[i] : 0.f) : (i < na + nb ? (b ? b[i - na] : 0.f) : (c ? c[i - na - nb] : 0.f));
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Tensor-parallel plan: q heads split evenly (remainder to the first ranks); each rank keeps the kv
// heads its q heads use; intermediate split in blocks of 16; vocabulary split evenly.
// ------------------------------------------------------------------------------------------------
static void make_plan(const shd_model_config& c, shd_shard_info& s) {
  const int W = std::max(1, c.tp_world), r = c.tp_rank;
  auto split = [&](int n, int unit, int& b, int& cnt) {
    const int blocks = n / unit;
    const int b0 = (int)((long long)blocks * r / W), b1 = (int)((long long)blocks * (r + 1) / W);
    b = b0 * unit;
    cnt = (r == W - 1) ? n - b : (b1 - b0) * unit;
  };
  split(c.n_heads, 1, s.q_head_begin, s.q_head_count);
  const int group = c.n_heads / c.n_kv_heads;
  if (s.q_head_count > 0) {
    s.kv_head_begin = s.q_head_begin / group;
    s.kv_head_count = (s.q_head_begin + s.q_head_count - 1) / group - s.kv_head_begin + 1;
  } else {
    s.kv_head_begin = 0;
    s.kv_head_count = 0;
  }
  split(c.intermediate, 16, s.inter_begin, s.inter_count);
  split(c.vocab, 1, s.vocab_begin, s.vocab_count);
}

int shd_model::use_stream() {
  saved_stream = ctx->stream;
  ctx->stream = stream;
  return SHD_OK;
}

void shd_model::restore_stream() { ctx->stream = saved_stream; }

// Order the model stream after the caller's stream (entry) and the caller's after ours (exit).
int shd_model::enter() {
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  SHD_CHECK_CUDA(ctx, cudaEventRecord(ev_in, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamWaitEvent(stream, ev_in, 0));
  use_stream();
  return SHD_OK;
}

int shd_model::leave(int rc) {
  restore_stream();
  if (cudaEventRecord(ev_out, stream) == cudaSuccess) cudaStreamWaitEvent(ctx->stream, ev_out, 0);
  return rc;
}

extern "C" int shd_model_create(shd_ctx* ctx, const shd_model_config* cfg, shd_model** out) {
  if (!ctx || !cfg || !out) return SHD_ERR_ARG;
  *out = nullptr;
  const shd_model_config& c = *cfg;
  SHD_REQUIRE(ctx, c.hidden > 0 && c.n_layers > 0 && c.n_heads > 0 && c.n_kv_heads > 0 &&
                       c.intermediate > 0 && c.vocab > 0,
              "shd_model_create: empty dimension");
  SHD_REQUIRE(ctx, c.n_heads % c.n_kv_heads == 0, "shd_model_create: n_heads % n_kv_heads != 0");
  SHD_REQUIRE(ctx, c.head_dim == 64 || c.head_dim == 128, "shd_model_create: head_dim must be 64 or 128");
  SHD_REQUIRE(ctx, c.hidden % 4 == 0, "shd_model_create: hidden % 4 != 0");
  SHD_REQUIRE(ctx, c.intermediate % 16 == 0, "shd_model_create: intermediate % 16 != 0");
  SHD_REQUIRE(ctx, c.max_batch >= 1 && c.max_batch <= kMaxRows, "shd_model_create: max_batch must be 1..8");
  SHD_REQUIRE(ctx, c.max_seq >= 1, "shd_model_create: max_seq < 1");
  SHD_REQUIRE(ctx, c.tp_world >= 1 && c.tp_rank >= 0 && c.tp_rank < c.tp_world, "shd_model_create: bad tp rank/world");
  SHD_REQUIRE(ctx, c.tp_world <= c.n_heads, "shd_model_create: more ranks than attention heads");
  for (int v : {c.variant_decode, c.variant_prefill, c.variant_attn})
    SHD_REQUIRE(ctx, v >= 0 && v <= 2, "shd_model_create: unknown nonlinear variant");
  if (c.tp_world > 1) SHD_REQUIRE(ctx, ctx->nccl_comm != nullptr, "shd_model_create: tp_world > 1 needs shd_tp_init first");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));

  shd_model* m = new shd_model();
  m->ctx = ctx;
  m->cfg = c;
  make_plan(c, m->sh);
  const int d = c.head_dim, h = c.hidden;
  m->qd = m->sh.q_head_count * d;
  m->kvd = m->sh.kv_head_count * d;
  m->I = m->sh.inter_count;
  m->V = m->sh.vocab_count;
  m->R = std::max(c.max_batch, kPrefillRows);
  m->T = c.max_seq;
  m->layers.resize(c.n_layers);
  m->len.assign(c.max_batch, 0);
  m->hist_cap = 4096;
  auto fail = [&](int rc) {
    shd_model_destroy(m);
    return rc;
  };
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming) != cudaSuccess)
    return fail(shd_fail(ctx, SHD_ERR_CUDA, "shd_model_create: stream/event creation failed"));
  int rc = build_rope_table(ctx, d, c.max_seq, c.rope_theta, &m->rope_cos, &m->rope_sin);
  if (rc) return fail(rc);
  m->owned.push_back(m->rope_cos);
  m->owned.push_back(m->rope_sin);
  const size_t R = m->R;
  const size_t kv_elems = (size_t)c.n_layers * c.max_batch * c.max_seq * std::max(m->kvd, 1);
  struct A {
    void** p;
    size_t bytes;
  } allocs[] = {
      {(void**)&m->Hbuf[0], 2 * R * h * 4},  {(void**)&m->Hbuf[1], 2 * R * h * 4},
      {(void**)&m->Dbuf, 2 * R * h * 4},     {(void**)&m->Xbuf, 2 * R * h * 4},
      {(void**)&m->Qbuf, R * std::max(m->qd, 1) * 4},
      {(void**)&m->Abuf, 2 * R * std::max(m->qd, 1) * 4},
      {(void**)&m->ACTbuf, 2 * R * std::max(m->I, 1) * 4},
      {(void**)&m->LOGbuf, 2 * (size_t)std::max(m->V, 1) * 4},
      {(void**)&m->LOGfull, c.tp_world > 1 ? 2 * (size_t)c.vocab * 4 : 16},
      {(void**)&m->kcache, kv_elems * 4},    {(void**)&m->vcache, kv_elems * 4},
      {(void**)&m->tokens, R * 4},           {(void**)&m->pos, R * 4},
      {(void**)&m->seq, R * 4},              {(void**)&m->p_pos, R * 4},
      {(void**)&m->p_seq, R * 4},            {(void**)&m->p_tokens, R * 4},
      {(void**)&m->amax, R * 8},             {(void**)&m->step, 8},
      {(void**)&m->hist, (size_t)m->hist_cap * c.max_batch * 4},
      {(void**)&m->final_norm, (size_t)h * 4},
  };
  for (auto& a : allocs) {
    cudaError_t e = cudaMalloc(a.p, a.bytes);
    if (e != cudaSuccess) return fail(shd_cuda_fail(ctx, e, "shd_model_create: cudaMalloc"));
    m->owned.push_back(*a.p);
  }
  for (auto& L : m->layers) {
    cudaError_t e = cudaMalloc(&L.g1, (size_t)h * 4);
    if (e == cudaSuccess) {
      m->owned.push_back(L.g1);
      e = cudaMalloc(&L.g2, (size_t)h * 4);
    }
    if (e != cudaSuccess) return fail(shd_cuda_fail(ctx, e, "shd_model_create: cudaMalloc(norm)"));
    m->owned.push_back(L.g2);
  }
  // sequence-slot map and attention head groups (q heads sharing a kv head, <= 8 per group)
  std::vector<int> seqv(R);
  for (size_t i = 0; i < R; ++i) seqv[i] = (int)i;
  const int group = c.n_heads / c.n_kv_heads;
  const std::vector<int4> groups = attn_groups(m->sh.q_head_begin, m->sh.q_head_count, m->sh.kv_head_begin, group);
  m->n_groups = (int)groups.size();
  cudaError_t e = cudaMemcpy(m->seq, seqv.data(), R * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&m->attn_groups_dev, groups.size() * sizeof(int4) + 16);
  if (e == cudaSuccess) {
    m->owned.push_back(m->attn_groups_dev);
    e = cudaMemcpy(m->attn_groups_dev, groups.data(), groups.size() * sizeof(int4), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess && group > 4) {
    // batched launches: one group of up to 8 q heads per kv head, so every K/V row is read once
    const std::vector<int4> g8 = attn_groups(m->sh.q_head_begin, m->sh.q_head_count, m->sh.kv_head_begin, group, 8);
    m->n_groups8 = (int)g8.size();
    e = cudaMalloc(&m->attn_groups8_dev, g8.size() * sizeof(int4) + 16);
    if (e == cudaSuccess) {
      m->owned.push_back(m->attn_groups8_dev);
      e = cudaMemcpy(m->attn_groups8_dev, g8.data(), g8.size() * sizeof(int4), cudaMemcpyHostToDevice);
    }
  }
  if (e == cudaSuccess) e = cudaMemset(m->step, 0, 8);
  if (e == cudaSuccess) e = cudaMemset(m->kcache, 0, kv_elems * 4);
  if (e == cudaSuccess) e = cudaMemset(m->vcache, 0, kv_elems * 4);
  if (e != cudaSuccess) return fail(shd_cuda_fail(ctx, e, "shd_model_create: init"));
  SHD_REQUIRE(ctx, (int)R * std::max(m->n_groups, 1) <= 8192, "shd_model_create: too many head groups x rows");
  *out = m;
  return SHD_OK;
}

shd_model::~shd_model() {
  if (graph) cudaGraphExecDestroy(graph);
  for (cudaEvent_t ev : prof_events) cudaEventDestroy(ev);
  cudaFree(d_trace);
  for (auto& L : layers) {
    shd_weight_destroy(L.qkv);
    shd_weight_destroy(L.o);
    shd_weight_destroy(L.gateup);
    shd_weight_destroy(L.down);
  }
  shd_weight_destroy(lm_head);
  for (void* p : owned) cudaFree(p);
  cudaFree(embed);
  cudaFree(masks);
  if (ev_in) cudaEventDestroy(ev_in);
  if (ev_out) cudaEventDestroy(ev_out);
  if (stream) cudaStreamDestroy(stream);
}

extern "C" int shd_model_destroy(shd_model* m) {
  if (!m) return SHD_OK;
  cudaSetDevice(m->ctx->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  delete m;
  return SHD_OK;
}

extern "C" int shd_model_shard_info(const shd_model* m, shd_shard_info* out) {
  if (!m || !out) return SHD_ERR_ARG;
  *out = m->sh;
  return SHD_OK;
}

extern "C" int shd_tp_plan(const shd_model_config* cfg, shd_shard_info* out) {
  if (!cfg || !out) return SHD_ERR_ARG;
  const shd_model_config& c = *cfg;
  if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.intermediate <= 0 || c.vocab <= 0 ||
      c.n_heads % c.n_kv_heads != 0 || c.intermediate % 16 != 0 || c.tp_world < 1 ||
      c.tp_rank < 0 || c.tp_rank >= c.tp_world || c.tp_world > c.n_heads)
    return SHD_ERR_ARG;
  make_plan(c, *out);
  return SHD_OK;
}

extern "C" int shd_model_seq_len(const shd_model* m, int slot) {
  if (!m || slot < 0 || slot >= m->cfg.max_batch) return SHD_ERR_ARG;
  return m->len[slot];
}

extern "C" int shd_model_set_layer(shd_model* m, int layer, const uint16_t* wq, const uint16_t* wk,
                                   const uint16_t* wv, const uint16_t* wo, const uint16_t* wg,
                                   const uint16_t* wu, const uint16_t* wd, const float* bq,
                                   const float* bk, const float* bv, const float* g1, const float* g2) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, layer >= 0 && layer < m->cfg.n_layers, "shd_model_set_layer: layer out of range");
  SHD_REQUIRE(ctx, wq && wk && wv && wo && wg && wu && wd && g1 && g2, "shd_model_set_layer: null weight");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  auto& L = m->layers[layer];
  const int h = m->cfg.hidden, d = m->cfg.head_dim;
  const long long nq = (long long)m->qd * h, nk = (long long)m->kvd * h;
  uint16_t* tmp = nullptr;
  float* btmp = nullptr;
  const long long need = std::max(nq + 2 * nk, 2LL * m->I * h);
  SHD_CHECK_CUDA(ctx, cudaMalloc(&tmp, (size_t)need * 2));
  cudaError_t e = cudaMalloc(&btmp, (size_t)(m->qd + 2 * m->kvd) * 4);
  if (e != cudaSuccess) {
    cudaFree(tmp);
    return shd_cuda_fail(ctx, e, "cudaMalloc");
  }
  int rc = SHD_OK;
  auto cleanup = [&](int r) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    cudaFree(btmp);
    return r;
  };
  const int grid = ctx->num_sms * 4;
  concat_rows_kernel<<<grid, 256, 0, ctx->stream>>>(wq, nq, wk, nk, wv, nk, tmp);
  concat_f32_kernel<<<8, 256, 0, ctx->stream>>>(bq, m->qd, bk, m->kvd, bv, m->kvd, btmp);
  if ((e = cudaGetLastError()) != cudaSuccess) return cleanup(shd_cuda_fail(ctx, e, "concat qkv"));
  shd_weight_destroy(L.qkv);
  L.qkv = nullptr;
  const bool has_bias = bq || bk || bv;
  rc = shd_weight_from_bf16(ctx, tmp, has_bias ? btmp : nullptr, h, m->qd + 2 * m->kvd, SHD_ROWS_QKV, d, &L.qkv);
  if (rc) return cleanup(rc);
  cudaStreamSynchronize(ctx->stream);
  concat_rows_kernel<<<grid, 256, 0, ctx->stream>>>(wg, (long long)m->I * h, wu, (long long)m->I * h, nullptr, 0, tmp);
  if ((e = cudaGetLastError()) != cudaSuccess) return cleanup(shd_cuda_fail(ctx, e, "concat gate/up"));
  shd_weight_destroy(L.gateup);
  L.gateup = nullptr;
  rc = shd_weight_from_bf16(ctx, tmp, nullptr, h, 2 * m->I, SHD_ROWS_GATEUP, 0, &L.gateup);
  if (rc) return cleanup(rc);
  shd_weight_destroy(L.o);
  L.o = nullptr;
  rc = shd_weight_from_bf16(ctx, wo, nullptr, m->qd, h, SHD_ROWS_PLAIN, 0, &L.o);
  if (rc) return cleanup(rc);
  shd_weight_destroy(L.down);
  L.down = nullptr;
  rc = shd_weight_from_bf16(ctx, wd, nullptr, m->I, h, SHD_ROWS_PLAIN, 0, &L.down);
  if (rc) return cleanup(rc);
  e = cudaMemcpyAsync(L.g1, g1, (size_t)h * 4, cudaMemcpyDeviceToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(L.g2, g2, (size_t)h * 4, cudaMemcpyDeviceToDevice, ctx->stream);
  if (e != cudaSuccess) return cleanup(shd_cuda_fail(ctx, e, "copy norms"));
  if (m->graph) {  // weights changed: the captured graph holds old pointers
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  return cleanup(SHD_OK);
}

extern "C" int shd_model_set_embedding(shd_model* m, const uint16_t* table) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, table, "shd_model_set_embedding: null table");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const size_t bytes = (size_t)m->cfg.vocab * m->cfg.hidden * 2;
  if (!m->embed) SHD_CHECK_CUDA(ctx, cudaMalloc(&m->embed, bytes));
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(m->embed, table, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SHD_OK;
}

extern "C" int shd_model_set_head(shd_model* m, const uint16_t* lm_head, const float* final_norm) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, lm_head && final_norm, "shd_model_set_head: null pointer");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  shd_weight_destroy(m->lm_head);
  m->lm_head = nullptr;
  int rc = shd_weight_from_bf16(ctx, lm_head, nullptr, m->cfg.hidden, m->V, SHD_ROWS_PLAIN, 0, &m->lm_head);
  if (rc) return rc;
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(m->final_norm, final_norm, (size_t)m->cfg.hidden * 4,
                                      cudaMemcpyDeviceToDevice, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  return SHD_OK;
}

extern "C" int shd_model_set_masks(shd_model* m, const float* masks, int64_t stride) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  cudaFree(m->masks);
  m->masks = nullptr;
  m->mask_stride = 0;
  if (!masks) return SHD_OK;
  const int h = m->cfg.hidden;
  SHD_REQUIRE(ctx, stride >= 3LL * h + m->cfg.intermediate &&
                       stride >= (int64_t)h + (int64_t)m->cfg.n_heads * m->cfg.head_dim,
              "shd_model_set_masks: stride shorter than 3*hidden + intermediate");
  const size_t bytes = (size_t)m->cfg.n_layers * stride * 4;
  SHD_CHECK_CUDA(ctx, cudaMalloc(&m->masks, bytes));
  SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(m->masks, masks, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  m->mask_stride = stride;
  return SHD_OK;
}

extern "C" int shd_model_reset(shd_model* m) {
  if (!m) return SHD_ERR_ARG;
  std::fill(m->len.begin(), m->len.end(), 0);
  m->n_active = 0;
  return SHD_OK;
}

// ------------------------------------------------------------------------------------------------
// Enqueue the layers for M rows (positions pos[m] of slots seq[m]) starting from embedding shares in
// Hbuf[0] and a zero D. Leaves the final residual in (Hbuf[cur], D) for the head.
// ------------------------------------------------------------------------------------------------
// RMSNorm of (D + H) feeding a GEMV: fused into the GEMV prologue when the M normalized rows fit in
// shared memory next to the weight pipeline, else a separate norm kernel writes Xbuf (the
// tensor-core path computes it in its plane split).
static bool norm_fusable(const shd_weight* w, int M) {
  return (size_t)M * 2 * w->nKC * kChunkBf16 * 4 <= 120 * 1024 && !tc_preferred(w, M);
}

int shd_model::norm_into(GemvArgs& g, const shd_weight* w, int M, const float* Hc, const float* Hs,
                         const float* Dc, const float* Ds, float* Oc, float* Os, const float* gamma,
                         int variant, const float* mask, bool& fused) {
  const int h = cfg.hidden;
  has_pend_norm = false;
  fused = norm_fusable(w, M);
  if (fused) {
    g.nHc = Hc; g.nHs = Hs; g.nDc = Dc; g.nDs = Ds; g.nHout_c = Oc; g.nHout_s = Os; g.n_ldh = h;
    g.gamma = gamma; g.eps = cfg.rms_eps; g.nvariant = variant; g.nmask = mask; g.n_ldmask = 0;
    return SHD_OK;
  }
  NormArgs na{};
  na.Hc = Hc; na.Hs = Hs; na.Dc = Dc; na.Ds = Ds; na.Hout_c = Oc; na.Hout_s = Os; na.ldh = h;
  na.gamma = gamma; na.eps = cfg.rms_eps; na.variant = variant; na.mask = mask; na.ldmask = 0;
  na.Xc = Xbuf; na.Xs = Xbuf + (size_t)M * h; na.ldx = h; na.n = h;
  g.Xc = Xbuf; g.Xs = Xbuf + (size_t)M * h; g.ldx = h;
  if (tc_preferred(w, M)) {
    // the tensor-core linear computes the norm itself while it splits the bf16 planes (op_gemv)
    pend_norm = na;
    has_pend_norm = true;
    return SHD_OK;
  }
  return launch_norm(ctx, na, M);
}

int shd_model::op_gemv(const shd_weight* w, int M, int epi, const GemvArgs& g, bool norm,
                       const PlaneOut* out_planes, bool* wrote_out) {
  if (wrote_out) *wrote_out = false;
  const bool pend = has_pend_norm;
  has_pend_norm = false;
  if (!norm && tc_preferred(w, M))
    return launch_linear_tc(ctx, w, M, epi, g, pend ? &pend_norm : nullptr, false, out_planes, wrote_out);
  if (pend) {
    const int rc = launch_norm(ctx, pend_norm, M);
    if (rc) return rc;
  }
  return launch_gemv_f32(ctx, w, M, epi, g, norm);
}

int shd_model::enqueue_layers(int M, const int* d_pos, const int* d_seq, int variant, int& cur, bool decode) {
  const shd_model_config& c = cfg;
  const int h = c.hidden, d = c.head_dim;
  const size_t kv_layer = (size_t)c.max_batch * c.max_seq * kvd;
  const float* mk = masks;
  int rc;
  bool fused;
  cur = 0;
  for (int l = 0; l < c.n_layers; ++l) {
    const LayerW& Lw = layers[l];
    const float* lm = mk ? mk + (size_t)l * mask_stride : nullptr;
    float* Hc = Hbuf[cur];
    float* Ho = Hbuf[cur ^ 1];
    // input norm (h = D + H -> Ho, x = reshare(norm(h))) + q/k/v with RoPE and KV-cache write
    GemvArgs g{};
    if ((rc = norm_into(g, Lw.qkv, M, Hc, Hc + (size_t)M * h, Dbuf, Dbuf + (size_t)M * h, Ho,
                        Ho + (size_t)M * h, Lw.g1, variant, lm, fused)))
      return rc;
    g.bias = Lw.qkv->d_bias;
    g.q_dim = qd; g.kv_dim = kvd; g.head_dim = d;
    g.rope_cos = rope_cos; g.rope_sin = rope_sin; g.rope_max_seq = cfg.max_seq;
    g.pos = d_pos; g.seq = d_seq;
    g.Q = Qbuf; g.ldq = qd;
    g.Kcache = kcache + (size_t)l * kv_layer; g.Vcache = vcache + (size_t)l * kv_layer;
    g.kv_seq_stride = (int64_t)c.max_seq * kvd;
    g.trace = trace_slot(0);
    if ((rc = prof_mark(0, Lw.qkv, true))) return rc;
    if ((rc = op_gemv(Lw.qkv, M, EPI_QKV, g, fused))) return rc;
    if ((rc = prof_mark(0, Lw.qkv, false))) return rc;
    // attention -> A shares
    AttnArgs at{};
    at.Q = Qbuf; at.ldq = qd;
    at.Kcache = g.Kcache; at.Vcache = g.Vcache; at.kv_seq_stride = g.kv_seq_stride; at.kvd = kvd;
    at.groups = attn_groups_dev; at.n_groups = n_groups; at.head_dim = d;
    at.pos = d_pos; at.seq = d_seq; at.variant = c.variant_attn;
    at.scale = 1.0f / sqrtf((float)d);
    at.mask = lm ? lm + h + (size_t)sh.q_head_begin * d : nullptr; at.ldmask = 0;
    at.Oc = Abuf; at.Os = Abuf + (size_t)M * qd; at.ldo = qd;
    at.err = ctx->d_err;
    at.early_kv = decode ? 1 : 0;
    if (M >= kAttnWideRows && attn_groups8_dev) {
      at.groups = attn_groups8_dev;
      at.n_groups = n_groups8;
      at.group_cap = 8;
    }
    at.trace = trace_slot(5);
    if ((rc = prof_mark(5, nullptr, true))) return rc;
    if (!decode && M >= kFlashRows && flash_prefill_supported(at, M))
      rc = launch_flash_prefill(ctx, at, M);  // a prompt block: consecutive positions of one slot
    else
      rc = launch_attention(ctx, at, M);
    if (rc) return rc;
    if ((rc = prof_mark(5, nullptr, false))) return rc;
    // o projection -> D (partial under TP)
    GemvArgs go{};
    go.Xc = Abuf; go.Xs = Abuf + (size_t)M * qd; go.ldx = qd;
    go.Yc = Dbuf; go.Ys = Dbuf + (size_t)M * h; go.ldy = h;
    const bool push_o = tp_push(go, Lw.o, M, (size_t)2 * M * h);
    go.trace = trace_slot(1);
    if ((rc = prof_mark(1, Lw.o, true))) return rc;
    if ((rc = op_gemv(Lw.o, M, EPI_STORE, go, false))) return rc;
    if ((rc = prof_mark(1, Lw.o, false))) return rc;
    if ((rc = push_o ? allreduce_recv(Dbuf, (size_t)2 * M * h) : allreduce_sum(Dbuf, (size_t)2 * M * h))) return rc;
    // post-attention norm (h = D + Ho -> Hc) + gate/up + SwiGLU reshare -> ACT
    GemvArgs gu{};
    if ((rc = norm_into(gu, Lw.gateup, M, Ho, Ho + (size_t)M * h, Dbuf, Dbuf + (size_t)M * h, Hc,
                        Hc + (size_t)M * h, Lw.g2, variant, lm ? lm + 2 * (size_t)h : nullptr, fused)))
      return rc;
    gu.Yc = ACTbuf; gu.Ys = ACTbuf + (size_t)M * I; gu.ldy = I;
    gu.variant = variant;
    gu.mask = lm ? lm + 3 * (size_t)h + sh.inter_begin : nullptr; gu.ldmask = 0;
    gu.trace = trace_slot(2);
    if ((rc = prof_mark(2, Lw.gateup, true))) return rc;
    // gate/up with split K writes its output as the down linear's planes from the reduce kernel
    const PlaneOut d_planes = fused ? PlaneOut{} : tc_input_planes(ctx, Lw.down, M);
    bool down_ready = false;
    if ((rc = op_gemv(Lw.gateup, M, EPI_GATEUP, gu, fused, d_planes.p ? &d_planes : nullptr,
                      &down_ready)))
      return rc;
    if ((rc = prof_mark(2, Lw.gateup, false))) return rc;
    // down -> D
    GemvArgs gd{};
    gd.Xc = ACTbuf; gd.Xs = ACTbuf + (size_t)M * I; gd.ldx = I;
    gd.Yc = Dbuf; gd.Ys = Dbuf + (size_t)M * h; gd.ldy = h;
    const bool push_d = tp_push(gd, Lw.down, M, (size_t)2 * M * h);
    gd.trace = trace_slot(3);
    if ((rc = prof_mark(3, Lw.down, true))) return rc;
    if ((rc = down_ready ? launch_linear_tc(ctx, Lw.down, M, EPI_STORE, gd, nullptr, true)
                         : op_gemv(Lw.down, M, EPI_STORE, gd, false)))
      return rc;
    if ((rc = prof_mark(3, Lw.down, false))) return rc;
    if ((rc = push_d ? allreduce_recv(Dbuf, (size_t)2 * M * h) : allreduce_sum(Dbuf, (size_t)2 * M * h))) return rc;
    // the residual stream for the next layer is (Hc, D)
  }
  return SHD_OK;
}

// Final norm of row `row` of (Hbuf[cur], D) and the lm_head with argmax into amax[key_row].
int shd_model::enqueue_head(int M, int row, int cur, int variant, bool want_logits, int key_row) {
  const int h = cfg.hidden;
  const float* lm = masks ? masks + (size_t)(cfg.n_layers - 1) * mask_stride : nullptr;
  float* Hc = Hbuf[cur];
  GemvArgs g{};
  bool fused;
  int rc = norm_into(g, lm_head, 1, Hc + (size_t)row * h, Hc + (size_t)M * h + (size_t)row * h,
                     Dbuf + (size_t)row * h, Dbuf + (size_t)M * h + (size_t)row * h, nullptr, nullptr,
                     final_norm, variant, lm, fused);
  if (rc) return rc;
  g.amax = amax + key_row;
  g.idx_offset = sh.vocab_begin;
  if (want_logits) {
    g.Yc = LOGbuf; g.Ys = LOGbuf + V; g.ldy = V;
  }
  return launch_gemv_f32(ctx, lm_head, 1, EPI_LOGITS, g, fused);
}

// Decode head for all M rows (each its own slot): norm M rows, lm_head on M rows.
int shd_model::enqueue_head_rows(int M, int cur, int variant, float* logits) {
  const int h = cfg.hidden;
  const float* lm = masks ? masks + (size_t)(cfg.n_layers - 1) * mask_stride : nullptr;
  float* Hc = Hbuf[cur];
  GemvArgs g{};
  bool fused;
  int rc = norm_into(g, lm_head, M, Hc, Hc + (size_t)M * h, Dbuf, Dbuf + (size_t)M * h, nullptr, nullptr,
                     final_norm, variant, lm, fused);
  if (rc) return rc;
  g.amax = amax;
  g.idx_offset = sh.vocab_begin;
  if (logits) {
    g.Yc = logits; g.Ys = logits + (size_t)M * V; g.ldy = V;
  }
  g.trace = trace_slot(4);
  if ((rc = prof_mark(4, lm_head, true))) return rc;
  if ((rc = op_gemv(lm_head, M, EPI_LOGITS, g, fused))) return rc;
  return prof_mark(4, lm_head, false);
}

int shd_model::check_ready() {
  SHD_REQUIRE(ctx, embed && lm_head, "model: embedding and head must be set");
  for (auto& L : layers) SHD_REQUIRE(ctx, L.qkv && L.o && L.gateup && L.down, "model: a layer has no weights");
  return SHD_OK;
}

// Prefill of n positions of `slot` in chunks of kPrefillRows, from token ids (embedding shares
// generated on the device) or from hidden-state shares given by the caller (hc/hs host [n][h]).
// Optional outputs of the last position: the whole logit shares, and the final hidden state
// (the residual stream after the last layer, per share: H + D, as secure_add_gpu leaves it).
int shd_model::prefill_impl(int slot, int n, const int32_t* tokens_host, const float* hc_host, const float* hs_host,
                            float* logits_c_host, float* logits_s_host, float* final_c_host, float* final_s_host,
                            int32_t* next_token_host) {
  const int h = cfg.hidden;
  std::vector<int> hp(3 * kPrefillRows);
  int cur = 0, rc = SHD_OK, M_last = 0;
  for (int p0 = 0; p0 < n && rc == SHD_OK; p0 += kPrefillRows) {
    const int M = std::min(kPrefillRows, n - p0);
    M_last = M;
    // the staging vector is reused: finish the previous chunk's copies first
    if (cudaStreamSynchronize(stream) != cudaSuccess) { rc = shd_fail(ctx, SHD_ERR_CUDA, "prefill sync"); break; }
    for (int i = 0; i < M; ++i) {
      hp[i] = tokens_host ? tokens_host[p0 + i] : 0;
      hp[kPrefillRows + i] = len[slot] + p0 + i;
      hp[2 * kPrefillRows + i] = slot;
    }
    cudaError_t e = cudaMemcpyAsync(p_pos, hp.data() + kPrefillRows, M * 4, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(p_seq, hp.data() + 2 * kPrefillRows, M * 4, cudaMemcpyHostToDevice, stream);
    if (tokens_host) {
      if (e == cudaSuccess) e = cudaMemcpyAsync(p_tokens, hp.data(), M * 4, cudaMemcpyHostToDevice, stream);
    } else {
      // the caller's hidden-state shares (get_embeddings_direct output) stand in for the embedding
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(Hbuf[0], hc_host + (size_t)p0 * h, (size_t)M * h * 4, cudaMemcpyHostToDevice, stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(Hbuf[0] + (size_t)M * h, hs_host + (size_t)p0 * h, (size_t)M * h * 4,
                            cudaMemcpyHostToDevice, stream);
      if (e == cudaSuccess) e = cudaMemsetAsync(Dbuf, 0, (size_t)2 * M * h * 4, stream);
      if (e == cudaSuccess) e = cudaMemsetAsync(amax, 0, 8, stream);
    }
    if (e != cudaSuccess) { rc = shd_cuda_fail(ctx, e, "prefill staging"); break; }
    if (tokens_host) {
      EmbedArgs ea{};
      ea.table = embed; ea.vocab = cfg.vocab; ea.hidden = h; ea.tokens = p_tokens;
      ea.pos = p_pos; ea.seed = cfg.share_seed; ea.counter_base = (uint64_t)slot << 32;
      ea.Hc = Hbuf[0]; ea.Hs = Hbuf[0] + (size_t)M * h; ea.ldh = h;
      ea.Dc = Dbuf; ea.Ds = Dbuf + (size_t)M * h; ea.amax = amax; ea.err = ctx->d_err;
      if ((rc = launch_embed(ctx, ea, M))) break;
    }
    if ((rc = enqueue_layers(M, p_pos, p_seq, cfg.variant_prefill, cur, false))) break;
    if (p0 + M == n) {
      if ((rc = enqueue_head(M, M - 1, cur, cfg.variant_prefill, logits_c_host != nullptr, 0))) break;
      if ((rc = allreduce_max_keys(1))) break;
      if (logits_c_host && (rc = gather_logits(logits_c_host, logits_s_host))) break;
    }
  }
  std::vector<float> fin;
  if (rc == SHD_OK && final_c_host) {
    // row M_last - 1 of (H, D), both shares
    fin.resize((size_t)4 * h);
    const size_t off_c = (size_t)(M_last - 1) * h, off_s = (size_t)M_last * h + off_c;
    cudaError_t e = cudaMemcpyAsync(fin.data(), Hbuf[cur] + off_c, (size_t)h * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(fin.data() + h, Hbuf[cur] + off_s, (size_t)h * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(fin.data() + 2 * h, Dbuf + off_c, (size_t)h * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(fin.data() + 3 * h, Dbuf + off_s, (size_t)h * 4, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "prefill: final hidden");
  }
  if (rc == SHD_OK) {
    unsigned long long key = 0;
    cudaError_t e = cudaMemcpyAsync(&key, amax, 8, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_prefill");
    if (rc == SHD_OK) {
      const int tok = (int)(key & 0xffffffffu);
      const int next_pos = len[slot] + n;
      // decode state of the slot: input token and its position
      e = cudaMemcpyAsync(tokens + slot, &tok, 4, cudaMemcpyHostToDevice, stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(pos + slot, &next_pos, 4, cudaMemcpyHostToDevice, stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_prefill: state");
      len[slot] = next_pos;
      n_active = std::max(n_active, slot + 1);
      if (next_token_host) *next_token_host = tok;
      if (final_c_host) {
        for (int i = 0; i < h; ++i) {
          final_c_host[i] = fin[i] + fin[2 * h + i];  // secure_add_gpu: per-share add
          final_s_host[i] = fin[h + i] + fin[3 * h + i];
        }
      }
    }
  }
  return rc;
}

extern "C" int shd_model_prefill(shd_model* m, int slot, const int32_t* tokens_host, int n,
                                 int32_t* next_token_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_model_prefill: slot out of range");
  SHD_REQUIRE(ctx, tokens_host && n > 0, "shd_model_prefill: empty prompt (the reference rejects it)");
  SHD_REQUIRE(ctx, m->len[slot] + n <= m->cfg.max_seq, "shd_model_prefill: prompt exceeds max_seq");
  for (int i = 0; i < n; ++i)
    SHD_REQUIRE(ctx, tokens_host[i] >= 0 && tokens_host[i] < m->cfg.vocab, "shd_model_prefill: token id out of range");
  int rc = m->check_ready();
  if (rc) return rc;
  if ((rc = m->enter())) return rc;
  rc = m->prefill_impl(slot, n, tokens_host, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, next_token_host);
  rc = m->leave(rc);
  if (rc == SHD_OK) rc = shd_sync(ctx);
  return rc;
}

extern "C" int shd_model_prefill_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host, int n,
                                        float* logits_c_host, float* logits_s_host, float* final_c_host,
                                        float* final_s_host, int32_t* next_token_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_model_prefill_hidden: slot out of range");
  SHD_REQUIRE(ctx, hc_host && hs_host && n > 0, "shd_model_prefill_hidden: empty prompt (the reference rejects it)");
  SHD_REQUIRE(ctx, (logits_c_host == nullptr) == (logits_s_host == nullptr) &&
                   (final_c_host == nullptr) == (final_s_host == nullptr),
              "shd_model_prefill_hidden: output shares come in pairs");
  SHD_REQUIRE(ctx, m->len[slot] + n <= m->cfg.max_seq, "shd_model_prefill_hidden: prompt exceeds max_seq");
  int rc = m->check_ready();
  if (rc) return rc;
  if ((rc = m->enter())) return rc;
  rc = m->prefill_impl(slot, n, nullptr, hc_host, hs_host, logits_c_host, logits_s_host, final_c_host, final_s_host,
                       next_token_host);
  rc = m->leave(rc);
  if (rc == SHD_OK) rc = shd_sync(ctx);
  return rc;
}

extern "C" int shd_model_read_kv(shd_model* m, int slot, int pos0, int n, float* k_host, float* v_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_model_read_kv: slot out of range");
  SHD_REQUIRE(ctx, k_host && v_host && n >= 0 && pos0 >= 0 && pos0 + n <= m->len[slot],
              "shd_model_read_kv: positions beyond the slot's length");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  const size_t kvd = (size_t)m->kvd, row = kvd * 4;
  const size_t layer = (size_t)m->cfg.max_batch * m->cfg.max_seq * kvd;
  for (int l = 0; l < m->cfg.n_layers; ++l) {
    const size_t src = (size_t)l * layer + ((size_t)slot * m->cfg.max_seq + pos0) * kvd;
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(k_host + (size_t)l * n * kvd, m->kcache + src, n * row, cudaMemcpyDeviceToHost, m->stream));
    SHD_CHECK_CUDA(ctx, cudaMemcpyAsync(v_host + (size_t)l * n * kvd, m->vcache + src, n * row, cudaMemcpyDeviceToHost, m->stream));
  }
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(m->stream));
  return SHD_OK;
}

// One decode step for slots [0, M): embed the current tokens at pos, all layers, head, tokens.
int shd_model::enqueue_decode_step(int M) {
  const int h = cfg.hidden;
  EmbedArgs ea{};
  ea.table = embed; ea.vocab = cfg.vocab; ea.hidden = h; ea.tokens = tokens; ea.pos = pos;
  ea.seed = cfg.share_seed; ea.counter_base = 0;
  ea.Hc = Hbuf[0]; ea.Hs = Hbuf[0] + (size_t)M * h; ea.ldh = h;
  ea.Dc = Dbuf; ea.Ds = Dbuf + (size_t)M * h; ea.amax = amax; ea.err = ctx->d_err;
  ea.slot_counter = 1;
  int rc;
  if ((rc = launch_embed(ctx, ea, M))) return rc;
  int cur = 0;
  if ((rc = enqueue_layers(M, pos, seq, cfg.variant_decode, cur, true))) return rc;
  if ((rc = enqueue_head_rows(M, cur, cfg.variant_decode))) return rc;
  if ((rc = allreduce_max_keys(M))) return rc;
  SHD_CHECK_CUDA(ctx, launch_pdl(finish_step_kernel, dim3(1), dim3(32), 0, stream, (const unsigned long long*)amax,
                                 tokens, pos, hist, hist_cap, step, M));
  ctx->launches++;
  return SHD_OK;
}

extern "C" int shd_model_decode_async(shd_model* m, int n_steps) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, n_steps >= 0, "shd_model_decode_async: n_steps < 0");
  SHD_REQUIRE(ctx, m->n_active > 0, "shd_model_decode_async: no prefilled sequence");
  const int M = m->n_active;
  for (int s = 0; s < M; ++s)
    SHD_REQUIRE(ctx, m->len[s] > 0, "shd_model_decode_async: active slots must all be prefilled");
  for (int s = 0; s < M; ++s)
    SHD_REQUIRE(ctx, m->len[s] + n_steps <= m->cfg.max_seq, "shd_model_decode_async: would exceed max_seq");
  if (n_steps == 0) return SHD_OK;
  int rc = m->check_ready();
  if (rc) return rc;
  if ((rc = m->enter())) return rc;
  int done = 0;
  if (!m->graph || m->graph_rows != M) {
    if (m->graph) {
      cudaGraphExecDestroy(m->graph);
      m->graph = nullptr;
    }
    // one eager step (sets kernel attributes, real work), then capture the step
    rc = m->enqueue_decode_step(M);
    done = 1;
    if (rc == SHD_OK && m->profiling) {
      const size_t need = (size_t)2 * (5 * m->cfg.n_layers + 1);
      while (m->prof_events.size() < need) {
        cudaEvent_t ev;
        if (cudaEventCreate(&ev) != cudaSuccess) { rc = shd_fail(ctx, SHD_ERR_CUDA, "cudaEventCreate"); break; }
        m->prof_events.push_back(ev);
      }
    }
    if (rc == SHD_OK && m->profiling == 2 && !m->d_trace) {
      const int cap = 8 * m->cfg.n_layers + 8;
      if (cudaMalloc(&m->d_trace, (size_t)cap * 8 * sizeof(uint64_t)) != cudaSuccess)
        rc = shd_fail(ctx, SHD_ERR_CUDA, "timeline buffer");
      else
        m->trace_cap = cap;
    }
    if (rc == SHD_OK) {
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
      if (e == cudaSuccess) {
        m->graph_launch_mark = ctx->launches;
        m->prof_active = m->profiling != 0;
        m->prof_next = 0;
        m->prof_kind.clear();
        m->prof_bytes.clear();
        m->trace_kind.clear();
        if (m->profiling == 2) {
          e = cudaMemsetAsync(m->d_trace, 0xFF, (size_t)m->trace_cap * 8 * sizeof(uint64_t), m->stream);
          if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "timeline preset");
        }
        if (rc == SHD_OK) rc = m->enqueue_decode_step(M);
        m->prof_active = false;
        m->prof_count = m->prof_next;
        e = cudaStreamEndCapture(m->stream, &g);
        if (rc == SHD_OK && e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "capture decode step");
      } else {
        rc = shd_cuda_fail(ctx, e, "cudaStreamBeginCapture");
      }
      if (rc == SHD_OK) {
        e = cudaGraphInstantiate(&m->graph, g, 0);
        if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "cudaGraphInstantiate");
        m->graph_rows = M;
        m->graph_launches = ctx->launches - m->graph_launch_mark;
      }
      if (g) cudaGraphDestroy(g);
    }
  }
  for (int i = done; i < n_steps && rc == SHD_OK; ++i) {
    cudaError_t e = cudaGraphLaunch(m->graph, m->stream);
    if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "cudaGraphLaunch");
  }
  if (rc == SHD_OK) {
    for (int s = 0; s < M; ++s) m->len[s] += n_steps;
    m->steps_done += n_steps;
  }
  return m->leave(rc);
}

extern "C" int shd_model_read_tokens(shd_model* m, int count, int32_t* tokens_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  const int M = m->n_active;
  SHD_REQUIRE(ctx, count >= 0 && count <= m->hist_cap && count <= m->steps_done,
              "shd_model_read_tokens: count exceeds the decoded steps kept");
  SHD_REQUIRE(ctx, tokens_host || count == 0, "shd_model_read_tokens: null output");
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(m->stream));
  std::vector<int> all((size_t)m->hist_cap * M);
  SHD_CHECK_CUDA(ctx, cudaMemcpy(all.data(), m->hist, all.size() * 4, cudaMemcpyDeviceToHost));
  for (int i = 0; i < count; ++i) {
    const long long s = m->steps_done - count + i;
    std::memcpy(tokens_host + (size_t)i * M, all.data() + (size_t)(s % m->hist_cap) * M, (size_t)M * 4);
  }
  return shd_sync(ctx);
}

extern "C" int shd_model_forward_host_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host,
                                             float* logits_c_host, float* logits_s_host, float* hidden_c_host,
                                             float* hidden_s_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_model_forward_host: slot out of range");
  SHD_REQUIRE(ctx, hc_host && hs_host && logits_c_host && logits_s_host, "shd_model_forward_host: null buffer");
  SHD_REQUIRE(ctx, (hidden_c_host == nullptr) == (hidden_s_host == nullptr),
              "shd_model_forward_host: output shares come in pairs");
  SHD_REQUIRE(ctx, m->len[slot] < m->cfg.max_seq, "shd_model_forward_host: sequence full");
  int rc = m->check_ready();
  if (rc) return rc;
  if ((rc = m->enter())) return rc;
  const int h = m->cfg.hidden;
  const int p = m->len[slot];
  int meta[2] = {p, slot};
  std::vector<float> fin(hidden_c_host ? (size_t)4 * h : 0);
  cudaError_t e = cudaMemcpyAsync(m->Hbuf[0], hc_host, (size_t)h * 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->Hbuf[0] + h, hs_host, (size_t)h * 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->p_pos, &meta[0], 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->p_seq, &meta[1], 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->Dbuf, 0, (size_t)2 * h * 4, m->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->amax, 0, 8, m->stream);
  if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_forward_host: upload");
  int cur = 0;
  if (rc == SHD_OK) rc = m->enqueue_layers(1, m->p_pos, m->p_seq, m->cfg.variant_decode, cur, true);
  if (rc == SHD_OK) rc = m->enqueue_head(1, 0, cur, m->cfg.variant_decode, true, 0);
  if (rc == SHD_OK) rc = m->gather_logits(logits_c_host, logits_s_host);
  if (rc == SHD_OK && hidden_c_host) {
    // the residual stream after the last layer: (H, D) of row 0, both shares
    e = cudaMemcpyAsync(fin.data(), m->Hbuf[cur], (size_t)2 * h * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(fin.data() + 2 * h, m->Dbuf, (size_t)2 * h * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_forward_host: hidden");
  }
  if (rc == SHD_OK) {
    e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
      rc = shd_cuda_fail(ctx, e, "shd_model_forward_host");
    } else {
      m->len[slot] = p + 1;
      if (hidden_c_host)
        for (int i = 0; i < h; ++i) {
          hidden_c_host[i] = fin[i] + fin[2 * h + i];  // secure_add_gpu: per-share add
          hidden_s_host[i] = fin[h + i] + fin[3 * h + i];
        }
    }
  }
  rc = m->leave(rc);
  if (rc == SHD_OK) rc = shd_sync(ctx);
  return rc;
}

extern "C" int shd_model_forward_host_rows(shd_model* m, int M, const int32_t* slots, const float* hc_host,
                                           const float* hs_host, float* logits_c_host, float* logits_s_host) {
  if (!m) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, M >= 1 && M <= m->cfg.max_batch, "shd_model_forward_host_rows: rows must be 1..max_batch");
  SHD_REQUIRE(ctx, slots && hc_host && hs_host && logits_c_host && logits_s_host,
              "shd_model_forward_host_rows: null buffer");
  std::vector<char> seen(m->cfg.max_batch, 0);
  for (int r = 0; r < M; ++r) {
    SHD_REQUIRE(ctx, slots[r] >= 0 && slots[r] < m->cfg.max_batch, "shd_model_forward_host_rows: slot out of range");
    SHD_REQUIRE(ctx, !seen[slots[r]], "shd_model_forward_host_rows: a slot appears twice");
    seen[slots[r]] = 1;
    SHD_REQUIRE(ctx, m->len[slots[r]] < m->cfg.max_seq, "shd_model_forward_host_rows: sequence full");
  }
  int rc = m->check_ready();
  if (rc) return rc;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  if (!m->LOGrows) {
    SHD_CHECK_CUDA(ctx, cudaMalloc(&m->LOGrows, (size_t)2 * m->cfg.max_batch * std::max(m->V, 1) * 4));
    m->owned.push_back(m->LOGrows);
  }
  if ((rc = m->enter())) return rc;
  const int h = m->cfg.hidden, vocab = m->cfg.vocab;
  std::vector<int> meta(2 * (size_t)M);
  for (int r = 0; r < M; ++r) {
    meta[r] = m->len[slots[r]];
    meta[M + r] = slots[r];
  }
  const size_t rows = (size_t)M * h * 4;
  cudaError_t e = cudaMemcpyAsync(m->Hbuf[0], hc_host, rows, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->Hbuf[0] + (size_t)M * h, hs_host, rows, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->p_pos, meta.data(), (size_t)M * 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->p_seq, meta.data() + M, (size_t)M * 4, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->Dbuf, 0, 2 * rows, m->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->amax, 0, (size_t)M * 8, m->stream);
  if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_forward_host_rows: upload");
  int cur = 0;
  if (rc == SHD_OK) rc = m->enqueue_layers(M, m->p_pos, m->p_seq, m->cfg.variant_decode, cur, true);
  if (rc == SHD_OK) rc = m->enqueue_head_rows(M, cur, m->cfg.variant_decode, m->LOGrows);
  if (rc == SHD_OK && ctx->tp_world <= 1) {
    e = cudaMemcpyAsync(logits_c_host, m->LOGrows, (size_t)M * vocab * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(logits_s_host, m->LOGrows + (size_t)M * m->V, (size_t)M * vocab * 4, cudaMemcpyDeviceToHost,
                          m->stream);
    if (e != cudaSuccess) rc = shd_cuda_fail(ctx, e, "shd_model_forward_host_rows: logits");
  }
  for (int r = 0; r < M && rc == SHD_OK && ctx->tp_world > 1; ++r)
    rc = m->gather_logits(logits_c_host + (size_t)r * vocab, logits_s_host + (size_t)r * vocab,
                          m->LOGrows + (size_t)r * m->V, m->LOGrows + (size_t)(M + r) * m->V);
  if (rc == SHD_OK) {
    e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
      rc = shd_cuda_fail(ctx, e, "shd_model_forward_host_rows");
    } else {
      for (int r = 0; r < M; ++r) m->len[slots[r]] += 1;
    }
  }
  rc = m->leave(rc);
  if (rc == SHD_OK) rc = shd_sync(ctx);
  return rc;
}

extern "C" int shd_model_forward_host(shd_model* m, int slot, const float* hc_host, const float* hs_host,
                                      float* logits_c_host, float* logits_s_host) {
  return shd_model_forward_host_hidden(m, slot, hc_host, hs_host, logits_c_host, logits_s_host, nullptr, nullptr);
}

int shd_model::prof_mark(int kind, const shd_weight* w, bool begin) {
  if (!prof_active || profiling != 1) return SHD_OK;
  if (prof_next + 1 >= prof_events.size()) return SHD_OK;
  if (begin) {
    prof_kind.push_back(kind);
    prof_bytes.push_back(w ? (double)w->N * (double)w->K * 2.0 : 0.0);
    SHD_CHECK_CUDA(ctx, cudaEventRecordWithFlags(prof_events[prof_next], stream, cudaEventRecordExternal));
  } else {
    SHD_CHECK_CUDA(ctx, cudaEventRecordWithFlags(prof_events[prof_next + 1], stream, cudaEventRecordExternal));
    prof_next += 2;
  }
  return SHD_OK;
}

unsigned long long* shd_model::trace_slot(int kind) {
  if (!prof_active || profiling != 2 || (int)trace_kind.size() >= trace_cap) return nullptr;
  trace_kind.push_back(kind);
  return d_trace + (size_t)8 * (trace_kind.size() - 1);
}

extern "C" int64_t shd_model_step_launches(const shd_model* m) { return m ? m->graph_launches : -1; }

extern "C" int shd_model_set_profiling(shd_model* m, int on) {
  if (!m) return SHD_ERR_ARG;
  if ((on != 0) != (m->profiling != 0) && m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  m->profiling = (on == 1 || on == 2) ? on : 0;
  return SHD_OK;
}

extern "C" int shd_model_timeline(shd_model* m, int cap, int32_t* kinds, uint64_t* stamps, int* n_out) {
  if (!m || !n_out) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_REQUIRE(ctx, m->profiling == 2 && m->graph && !m->trace_kind.empty(),
              "shd_model_timeline: no traced decode step yet (shd_model_set_profiling(m, 2), then decode)");
  const int n = (int)m->trace_kind.size();
  *n_out = n;
  if (cap < n || !kinds || !stamps) return SHD_OK;  // size query
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(m->stream));
  SHD_CHECK_CUDA(ctx, cudaMemcpy(stamps, m->d_trace, (size_t)n * 8 * sizeof(uint64_t), cudaMemcpyDeviceToHost));
  for (int i = 0; i < n; ++i) kinds[i] = m->trace_kind[i];
  return SHD_OK;
}

extern "C" int shd_model_linear_times(shd_model* m, float* ms_out6, double* bytes_out6) {
  if (!m || !ms_out6 || !bytes_out6) return SHD_ERR_ARG;
  shd_ctx* ctx = m->ctx;
  SHD_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
  SHD_CHECK_CUDA(ctx, cudaStreamSynchronize(m->stream));
  SHD_REQUIRE(ctx, m->prof_count > 0, "shd_model_linear_times: no profiled decode step yet");
  for (int k = 0; k < 6; ++k) {
    ms_out6[k] = 0.f;
    bytes_out6[k] = 0.0;
  }
  for (size_t i = 0; i + 1 < m->prof_count; i += 2) {
    float ms = 0.f;
    SHD_CHECK_CUDA(ctx, cudaEventElapsedTime(&ms, m->prof_events[i], m->prof_events[i + 1]));
    const int k = m->prof_kind[i / 2];
    ms_out6[k] += ms;
    bytes_out6[k] += m->prof_bytes[i / 2];
  }
  return SHD_OK;
}
