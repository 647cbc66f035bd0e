// Internal definition of shd_model (the device-resident layer loop).
#pragma once

#include <vector>

#include "shd_gemv.cuh"
#include "shd_nonlinear.cuh"
#include "shd_planes.cuh"

struct LayerW {
  shd_weight* qkv = nullptr;     // fused q|k|v, SHD_ROWS_QKV
  shd_weight* o = nullptr;       // [h][q_local]
  shd_weight* gateup = nullptr;  // fused gate|up, SHD_ROWS_GATEUP
  shd_weight* down = nullptr;    // [h][inter_local]
  float* g1 = nullptr;           // input RMSNorm gamma
  float* g2 = nullptr;           // post-attention RMSNorm gamma
};

struct shd_model {
  shd_ctx* ctx = nullptr;
  shd_model_config cfg{};
  shd_shard_info sh{};
  cudaStream_t stream = nullptr, saved_stream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  int qd = 0, kvd = 0, I = 0, V = 0;  // local widths
  int R = 8;                          // activation rows
  int T = 0;                          // KV capacity per slot
  std::vector<LayerW> layers;
  shd_weight* lm_head = nullptr;
  float* final_norm = nullptr;
  uint16_t* embed = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;  // RopeFrequencies table [max_seq][head_dim/2]
  // activations: [2][rows][width], client rows then server rows
  float* Hbuf[2] = {nullptr, nullptr};
  float *Dbuf = nullptr, *Xbuf = nullptr, *Qbuf = nullptr, *Abuf = nullptr, *ACTbuf = nullptr;
  float *LOGbuf = nullptr, *LOGfull = nullptr;
  float* gather_buf = nullptr;  // TP logit all-gather staging
  float *kcache = nullptr, *vcache = nullptr;  // [L][slots][T][kvd]
  int *tokens = nullptr, *pos = nullptr, *seq = nullptr;
  int *p_tokens = nullptr, *p_pos = nullptr, *p_seq = nullptr;
  int4* attn_groups_dev = nullptr;  // attention head groups (kv head, first q head, count), <= 4 q heads
  int4* attn_groups8_dev = nullptr; // the same with up to 8 q heads (null when no kv head has more than 4)
  int n_groups8 = 0;
  int n_groups = 0;
  unsigned long long* amax = nullptr;
  unsigned long long* step = nullptr;
  int* hist = nullptr;
  int hist_cap = 0;
  long long steps_done = 0;
  float* masks = nullptr;
  int64_t mask_stride = 0;
  std::vector<void*> owned;
  std::vector<int> len;
  int n_active = 0;
  cudaGraphExec_t graph = nullptr;
  int graph_rows = 0;
  int64_t graph_launches = 0, graph_launch_mark = 0;
  // profiling: CUDA events recorded around each linear launch of the captured step
  int profiling = 0;
  bool prof_active = false;
  std::vector<cudaEvent_t> prof_events;
  std::vector<int> prof_kind;
  std::vector<double> prof_bytes;
  size_t prof_next = 0, prof_count = 0;
  int prof_mark(int kind, const shd_weight* w, bool begin);
  // timeline (profiling == 2): one slot of 8 u64 per traced launch of the captured step, preset
  // to all ones by a memset node at the start of the step (TraceField in shd_common.cuh)
  unsigned long long* d_trace = nullptr;
  int trace_cap = 0;
  std::vector<int> trace_kind;
  unsigned long long* trace_slot(int kind);

  // launch one linear of the layer loop (tensor cores or the GEMV, with a pending norm)
  // out_planes / wrote_out: see launch_linear_tc (tensor-core path only)
  int op_gemv(const shd_weight* w, int M, int epi, const shd::GemvArgs& g, bool norm,
              const shd::PlaneOut* out_planes = nullptr, bool* wrote_out = nullptr);

  ~shd_model();
  int use_stream();
  void restore_stream();
  int enter();
  int leave(int rc);
  int check_ready();
  int norm_into(shd::GemvArgs& g, const shd_weight* w, int M, const float* Hc, const float* Hs,
                const float* Dc, const float* Ds, float* Oc, float* Os, const float* gamma, int variant,
                const float* mask, bool& fused);
  // decode: one new K/V row per sequence row (attention may read the older rows before the wait)
  int enqueue_layers(int M, const int* d_pos, const int* d_seq, int variant, int& cur, bool decode);
  int enqueue_head(int M, int row, int cur, int variant, bool want_logits, int key_row);
  // logits (nullable): [2][M][V] local logit shares written beside the argmax keys
  int enqueue_head_rows(int M, int cur, int variant, float* logits = nullptr);
  int enqueue_decode_step(int M);
  int prefill_impl(int slot, int n, const int32_t* tokens_host, const float* hc_host, const float* hs_host,
                   float* logits_c_host, float* logits_s_host, float* final_c_host, float* final_s_host,
                   int32_t* next_token_host);
  // tensor parallel collectives (no-ops at tp_world == 1)
  int allreduce_sum(float* buf, size_t n);
  bool tp_push(shd::GemvArgs& g, const shd_weight* w, int M, size_t n);
  // norm left for the next tensor-core linear to compute with its plane split (norm_into -> op_gemv)
  shd::NormArgs pend_norm{};
  bool has_pend_norm = false;
  int allreduce_recv(float* buf, size_t n);
  int allreduce_max_keys(int M);
  // the whole vocabulary's logit shares of one row to the host (src: local [V] client, server
  // shares; null = LOGbuf)
  int gather_logits(float* lc_host, float* ls_host, const float* src_c = nullptr, const float* src_s = nullptr);
  float* LOGrows = nullptr;  // [2][max_batch][V] logit rows of shd_model_forward_host_rows (lazy)
};
