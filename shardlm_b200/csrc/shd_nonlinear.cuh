// Internal interface of the nonlinear, embedding and attention kernels (used by the model loop).
#pragma once

#include <vector>

#include "shd_common.cuh"

namespace shd {

struct NormArgs {
  const float* Hc;     // residual stream shares [M][ldh]
  const float* Hs;
  const float* Dc;     // sublayer output shares to add first (nullable)
  const float* Ds;
  float* Hout_c;       // h = D + H written here when given (nullable)
  float* Hout_s;
  int ldh;
  const float* gamma;
  float eps;
  int variant;
  const float* mask;   // reshare mask [M][ldmask] (nullable -> (y, 0))
  int ldmask;
  float* Xc;           // normalized shares out [M][ldx]
  float* Xs;
  int ldx;
  int n;
};

int launch_norm(shd_ctx* ctx, const NormArgs& a, int M);

struct EmbedArgs {
  const uint16_t* table;  // bf16 [vocab][hidden]
  int vocab, hidden;
  const int32_t* tokens;  // [M] device
  const int* pos;         // [M] device (nullable -> row index)
  uint64_t seed;
  uint64_t counter_base;
  int slot_counter;       // counter = (row << 32) + pos[row] instead of counter_base + pos[row]
  float* Hc;
  float* Hs;
  int ldh;
  float* Dc;              // zeroed when given
  float* Ds;
  unsigned long long* amax;  // reset to 0 when given
  int* err;
};

int launch_embed(shd_ctx* ctx, const EmbedArgs& a, int M);
int launch_keys_to_tokens(shd_ctx* ctx, const unsigned long long* keys, int* tokens, int M);

constexpr int kAttnGroupMax = 8;  // q heads handled together (sharing one kv head)

struct AttnArgs {
  const float* Q;          // reconstructed queries [M][ldq], local heads
  int ldq;
  const float* Kcache;     // [seq][T][kvd] reconstructed
  const float* Vcache;
  int64_t kv_seq_stride;   // floats between sequence slots
  int kvd;                 // local kv heads * head_dim
  const int4* groups;      // [n_groups] (local kv head, first local q head, q head count <= 8, 0)
  int n_groups;
  int head_dim;            // 64 or 128
  const int* pos;          // [M] position of the query row; it attends to [0, pos]
  const int* seq;          // [M] sequence slot (nullable -> 0)
  int variant;             // SHD_NL_APPROX/GPU: clamp(-40,40); SHD_NL_MPC: plain exp
  float scale;
  const float* mask;       // reshare mask [M][ldo] (nullable)
  int ldmask;
  float* Oc;               // attention output shares [M][ldo]
  float* Os;
  int ldo;
  // Decode launches: every K/V row before pos[m] of row m's slot, and pos/seq themselves, were
  // written before the previous step ended (only row pos[m] comes from the q/k/v kernel right
  // before), so they may be read before the wait on that kernel. 0 for prefill chunks.
  int early_kv;
  int group_cap;           // 8: `groups` hold up to 8 q heads each; otherwise up to 4
  int* err;
  unsigned long long* trace;  // launch timeline slot (nullable; TraceField in shd_common.cuh)
};

int launch_attention(shd_ctx* ctx, const AttnArgs& a, int M);
// Prompt blocks on the tensor cores (shd_flash.cu): rows m are positions pos[0] + m of slot seq[0]
// and attend to [0, pos[0] + m]. Supported: head_dim 128, 16-byte aligned rows.
bool flash_prefill_supported(const AttnArgs& a, int M);
int launch_flash_prefill(shd_ctx* ctx, const AttnArgs& a, int M);
// Groups of at most `cap` (4 or 8) consecutive local q heads sharing one kv head. Local q heads are
// [q_begin, q_begin + q_count) of the model, local kv heads start at kv_begin; group = H / Hkv.
std::vector<int4> attn_groups(int q_begin, int q_count, int kv_begin, int group, int cap = 4);

int shd_build_rope(shd_ctx* ctx, int head_dim, int max_seq, float theta);
// RopeFrequencies::new table ([max_seq][head_dim/2] cos and sin) in new device allocations.
int build_rope_table(shd_ctx* ctx, int head_dim, int max_seq, float theta, float** cos_out,
                     float** sin_out);

}  // namespace shd
