// Persistent decode step: one kernel launch runs a whole decode step of the secret-shared model as
// a list of jobs (embedding shares, per layer q/k/v + attention + o + gate/up + down, the head and
// the greedy token update). Host side: the job list is recorded from the same enqueue code that
// drives the per-kernel path, then uploaded once per batch size.
#pragma once

#include <vector>

#include "shd_gemv.cuh"
#include "shd_nonlinear.cuh"

namespace shd {

enum StepJobType : int { JOB_GEMV = 0, JOB_ATTN = 1, JOB_EMBED = 2, JOB_NORM = 3 };

// Profiling classes of jobs (the per-kind breakdown of shd_model_linear_times).
enum StepKind : int { KIND_QKV = 0, KIND_O = 1, KIND_GATEUP = 2, KIND_DOWN = 3, KIND_HEAD = 4, KIND_ATTN = 5, KIND_OTHER = 6 };

struct StepJob {
  int type;   // StepJobType
  int epi;    // JOB_GEMV: EPI_*
  int norm;   // JOB_GEMV: fused RMSNorm prologue (activations computed, not staged)
  int kind;   // StepKind
  double bytes;  // algorithmic weight bytes (profiling)
  GemvArgs g;
  AttnArgs at;
  EmbedArgs ea;
  NormArgs na;
};

struct StepArgs {
  const StepJob* jobs;
  int n_jobs;
  unsigned long long* sync;   // [0] grid-barrier arrivals, [1] abort flag; zeroed before each launch
  int* err;
  // greedy token update after the head (finish of the step)
  const unsigned long long* amax;
  int* tokens;
  int* pos;
  int* hist;
  int hist_cap;
  unsigned long long* step;
  int M;
  // pipeline geometry
  int nstages;
  int stage_bytes;
  int aux_floats;  // fused-norm activations / attention tile scratch
  // profiling (nullable): per job first start and last end of this launch, and running sums
  unsigned long long* prof_t;     // [2][n_jobs]: starts (reset to ~0), ends (reset to 0)
  unsigned long long* prof_acc;   // [n_jobs + 1]: summed spans in ns, [n_jobs] = launches
};

struct StepPlan {
  int M = 0;
  int n_jobs = 0;
  StepJob* d_jobs = nullptr;
  unsigned long long* d_sync = nullptr;
  float* d_attn_part = nullptr;
  int* d_attn_cnt = nullptr;
  unsigned long long* d_prof = nullptr;  // [2 * n_jobs] + [n_jobs + 1]
  int nstages = 0, stage_bytes = 0, aux_floats = 0;
  int grid = 0;  // CTAs: one or two per SM, all resident
  size_t smem = 0;
  std::vector<int> kinds;
  std::vector<double> bytes;
};

// Upload `jobs` as the step of M rows: chooses the pipeline geometry, the attention split and
// allocates the plan's buffers. SHD_ERR_UNSUPPORTED when the step does not fit one CTA per SM.
int step_plan_build(shd_ctx* ctx, StepPlan& plan, std::vector<StepJob>& jobs, int M);
void step_plan_free(StepPlan& plan);
// Enqueue one step on `stream`: reset the barrier, launch the persistent kernel.
int step_launch(shd_ctx* ctx, const StepPlan& plan, cudaStream_t stream, const unsigned long long* amax,
                int* tokens, int* pos, int* hist, int hist_cap, unsigned long long* step, bool profile);
// Mean per-kind span (ms) over the profiled launches and the algorithmic bytes per kind.
int step_prof_read(shd_ctx* ctx, const StepPlan& plan, float* ms_out6, double* bytes_out6);
int step_prof_reset(shd_ctx* ctx, const StepPlan& plan, cudaStream_t stream);

}  // namespace shd
