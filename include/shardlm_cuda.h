/*
 * shardlm_cuda.h -- C ABI of libshardlm_cuda.so, the B200 (sm_100a) kernels behind ShardLM's
 * secret-shared transformer forward pass.
 *
 * Conventions
 *  - Every entry point returns 0 (SHD_OK) or a negative SHD_ERR_* code. The message of the last
 *    failure on a context is returned by shd_last_error().
 *  - Tensor pointers are DEVICE pointers owned by the caller (cudarc CudaSlice in the Rust server)
 *    unless a parameter name ends in _host. The library never frees caller memory.
 *  - All work is enqueued on the context's stream (shd_set_stream); nothing synchronises unless the
 *    entry point says so. Each entry point makes the context's device current itself, so calls may
 *    come from any host thread, but one context must not be used by two threads at once.
 *  - Shares are additive: value = client + server. f32 shares follow crates/v2 (IEEE f32 add);
 *    ring shares follow crates/fixed_point (Z_2^32, wrapping i32, Q16.16 by default).
 *  - Row-major [M][features] activations; M is the number of token rows processed together.
 *  - There is no CPU fallback: without a usable sm_100 GPU every entry point fails.
 */
#ifndef SHARDLM_CUDA_H
#define SHARDLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SHD_OK 0
#define SHD_ERR_ARG (-1)         /* bad argument: shape, alignment, null pointer          */
#define SHD_ERR_CUDA (-2)        /* a CUDA runtime call failed                             */
#define SHD_ERR_NCCL (-3)        /* an NCCL call failed or NCCL could not be loaded        */
#define SHD_ERR_TIMEOUT (-4)     /* a bounded device-side or collective wait ran out       */
#define SHD_ERR_UNSUPPORTED (-5) /* valid request this build does not implement            */
#define SHD_ERR_NUMERIC (-6)     /* non-finite value where the reference would panic       */

/* Nonlinear variants: which reference formula a reconstruct-compute-reshare op follows. */
#define SHD_NL_APPROX 0 /* secure_*_approx (crates/v2/sharing/src/secure_nonlinear.rs:131-380):
                           RMSNorm 1/sqrt, SiLU sigmoid on clamp(x,-20,20), softmax clamp(-40,40) */
#define SHD_NL_GPU 1    /* NVRTC kernels of crates/v2/core/src/kernel.rs:38-144 (prefill path):
                           RMSNorm rsqrtf, SiLU x/(1+exp(-x)) without clamp                   */
#define SHD_NL_MPC 2    /* secure_*_mpc (crates/v2/sharing/src/secure_nonlinear_mpc.rs:63-250):
                           guards on rms and non-finite values, mask reshare (y - m, m)       */

typedef struct shd_ctx shd_ctx;
typedef struct shd_weight shd_weight;
typedef struct shd_model shd_model;

/* ----------------------------------------------------------------------------------------------
 * Context
 * -------------------------------------------------------------------------------------------- */

/* Create a context on CUDA device `device` (replaces GpuDevice::new + KernelContext::new,
 * crates/v2/core/src/gpu.rs:21-170, crates/v2/core/src/kernel.rs:677-733). Allocates the
 * context's scratch (split-K partials, tile counters, an error word) once. */
int shd_init(int device, shd_ctx** out);
int shd_destroy(shd_ctx* ctx);
/* Use the caller's stream (a cudaStream_t) for all later work; NULL = the legacy default stream. */
int shd_set_stream(shd_ctx* ctx, void* stream);
const char* shd_last_error(shd_ctx* ctx);
/* Synchronise the stream and report any error a kernel recorded in the context's error word
 * (a bounded wait that ran out -> SHD_ERR_TIMEOUT). Clears the word. */
int shd_sync(shd_ctx* ctx);
/* Number of kernels this context has launched so far (for launch accounting in benchmarks). */
int64_t shd_launch_count(shd_ctx* ctx);

/* ----------------------------------------------------------------------------------------------
 * Weights
 * -------------------------------------------------------------------------------------------- */

/* Row orders of the tiled device format (see DESIGN.md "weight tiling"). */
#define SHD_ROWS_PLAIN 0   /* rows in output order                                          */
#define SHD_ROWS_QKV 1     /* fused q|k|v, RoPE pairs (i, i+head_dim/2) adjacent per head     */
#define SHD_ROWS_GATEUP 2  /* fused gate|up, 16 gate rows then the same 16 up rows per tile   */

/* GpuSecureLinear::from_cpu (crates/v2/sharing/src/secure_linear.rs:165-200): weight given in the
 * reference's host layout [in][out] f32. Values must be exact bf16 upcasts, as the reference's
 * always are (crates/v2/server/src/secure_weights.rs:432-440); any other value -> SHD_ERR_UNSUPPORTED.
 * The weight is stored on the device as tiled bf16, read once per call for both shares. */
int shd_weight_upload_f32_as_bf16(shd_ctx* ctx, const float* w_in_out_host, int in_features,
                                  int out_features, shd_weight** out);
/* Same weight from a DEVICE bf16 matrix in [out][in] layout (the safetensors / HF layout the
 * reference's loader reads, crates/v2/model/src/sharded_loader.rs:445-486). `rows` is one of
 * SHD_ROWS_*; for SHD_ROWS_QKV `out_features` = q_dim + 2*kv_dim and head_dim gives the pairing;
 * for SHD_ROWS_GATEUP `out_features` = 2*intermediate with gate rows first. bias (device,
 * nullable, out_features floats in the same row order as w) is added to the server share. */
int shd_weight_from_bf16(shd_ctx* ctx, const uint16_t* w_out_in_dev, const float* bias_dev,
                         int in_features, int out_features, int rows, int head_dim,
                         shd_weight** out);
/* v1 ring weight: LinearServer::new (crates/sharing/src/linear.rs:186-214), host [in][out] i32
 * Q16.16 raw values, optional host i32 bias added (wrapping) to the server share. */
int shd_weight_upload_i32(shd_ctx* ctx, const int32_t* w_in_out_host, const int32_t* bias_host,
                          int in_features, int out_features, shd_weight** out);
int shd_weight_destroy(shd_weight* w);
/* Bytes the weight occupies on the device (tiled, padded). */
int64_t shd_weight_device_bytes(const shd_weight* w);

/* ----------------------------------------------------------------------------------------------
 * Share-wise linear layers
 * -------------------------------------------------------------------------------------------- */

/* GpuSecureLinear::forward_secure_gpu_tensor (crates/v2/sharing/src/secure_linear.rs:357-404):
 *   yc = xc . W^T (+ residual_c),   ys = xs . W^T + bias (+ residual_s)
 * xc, xs: [M][in]; yc, ys, residual_*: [M][out]. One pass over W serves both shares and all M rows
 * (M <= 8). bias (device, nullable, [out]) overrides the bias stored with the weight when given.
 * residual_c/residual_s are both null or both set (secure_add_gpu fused in,
 * crates/v2/sharing/src/secure_nonlinear_gpu.rs:195-212). Requires in % 8 == 0 and 16-byte aligned
 * rows. f32 result within the tolerance stated in tests/test_linear.py of the reference's order. */
int shd_linear_dual_f32(shd_ctx* ctx, const shd_weight* w, const float* bias, const float* xc,
                        const float* xs, float* yc, float* ys, int M, const float* residual_c,
                        const float* residual_s);

/* LinearServer::handle_request / multiply_vector (crates/sharing/src/linear.rs:204-274), bit-exact:
 *   acc_j = sum_i (i64)x_i * (i64)W_ij (wrapping), y_j = (i32)(acc_j >> scale),
 *   ys_j = ys_j wrapping_add bias_j (bias from the weight, or `bias` when non-null).
 * xc, xs: [M][in] i32; yc, ys: [M][out] i32; M <= 8; in % 4 == 0. */
int shd_linear_dual_ring(shd_ctx* ctx, const shd_weight* w, const int32_t* bias, const int32_t* xc,
                         const int32_t* xs, int32_t* yc, int32_t* ys, int M, int scale);

/* ----------------------------------------------------------------------------------------------
 * Reconstruct / reshare and elementwise share ops (all device pointers, n elements)
 * -------------------------------------------------------------------------------------------- */

/* y = c + s (client-side reconstruct, crates/v2/client/src/lib.rs:638-640). */
int shd_reconstruct_f32(shd_ctx* ctx, const float* c, const float* s, float* y, int64_t n);
/* Reshare y as (y - mask, mask); mask == NULL gives (y, 0) as every V3 op does
 * (crates/v2/sharing/src/secure_nonlinear_mpc.rs:98-106). */
int shd_reshare_f32(shd_ctx* ctx, const float* y, const float* mask, float* out_c, float* out_s,
                    int64_t n);
/* secure_add_gpu (crates/v2/sharing/src/secure_nonlinear_gpu.rs:195-212): per-share add. */
int shd_add_shares(shd_ctx* ctx, const float* ac, const float* as, const float* bc,
                   const float* bs, float* yc, float* ys, int64_t n);

/* ----------------------------------------------------------------------------------------------
 * Beaver triples (V3-MPC)
 * -------------------------------------------------------------------------------------------- */

/* secure_multiply_batch / secure_multiply_mpc (crates/v2/sharing/src/beaver.rs:167-233), f32,
 * bit-exact with the reference's operation order (no FMA contraction):
 *   d = (xc - ac) + (xs - as), e = (yc - bc) + (ys - bs)
 *   zc = cc + ac*e + d*bc + d*e,  zs = cs + as*e + d*bs
 * d_out / e_out (nullable) receive the opened values. */
int shd_beaver_mul_f32(shd_ctx* ctx, const float* xc, const float* xs, const float* yc,
                       const float* ys, const float* ac, const float* as, const float* bc,
                       const float* bs, const float* cc, const float* cs, float* d_out,
                       float* e_out, float* zc, float* zs, int64_t n);
/* The same algebra over Z_2^32 with Fixed's wrapping add/sub/mul (crates/fixed_point/src/fixed.rs:
 * 78-105): z = x*y mod 2^32 exactly. trunc_shift > 0 additionally applies the two-party local
 * truncation of SecureML (client z_c >> f arithmetic, server -((-z_s) >> f)). */
int shd_beaver_mul_ring(shd_ctx* ctx, const uint32_t* xc, const uint32_t* xs, const uint32_t* yc,
                        const uint32_t* ys, const uint32_t* ac, const uint32_t* as,
                        const uint32_t* bc, const uint32_t* bs, const uint32_t* cc,
                        const uint32_t* cs, uint32_t* d_out, uint32_t* e_out, uint32_t* zc,
                        uint32_t* zs, int64_t n, int trunc_shift);
/* BeaverTriple::random (crates/v2/sharing/src/beaver.rs:44-68) with a counter-based generator
 * (Philox4x32-10 keyed by seed, element index + offset as counter) instead of thread_rng:
 * a, b ~ U(-1,1), c = a*b, server parts ~ U(-10,10), client = value - server. Any output may be
 * NULL. */
int shd_beaver_triples_f32(shd_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n, float* a,
                           float* b, float* c, float* ac, float* as, float* bc, float* bs,
                           float* cc, float* cs);
/* Ring triples: a, b uniform in Z_2^32, c = a*b mod 2^32, server parts uniform. */
int shd_beaver_triples_ring(shd_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n,
                            uint32_t* ac, uint32_t* as, uint32_t* bc, uint32_t* bs, uint32_t* cc,
                            uint32_t* cs);
/* Uniform f32 in [lo, hi) from the same generator (reshare masks, share generation). */
int shd_fill_uniform_f32(shd_ctx* ctx, uint64_t seed, uint64_t offset, float lo, float hi,
                         float* out, int64_t n);

#ifdef __cplusplus
}
#endif
#endif /* SHARDLM_CUDA_H */
