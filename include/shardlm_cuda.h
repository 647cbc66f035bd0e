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
/* Failure-path self-test (no counterpart in the reference): enqueue a kernel that waits on a device
 * flag nothing sets, bounded by limit_ms (1..2000) of GPU time, then records a timeout in the error
 * word exactly as an expired pipeline wait does. The next shd_sync returns SHD_ERR_TIMEOUT and clears
 * the word; the context stays usable. No fault, trap or hang is involved. */
int shd_wait_selftest(shd_ctx* ctx, int limit_ms);
/* Number of kernels this context has launched so far (for launch accounting in benchmarks). */
int64_t shd_launch_count(shd_ctx* ctx);

/* ----------------------------------------------------------------------------------------------
 * Weights
 * -------------------------------------------------------------------------------------------- */

/* Row orders of the tiled device format: blocks of 32 output rows x 256 input columns (bf16,
 * 16 KB), block (t, c) at offset (t * column_blocks + c) * 16 KB, zero-padded. */
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
 * nullable, out_features floats in the same row order as w) is added to the server share.
 * Reads the inputs in the context's stream order and returns once the tiles are written (it
 * synchronizes that stream), so the weight may then be used from any stream.
 * Every shd_weight_* constructor returns a complete weight in this sense. */
int shd_weight_from_bf16(shd_ctx* ctx, const uint16_t* w_out_in_dev, const float* bias_dev,
                         int in_features, int out_features, int rows, int head_dim,
                         shd_weight** out);
/* v1 ring weight: LinearServer::new (crates/sharing/src/linear.rs:186-214), host [in][out] i32
 * Q16.16 raw values, optional host i32 bias added (wrapping) to the server share. */
int shd_weight_upload_i32(shd_ctx* ctx, const int32_t* w_in_out_host, const int32_t* bias_host,
                          int in_features, int out_features, shd_weight** out);
/* Frees the weight; no call that reads it may still be running on any stream. */
int shd_weight_destroy(shd_weight* w);
/* Bytes the weight occupies on the device (tiled, padded). */
int64_t shd_weight_device_bytes(const shd_weight* w);

/* ----------------------------------------------------------------------------------------------
 * Share-wise linear layers
 * -------------------------------------------------------------------------------------------- */

/* GpuSecureLinear::forward_secure_gpu_tensor (crates/v2/sharing/src/secure_linear.rs:357-404):
 *   yc = xc . W^T (+ residual_c),   ys = xs . W^T + bias (+ residual_s)
 * xc, xs: [M][in]; yc, ys, residual_*: [M][out]. Few rows (up to 4 for weights under 48 M entries,
 * up to 2 for larger ones): one streaming pass over W on the CUDA cores serves both shares and all
 * rows. More rows: the tcgen05 tensor-core path, each f32 share split
 * exactly into three bf16 terms, f32 accumulation in tensor memory (same tolerance). bias (device,
 * nullable, [out]) overrides the bias stored with the weight when given.
 * residual_c/residual_s are both null or both set (secure_add_gpu fused in,
 * crates/v2/sharing/src/secure_nonlinear_gpu.rs:195-212). Inputs whose rows are not 16-byte
 * aligned (in % 4 != 0) are first copied into context scratch. The f32 result agrees with the
 * reference's sequential order within the f32 summation bound 2*gamma_in*sum|x||W|. */
int shd_linear_dual_f32(shd_ctx* ctx, const shd_weight* w, const float* bias, const float* xc,
                        const float* xs, float* yc, float* ys, int M, const float* residual_c,
                        const float* residual_s);

/* Allocation-free form of shd_linear_dual_f32 (no counterpart in the reference). For callers that
 * cannot allocate device memory while they run a layer -- a host framework that owns and freezes the
 * GPU's memory up front, or a request path that must not allocate. Same computation and arguments
 * (weight from an earlier shd_weight_* call; stream = the caller's cudaStream_t, NULL = legacy
 * default stream), but the split-K scratch is a static device array of about 1.3 MB that every GPU
 * loading the library keeps until exit; nothing is allocated or freed. Limits: out_features <=
 * 262144, in_features % 4 == 0 and 16-byte aligned rows (SHD_ERR_ARG otherwise). The first call on
 * a device looks up the array's device address and, with lazy module loading, may be when the
 * array is placed in device memory: make one call per device before the host framework freezes
 * device memory and before any stream capture. All calls share the array (its tile counters are
 * cleared at the start of each call): calls that overlap on the GPU race. The weight and the call
 * must not overlap its shd_weight_destroy. Device-side timeouts are not reported by this entry
 * point. */
int shd_linear_dual_f32_noalloc(const shd_weight* w, const float* bias, const float* xc,
                                const float* xs, float* yc, float* ys, int M,
                                const float* residual_c, const float* residual_s, void* stream);

/* LinearServer::handle_request / multiply_vector (crates/sharing/src/linear.rs:204-274), bit-exact:
 *   acc_j = sum_i (i64)x_i * (i64)W_ij (wrapping), y_j = (i32)(acc_j >> scale),
 *   ys_j = ys_j wrapping_add bias_j (bias from the weight, or `bias` when non-null).
 * xc, xs: [M][in] i32; yc, ys: [M][out] i32; any M and in (rows are staged when unaligned). */
int shd_linear_dual_ring(shd_ctx* ctx, const shd_weight* w, const int32_t* bias, const int32_t* xc,
                         const int32_t* xs, int32_t* yc, int32_t* ys, int M, int scale);

/* FixedVector::from_f64_slice / Fixed::from_f64 (crates/fixed_point/src/vector.rs:22-29,
 * fixed.rs:30-49) on n device doubles: out = round(x * 2^scale), half away from zero; NaN -> 0.
 * Synchronous: SHD_ERR_ARG "Overflow { value } / Underflow { value } at element i" for the first
 * element beyond i32 (the reference stops at the first error), "InvalidScale" for scale > 30. */
int shd_fixed_from_f64(shd_ctx* ctx, const double* x, int64_t n, int scale, int32_t* out);
/* SharePair::from_plaintext_seeded (crates/sharing/src/share.rs:116-135, Share::random_seeded
 * :44-54; LinearClient::new_seeded, linear.rs:88-106) on n device i32 values: xs[i] = word i of
 * ChaCha20Rng::seed_from_u64(seed) (rand_chacha 0.3.1 / rand_core 0.6.4, bit-exact), xc[i] = x[i]
 * wrapping_sub xs[i]. Asynchronous on the context's stream. */
int shd_ring_share_seeded(shd_ctx* ctx, const int32_t* x, int64_t n, uint64_t seed, int32_t* xc,
                          int32_t* xs);

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

/* ----------------------------------------------------------------------------------------------
 * Nonlinear reconstruct -> compute -> reshare ops, RoPE, attention, embedding shares, sampling
 * -------------------------------------------------------------------------------------------- */

/* secure_rms_norm_gpu / _approx / _mpc (crates/v2/sharing/src/secure_nonlinear_gpu.rs:53-95,
 * secure_nonlinear.rs:174-205, secure_nonlinear_mpc.rs:63-110) on M rows of n: reconstruct,
 * y = x * inv_rms * gamma (variant formula), reshare (y - mask, mask) (mask NULL -> (y, 0)). */
int shd_rmsnorm_reshare(shd_ctx* ctx, const float* xc, const float* xs, const float* gamma,
                        float eps, int variant, const float* mask, float* yc, float* ys, int M,
                        int n);
/* secure_swiglu_gpu / _approx / _mpc (secure_nonlinear_gpu.rs:131-158, secure_nonlinear.rs:354-380,
 * secure_nonlinear_mpc.rs:112-163): silu(g) * u on reconstructed values, then reshare. */
int shd_swiglu_reshare(shd_ctx* ctx, const float* gc, const float* gs, const float* uc,
                       const float* us, int variant, const float* mask, float* yc, float* ys,
                       int64_t n);
/* secure_silu_gpu / secure_silu_approx (secure_nonlinear_gpu.rs:28-48, secure_nonlinear.rs:131-158). */
int shd_silu_reshare(shd_ctx* ctx, const float* xc, const float* xs, int variant, const float* mask,
                     float* yc, float* ys, int64_t n);
/* RopeFrequencies::new (crates/v2/sharing/src/secure_attention.rs:42-63): the cos/sin table is built
 * on the host with libm powf/cosf/sinf in f32 exactly as the reference does, then uploaded. */
int shd_rope_init(shd_ctx* ctx, int head_dim, int max_seq, float theta);
/* RopeFrequencies::apply_to_share (secure_attention.rs:84-121) on both shares, in place, rows m at
 * positions pos + m: [x0 c - x1 s, x0 s + x1 c] with the reference's rounding (no FMA). */
int shd_rope_shares(shd_ctx* ctx, float* xc, float* xs, int M, int n_heads, int head_dim, int pos);
/* secure_attention_approx (crates/v2/sharing/src/secure_nonlinear.rs:287-333; variant APPROX/GPU)
 * or compute_mpc_attention_on_shares (crates/v2/server/src/routes/secure_inference_mpc.rs:568-663;
 * variant MPC) for M query rows: q [M][H*d] reconstructed, caches [kv_capacity][Hkv*d]
 * reconstructed, row m attends positions [0, pos_host[m]]. Output reshared (attn - mask, mask). */
int shd_attn_decode(shd_ctx* ctx, const float* q, const float* k_cache, const float* v_cache,
                    int kv_capacity, int H, int Hkv, int head_dim, const int32_t* pos_host, int M,
                    int variant, const float* mask, float* out_c, float* out_s);
/* The same attention for a block of M consecutive prompt positions pos0 .. pos0 + M - 1 of one
 * sequence (the prefill layer loop; the reference runs them one by one on the CPU), each row
 * attending to [0, its position], on the tensor cores: Q, K and V split exactly into three bf16
 * terms, QK^T and PV as tcgen05 MMAs with f32 accumulation, online softmax. q [M][H*128],
 * caches [kv_capacity][Hkv*128] (rows up to pos0 + M - 1 written), mask/out [M][H*128].
 * head_dim must be 128. */
int shd_attn_prefill(shd_ctx* ctx, const float* q, const float* k_cache, const float* v_cache,
                     int kv_capacity, int H, int Hkv, int head_dim, int pos0, int M, int variant,
                     const float* mask, float* out_c, float* out_s);
/* Server-side embedding share generation (get_embeddings_direct, crates/v2/server/src/routes/
 * secure_inference.rs:387-460): e = bf16 table row, server share uniform [0,1) (24-bit, rand's
 * Standard f32 construction) from Philox(seed, counter + m), client share e - s. */
int shd_embed_shares(shd_ctx* ctx, const uint16_t* table, int vocab, int hidden,
                     const int32_t* tokens, int M, uint64_t seed, uint64_t counter, float* hc,
                     float* hs);
/* get_embeddings_direct exactly as the reference draws it (secure_inference.rs:387-460): one
 * ChaCha20Rng::from_seed(session_id16 || 16 zero bytes) per request, token t's element k takes
 * keystream word t*hidden + k, s = (word >> 8) * 2^-24, c = e - s; tokens: n_tokens device ids
 * (out of range -> SHD_ERR_ARG at shd_sync, as the reference's InvalidRequest); hc, hs:
 * [n_tokens][hidden]. session_id16 is host memory (the UUID's 16 bytes). */
int shd_embed_shares_session(shd_ctx* ctx, const uint16_t* table, int vocab, int hidden,
                             const int32_t* tokens, int n_tokens, const uint8_t* session_id16,
                             float* hc, float* hs);
/* Client reconstruct + greedy sample (crates/v2/client/src/lib.rs:604-640): argmax of lc + ls,
 * the LAST index among equal maxima (Iterator::max_by). NaN -> SHD_ERR_NUMERIC at shd_sync. */
int shd_argmax_reconstruct(shd_ctx* ctx, const float* lc, const float* ls, int V, int M,
                           int32_t* tokens);

/* ----------------------------------------------------------------------------------------------
 * V3-OT: the server's side of the OT function-table lookups
 * -------------------------------------------------------------------------------------------- */

/* StandardOtTables::new(table_size) (crates/v2/sharing/src/secure_nonlinear_ot.rs:44-72,554-575):
 * writes [4][table_size] f32 to dev_out -- SiLU on [-8, 8], exp on [-10, 0], 1/sqrt on [0.01, 10],
 * 1/x on [0.01, 100] -- built with the reference's f32 operations and libm calls (identical bits).
 * Synchronous. */
int shd_ot_standard_tables(shd_ctx* ctx, int table_size, float* dev_out);
/* IknpOtExtension::process_query (crates/ot/src/iknp.rs:495-572) for one batch query against a
 * device-resident table (row_bytes per row, table_bytes / row_bytes rows): per entry, the item key
 * from SHA-256 over the session commitment (32 host bytes), the batch seed, the entry index and
 * ctr; the index and row key decrypted with its AES-128 PRF; the row masked with the row key's PRF.
 * One GPU thread per entry. query / response are host bytes (the route's Vec<u8>): query = u16 m ||
 * seed[32] || m x 20 bytes; response = m x row_bytes. *response_len = m * row_bytes; a NULL or small
 * `response` fails with SHD_ERR_ARG naming the size. SHD_ERR_ARG "InvalidMessageFormat" for a
 * malformed query, "InvalidIndex at entry j" when entry j's index is past the table (the first
 * such entry, as the reference stops there). Synchronous. */
int shd_ot_process_query(shd_ctx* ctx, const uint8_t* commitment32, uint64_t ctr, const uint8_t* query,
                         size_t query_len, const uint8_t* table_dev, size_t table_bytes, int row_bytes,
                         uint8_t* response, size_t response_cap, size_t* response_len);

/* ----------------------------------------------------------------------------------------------
 * Tensor parallelism (NCCL over NVLink, loaded at run time). Replaces the host-mediated
 * GpuCommunicator::all_reduce_sum (crates/v2/core/src/comm.rs:95-136, "TODO: Implement NCCL" :105).
 * -------------------------------------------------------------------------------------------- */
/* ncclGetUniqueId into 128 bytes (rank 0 creates it and shares it with the others). */
int shd_tp_unique_id(void* out_128_bytes);
/* Join the TP group as `rank` of `world` on the context's device (world == 1: no NCCL). Collective:
 * also maps a receive buffer of every rank into this one through CUDA IPC (NVLink / NVSwitch peer
 * memory) for the one-shot all-reduce of decode-sized messages; when any rank cannot, all use NCCL. */
int shd_tp_init(shd_ctx* ctx, int rank, int world, const void* unique_id_128_bytes);
int shd_tp_destroy(shd_ctx* ctx);
/* 1 when the peer-memory all-reduce is set up (messages up to 2 x 8 rows x 8192 floats use it: each
 * rank stores its partial into every rank's slot, then every rank sums the slots in rank order, so
 * all ranks hold identical sums); 0 when every all-reduce goes through NCCL. */
int shd_tp_peer_path(const shd_ctx* ctx);
/* In-place sum over the group of n floats on the context's stream -- the packed [2][M][h] partial
 * shares of a row-parallel projection -- then a host wait bounded by timeout_ms (<= 0: unbounded);
 * on timeout the communicator is aborted and SHD_ERR_TIMEOUT returned. */
int shd_allreduce_shares(shd_ctx* ctx, float* buf, size_t n, int timeout_ms);

/* ----------------------------------------------------------------------------------------------
 * Whole-model secret-shared forward pass: the layer loops of batched_full_forward_gpu /
 * generate_token_gpu (crates/v2/server/src/routes/secure_inference.rs:1553-1796), batched_prefill_
 * gpu_v3 (:2299-2632) and mpc_prefill (routes/secure_inference_mpc.rs:163-562), with the KV cache
 * resident on the device (reconstructed f32, as the reference holds it) and decode steps replayed
 * from a CUDA graph. Tensor parallel over tp_world ranks (one process per GPU): column-parallel
 * q/k/v and gate/up, row-parallel o/down with an NCCL all-reduce of the packed partial shares.
 * -------------------------------------------------------------------------------------------- */
typedef struct shd_model_config {
  int hidden, n_layers, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  float rope_theta, rms_eps;
  int max_seq;          /* KV capacity per sequence slot (also the RoPE table length) */
  int max_batch;        /* sequence slots decoded together (<= 8)                      */
  int variant_decode;   /* SHD_NL_* for norms / SwiGLU in decode (reference: APPROX)   */
  int variant_prefill;  /* SHD_NL_* in prefill (reference V3: GPU; V3-MPC: MPC)        */
  int variant_attn;     /* SHD_NL_APPROX or SHD_NL_MPC                                 */
  uint64_t share_seed;  /* seed of the embedding-share generator                       */
  int tp_rank, tp_world;
} shd_model_config;

/* This rank's slice of the model under tensor parallelism (computed by shd_model_create). */
typedef struct shd_shard_info {
  int q_head_begin, q_head_count;   /* local query heads                                  */
  int kv_head_begin, kv_head_count; /* kv heads those query heads use (may be replicated) */
  int inter_begin, inter_count;     /* local slice of the MLP intermediate dimension      */
  int vocab_begin, vocab_count;     /* local lm_head rows                                 */
} shd_shard_info;

int shd_model_create(shd_ctx* ctx, const shd_model_config* cfg, shd_model** out);
int shd_model_destroy(shd_model* m);
int shd_model_shard_info(const shd_model* m, shd_shard_info* out);
/* The same slice computed on the host for any (tp_rank, tp_world) of `cfg`, without a device or a
 * context (no counterpart in the reference, whose TP refuses head counts that do not divide,
 * crates/v2/core/src/parallel.rs:89-98). Query heads and vocab rows split evenly (the last rank
 * takes the remainder), the intermediate dimension in blocks of 16; kv heads are those the local
 * query heads read, so a kv head shared by two ranks is replicated on both. SHD_ERR_ARG on a
 * config shd_model_create would refuse for its shape or rank. */
int shd_tp_plan(const shd_model_config* cfg, shd_shard_info* out);
/* Layer weights of this rank's shard, DEVICE bf16 in [out][in] (safetensors) layout; copied.
 * wq [q_count*d][h], wk/wv [kv_count*d][h], wo [h][q_count*d], wg/wu [inter_count][h],
 * wd [h][inter_count]; biases f32 (nullable); norms f32 [h]. */
int shd_model_set_layer(shd_model* m, int layer, const uint16_t* wq, const uint16_t* wk,
                        const uint16_t* wv, const uint16_t* wo, const uint16_t* wg,
                        const uint16_t* wu, const uint16_t* wd, const float* bq, const float* bk,
                        const float* bv, const float* input_norm, const float* post_attn_norm);
/* Embedding table bf16 [vocab][h] (full, every rank), lm_head bf16 [vocab_count][h] of this rank
 * (tied models pass the embedding rows), final norm f32 [h]. Device pointers; copied. */
int shd_model_set_embedding(shd_model* m, const uint16_t* table);
int shd_model_set_head(shd_model* m, const uint16_t* lm_head, const float* final_norm);
/* V3-MPC reshare masks: per layer `stride` floats (device), sliced as mpc_prefill slices its
 * triple store: [0,h) input norm, [h, h+H*d) attention, [2h,3h) post-attention norm, [3h, 3h+I)
 * SwiGLU; the final norm uses layer L-1's [0,h). NULL clears (V3: reshare (y, 0)). */
int shd_model_set_masks(shd_model* m, const float* masks, int64_t stride);
/* Forget all sequences. */
int shd_model_reset(shd_model* m);
/* Prefill a prompt into sequence slot `slot` (chunks of up to 512 positions through the tensor-core
 * linears and prefill attention); writes the greedy next token to *next_token_host and leaves the
 * slot ready to decode. Synchronous. */
int shd_model_prefill(shd_model* m, int slot, const int32_t* tokens_host, int n,
                      int32_t* next_token_host);
/* Enqueue n_steps greedy decode steps for slots [0, n_active) from a captured CUDA graph; no host
 * synchronisation. Tokens accumulate on the device; read them with shd_model_read_tokens. */
int shd_model_decode_async(shd_model* m, int n_steps);
/* Copy the last `count` decoded steps' tokens ([count][n_active]) to the host (synchronises). */
int shd_model_read_tokens(shd_model* m, int count, int32_t* tokens_host);
/* generate_token_gpu semantics with host buffers (secure_inference.rs:1744-1796): hidden shares in
 * (H2D), all layers at the slot's next position, final norm, lm_head; logit shares out (D2H, the
 * full vocabulary on every rank). Synchronous. */
int shd_model_forward_host(shd_model* m, int slot, const float* hc_host, const float* hs_host,
                           float* logits_c_host, float* logits_s_host);
/* shd_model_forward_host for M sequences at once (generate_token_gpu of M sessions served in one
 * pass): row r is the next position of slot slots[r] (distinct slots); hidden shares in as
 * [M][hidden] client and server arrays, logit shares out as [M][vocab] arrays (the full vocabulary
 * on every rank). One weight pass serves all rows. Synchronous. */
int shd_model_forward_host_rows(shd_model* m, int M, const int32_t* slots, const float* hc_host,
                                const float* hs_host, float* logits_c_host, float* logits_s_host);
/* batched_prefill_gpu_v3 (secure_inference.rs:2299-2632) as the reference's route takes it: the
 * client's hidden-state shares of n prompt positions (host [n][h] each, get_embeddings_direct's
 * output) instead of token ids. Optional outputs (pairs, nullable): the last position's logit
 * shares [vocab] and its final hidden state shares [h] (the residual stream after the last layer).
 * The KV cache stays on the device; next_token_host (nullable) = greedy token. Synchronous. */
int shd_model_prefill_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host, int n,
                             float* logits_c_host, float* logits_s_host, float* final_c_host,
                             float* final_s_host, int32_t* next_token_host);
/* The reconstructed K and V rows of positions [pos0, pos0 + n) of a slot, every layer, as the
 * reference's prefill response carries them: host [n_layers][n][kv_dim] each (this rank's kv
 * heads under tensor parallelism). Synchronous. */
int shd_model_read_kv(shd_model* m, int slot, int pos0, int n, float* k_host, float* v_host);
/* shd_model_forward_host that also returns the position's output hidden state shares [h]
 * (BinaryDecodeResponse.hidden_*); hidden outputs nullable (as a pair). */
int shd_model_forward_host_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host,
                                  float* logits_c_host, float* logits_s_host, float* hidden_c_host,
                                  float* hidden_s_host);
/* The reference's binary wire format (crates/v2/server/src/routes/binary_protocol.rs:21-81; bincode
 * 1.3.3 default encoding: little-endian fixed-width integers, Vec<f32> = u64 length + raw f32s,
 * fields in declaration order). shd_bincode_prefill decodes a BinaryPrefillRequest, prefills it
 * into `slot` and encodes the BinaryPrefillResponse (batched_prefill_gpu_v3_binary,
 * secure_inference.rs:2635-2700); include_kv = 0 leaves k_cache and v_cache empty (the cache stays
 * on the device for decode). shd_bincode_decode takes a BinaryDecodeRequest (position must equal
 * the slot's length) and returns a BinaryDecodeResponse. *resp_len receives the response size;
 * a NULL or too small `resp` fails with SHD_ERR_ARG before any work, naming the size needed.
 * Malformed requests (truncated, trailing bytes, wrong dimensions) fail with SHD_ERR_ARG
 * ("Invalid binary request: ..."), as the route's InvalidRequest. Single-GPU models only. */
int shd_bincode_prefill(shd_model* m, int slot, const uint8_t* req, size_t req_len, int include_kv,
                        uint8_t* resp, size_t resp_cap, size_t* resp_len);
int shd_bincode_decode(shd_model* m, int slot, const uint8_t* req, size_t req_len, uint8_t* resp,
                       size_t resp_cap, size_t* resp_len);
/* Current length (positions held in the KV cache) of a slot. */
int shd_model_seq_len(const shd_model* m, int slot);
/* Kernels launched by one captured decode step (0 before the first decode). */
int64_t shd_model_step_launches(const shd_model* m);
/* Profiling: when on, the captured decode step records CUDA events around every share-wise linear
 * and attention launch; shd_model_linear_times then returns, for the most recent step, the summed
 * device time (ms) and the summed weight bytes of the launches of each kind: [0] qkv, [1] o,
 * [2] gate/up, [3] down, [4] lm_head, [5] attention (bytes 0). Turning it on or off re-captures
 * the graph at the next decode. */
int shd_model_set_profiling(shd_model* m, int on);
int shd_model_linear_times(shd_model* m, float* ms_out6, double* bytes_out6);
/* Timeline: shd_model_set_profiling(m, 2) makes the captured decode step stamp %globaltimer (ns)
 * inside the kernels themselves, without cutting the programmatic overlap between them. After a
 * decode, shd_model_timeline returns one record per traced launch in launch order: kinds[i] as
 * above (0 qkv, 1 o, 2 gate/up, 3 down, 4 lm_head, 5 attention, 6 tensor-parallel peer-exchange
 * receive; its field 3 is the last CTA's end of polling, before its wait) and stamps[8 i + f] for
 * f = 0 first CTA entry, 1 last CTA entry, 2 first return from the wait on the previous kernel,
 * 3 last end of the prologue (wait and fused norm), 4 first exit, 5 last exit (fields 1, 3, 5
 * stored complemented; all ones = not reached). Launches on the tensor-core path are not stamped.
 * With cap smaller than the count (or null outputs) only *n_out is set. */
int shd_model_timeline(shd_model* m, int cap, int32_t* kinds, uint64_t* stamps, int* n_out);

#ifdef __cplusplus
}
#endif
#endif /* SHARDLM_CUDA_H */
