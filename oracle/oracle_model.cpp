// ORACLE (test infrastructure only): reconstruct-compute-reshare nonlinear ops, RoPE, attention and
// the per-token layer loop of the reference, restated on the CPU. See oracle.cpp for the rules.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#define ORC_API extern "C" __attribute__((visibility("default")))

enum { NL_APPROX = 0, NL_GPU = 1, NL_MPC = 2 };

static inline float bf16f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

extern "C" void orc_linear_bf16(const uint16_t* w_in_out, const float* bias, int in, int out,
                                const float* xc, const float* xs, float* yc, float* ys, int M);

// ------------------------------------------------------------------------------------------------
// RopeFrequencies::new / apply_to_share (crates/v2/sharing/src/secure_attention.rs:42-121)
// ------------------------------------------------------------------------------------------------
ORC_API void orc_rope_table(int head_dim, int max_seq, float theta, float* cos_out, float* sin_out) {
  const int half = head_dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
  for (int p = 0; p < max_seq; ++p) {
    const float pf = (float)p;
    for (int i = 0; i < half; ++i) {
      cos_out[(size_t)p * half + i] = cosf(pf * inv[i]);
      sin_out[(size_t)p * half + i] = sinf(pf * inv[i]);
    }
  }
}

ORC_API void orc_rope_apply(const float* share, int n_heads, int head_dim, const float* cos_row,
                            const float* sin_row, float* out) {
  const int half = head_dim / 2;
  for (int h = 0; h < n_heads; ++h) {
    const int off = h * head_dim;
    for (int i = 0; i < half; ++i) {
      const float x0 = share[off + i], x1 = share[off + i + half];
      const float c = cos_row[i], s = sin_row[i];
      out[off + i] = x0 * c - x1 * s;
      out[off + i + half] = x0 * s + x1 * c;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// RMSNorm with reshare.
//  NL_APPROX: secure_rms_norm_approx (crates/v2/sharing/src/secure_nonlinear.rs:174-205)
//  NL_GPU   : secure_rms_norm_gpu -> rms_norm_kernel (crates/v2/core/src/kernel.rs:92-144);
//             the kernel's rsqrtf is approximated here by 1/sqrtf (tolerance, not bit-exact)
//  NL_MPC   : secure_rms_norm_mpc (crates/v2/sharing/src/secure_nonlinear_mpc.rs:63-110)
// mask (nullable): reshare (y - mask[i], mask[i]); null -> (y, 0).
// ------------------------------------------------------------------------------------------------
ORC_API void orc_rmsnorm_reshare(const float* xc, const float* xs, const float* gamma, float eps,
                                 int variant, const float* mask, float* yc, float* ys, int n) {
  std::vector<float> x(n);
  for (int i = 0; i < n; ++i) x[i] = xc[i] + xs[i];
  float sum_sq = 0.0f;
  for (int i = 0; i < n; ++i) sum_sq += x[i] * x[i];
  const float mean_sq = sum_sq / (float)n;
  float inv;
  if (variant == NL_GPU) {
    inv = 1.0f / sqrtf(mean_sq + eps);
  } else {
    const float rms = sqrtf(mean_sq + eps);
    if (variant == NL_MPC)
      inv = (rms > 1e-6f && std::isfinite(rms)) ? 1.0f / rms : 1.0f;
    else
      inv = 1.0f / rms;
  }
  for (int i = 0; i < n; ++i) {
    float r = x[i] * inv * gamma[i];
    if (variant == NL_MPC && !std::isfinite(r)) r = 0.0f;
    const float m = mask ? mask[i] : 0.0f;
    yc[i] = r - m;
    ys[i] = m;
  }
}

static inline float silu_v(float g, int variant) {
  if (variant == NL_APPROX) {
    const float gc = fminf(fmaxf(g, -20.0f), 20.0f);
    const float sig = 1.0f / (1.0f + expf(-gc));
    return g * sig;
  } else if (variant == NL_GPU) {
    return g / (1.0f + expf(-g));
  }
  if (!std::isfinite(g)) return 0.0f;
  const float sig = 1.0f / (1.0f + expf(-g));
  return g * sig;
}

static inline float swiglu_v(float g, float u, int variant) {
  const float s = silu_v(g, variant);
  if (variant == NL_MPC) {
    if (!(std::isfinite(s) && std::isfinite(u))) return 0.0f;
    const float p = s * u;
    return std::isfinite(p) ? p : 0.0f;
  }
  return s * u;
}

// secure_swiglu_approx (secure_nonlinear.rs:354-380), secure_swiglu_gpu (secure_nonlinear_gpu.rs:
// 131-158), secure_swiglu_mpc (secure_nonlinear_mpc.rs:112-163).
ORC_API void orc_swiglu_reshare(const float* gc, const float* gs, const float* uc, const float* us,
                                int variant, const float* mask, float* yc, float* ys, int n) {
  for (int i = 0; i < n; ++i) {
    const float g = gc[i] + gs[i];
    const float u = uc[i] + us[i];
    const float r = swiglu_v(g, u, variant);
    const float m = mask ? mask[i] : 0.0f;
    yc[i] = r - m;
    ys[i] = m;
  }
}

// secure_silu_approx (secure_nonlinear.rs:131-158) / silu_kernel / MPC guard.
ORC_API void orc_silu_reshare(const float* xc, const float* xs, int variant, const float* mask,
                              float* yc, float* ys, int n) {
  for (int i = 0; i < n; ++i) {
    const float r = silu_v(xc[i] + xs[i], variant);
    const float m = mask ? mask[i] : 0.0f;
    yc[i] = r - m;
    ys[i] = m;
  }
}

// secure_softmax_approx (secure_nonlinear.rs:224-267) on already reconstructed scores.
static void softmax_approx(const float* s, int n, float* w) {
  if (n == 0) return;
  if (n == 1) {
    w[0] = 1.0f;
    return;
  }
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, s[i]);
  float sum = 0.0f;
  std::vector<float> e(n);
  for (int i = 0; i < n; ++i) {
    float x = s[i] - mx;
    x = fminf(fmaxf(x, -40.0f), 40.0f);
    e[i] = expf(x);
    sum += e[i];
  }
  for (int i = 0; i < n; ++i) w[i] = e[i] / sum;
}

ORC_API void orc_softmax_approx(const float* sc, const float* ss, int n, float* w) {
  std::vector<float> s(n);
  for (int i = 0; i < n; ++i) s[i] = sc[i] + ss[i];
  softmax_approx(s.data(), n, w);
}

// Decode attention for one query row over kv_len cached positions.
//  NL_APPROX / NL_GPU: secure_attention_approx (secure_nonlinear.rs:287-333), output reshared
//                      as (attn - mask, mask) by the caller's rule ((attn, 0) when mask is null)
//  NL_MPC: compute_mpc_attention_on_shares (crates/v2/server/src/routes/secure_inference_mpc.rs:
//          568-663)
// q [H*d] reconstructed; kcache/vcache [kv_len][Hkv*d] reconstructed.
ORC_API void orc_attention(const float* q, const float* kcache, const float* vcache, int kv_len,
                           int H, int Hkv, int d, int variant, const float* mask, float* oc,
                           float* os) {
  const int group = H / Hkv;
  const float scale = 1.0f / sqrtf((float)d);
  const int kvd = Hkv * d;
  std::vector<float> out((size_t)H * d, 0.0f), sc(kv_len), w(kv_len);
  if (kv_len == 0) {
    for (int i = 0; i < H * d; ++i) {
      const float m = mask ? mask[i] : 0.0f;
      oc[i] = 0.0f - m;
      os[i] = m;
    }
    return;
  }
  for (int h = 0; h < H; ++h) {
    const int kvh = h / group;
    for (int t = 0; t < kv_len; ++t) {
      float s = 0.0f;
      for (int j = 0; j < d; ++j) s += q[h * d + j] * kcache[(size_t)t * kvd + kvh * d + j];
      sc[t] = s * scale;
    }
    if (variant == NL_MPC) {
      float mx = -INFINITY;
      for (int t = 0; t < kv_len; ++t) mx = fmaxf(mx, sc[t]);
      if (!std::isfinite(mx)) mx = 0.0f;
      float sum = 0.0f;
      for (int t = 0; t < kv_len; ++t) {
        w[t] = expf(sc[t] - mx);
        sum += w[t];
      }
      if (sum > 1e-10f && std::isfinite(sum)) {
        for (int t = 0; t < kv_len; ++t) w[t] = w[t] / sum;
      } else {
        for (int t = 0; t < kv_len; ++t) w[t] = 1.0f / (float)kv_len;
      }
      for (int j = 0; j < d; ++j) {
        float acc = 0.0f;
        for (int t = 0; t < kv_len; ++t) acc += w[t] * vcache[(size_t)t * kvd + kvh * d + j];
        out[h * d + j] = acc;
      }
    } else {
      softmax_approx(sc.data(), kv_len, w.data());
      for (int t = 0; t < kv_len; ++t)
        for (int j = 0; j < d; ++j) out[h * d + j] += w[t] * vcache[(size_t)t * kvd + kvh * d + j];
    }
  }
  for (int i = 0; i < H * d; ++i) {
    const float m = mask ? mask[i] : 0.0f;
    oc[i] = out[i] - m;
    os[i] = m;
  }
}

// Greedy sampling of the client (crates/v2/client/src/lib.rs:604-640): reconstruct, then
// max_by(partial_cmp) which returns the LAST index among equal maxima. Returns -1 on NaN
// (the reference's unwrap panics).
ORC_API int orc_argmax_last(const float* lc, const float* ls, int n) {
  int best = -1;
  float bv = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float v = lc[i] + ls[i];
    if (std::isnan(v)) return -1;
    if (best < 0 || v >= bv) {
      best = i;
      bv = v;
    }
  }
  return best;
}

// ------------------------------------------------------------------------------------------------
// Whole-model forward of one token position: the layer loop of batched_full_forward_gpu /
// generate_token_gpu (crates/v2/server/src/routes/secure_inference.rs:1601-1786) and, with
// NL_GPU, of batched_prefill_gpu_v3 (secure_inference.rs:2436-2590), with every linear layer on
// the CPU. Weights are bf16 in the reference's [in][out] host layout.
// ------------------------------------------------------------------------------------------------
struct OrcLayer {
  const uint16_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  const float *bq, *bk, *bv, *g1, *g2;
};

struct OrcModel {
  int h, L, H, Hkv, d, I, V, max_seq;
  float eps;
  std::vector<OrcLayer> layers;
  const uint16_t* lm_head = nullptr;  // [h][V]
  const float* final_norm = nullptr;
  std::vector<float> rope_cos, rope_sin;
  std::vector<std::vector<float>> kcache, vcache;  // per layer [t][Hkv*d]
  int len = 0;
};

ORC_API void* orc_model_create(int h, int L, int H, int Hkv, int d, int I, int V, float theta,
                               float eps, int max_seq) {
  OrcModel* m = new OrcModel();
  m->h = h; m->L = L; m->H = H; m->Hkv = Hkv; m->d = d; m->I = I; m->V = V;
  m->eps = eps;
  m->max_seq = max_seq;
  m->layers.resize(L);
  m->rope_cos.resize((size_t)max_seq * d / 2);
  m->rope_sin.resize((size_t)max_seq * d / 2);
  orc_rope_table(d, max_seq, theta, m->rope_cos.data(), m->rope_sin.data());
  m->kcache.assign(L, {});
  m->vcache.assign(L, {});
  return m;
}

ORC_API void orc_model_destroy(void* p) { delete static_cast<OrcModel*>(p); }

ORC_API void orc_model_set_layer(void* p, int l, const uint16_t* wq, const uint16_t* wk,
                                 const uint16_t* wv, const uint16_t* wo, const uint16_t* wg,
                                 const uint16_t* wu, const uint16_t* wd, const float* bq,
                                 const float* bk, const float* bv, const float* g1, const float* g2) {
  OrcModel* m = static_cast<OrcModel*>(p);
  m->layers[l] = {wq, wk, wv, wo, wg, wu, wd, bq, bk, bv, g1, g2};
}

ORC_API void orc_model_set_head(void* p, const uint16_t* lm_head, const float* final_norm) {
  OrcModel* m = static_cast<OrcModel*>(p);
  m->lm_head = lm_head;
  m->final_norm = final_norm;
}

// Give every layer a zero-filled cache of `len` positions (a bounded CPU sample at a late position
// without prefilling: attention cost depends on the length, not on the cached values).
ORC_API void orc_model_set_len(void* p, int len) {
  OrcModel* m = static_cast<OrcModel*>(p);
  const size_t kvd = (size_t)m->Hkv * m->d;
  for (auto& k : m->kcache) k.assign((size_t)len * kvd, 0.0f);
  for (auto& v : m->vcache) v.assign((size_t)len * kvd, 0.0f);
  m->len = len;
}

// The cached (reconstructed) K and V rows [L][n][Hkv*d] of positions [pos0, pos0 + n).
ORC_API int orc_model_get_kv(void* p, int pos0, int n, float* k_out, float* v_out) {
  OrcModel* m = static_cast<OrcModel*>(p);
  if (pos0 < 0 || n < 0 || pos0 + n > m->len) return -1;
  const size_t kvd = (size_t)m->Hkv * m->d;
  for (int l = 0; l < m->L; ++l) {
    std::memcpy(k_out + (size_t)l * n * kvd, m->kcache[l].data() + (size_t)pos0 * kvd, (size_t)n * kvd * 4);
    std::memcpy(v_out + (size_t)l * n * kvd, m->vcache[l].data() + (size_t)pos0 * kvd, (size_t)n * kvd * 4);
  }
  return 0;
}

ORC_API void orc_model_reset(void* p) {
  OrcModel* m = static_cast<OrcModel*>(p);
  for (auto& k : m->kcache) k.clear();
  for (auto& v : m->vcache) v.clear();
  m->len = 0;
}

// masks: nullable; else per layer `mask_stride` floats laid out as the MPC route slices its
// triple store: [0,h) input norm, [h, h+H*d) attention, [2h,3h) post-attention norm,
// [3h, 3h+I) SwiGLU; the final norm uses layer L-1's [0,h).
// n_layers_run < L runs only the first layers (bounded CPU samples); logits are then not produced.
ORC_API int orc_model_forward(void* p, const float* hc_in, const float* hs_in, int variant,
                              int attn_variant, const float* masks, int64_t mask_stride,
                              int n_layers_run, float* hc_out, float* hs_out, float* logits_c,
                              float* logits_s) {
  OrcModel* m = static_cast<OrcModel*>(p);
  const int h = m->h, H = m->H, Hkv = m->Hkv, d = m->d, I = m->I;
  const int qd = H * d, kvd = Hkv * d;
  const int pos = m->len;
  if (pos >= m->max_seq) return -1;
  const float* cosr = m->rope_cos.data() + (size_t)pos * d / 2;
  const float* sinr = m->rope_sin.data() + (size_t)pos * d / 2;
  std::vector<float> hc(hc_in, hc_in + h), hs(hs_in, hs_in + h);
  std::vector<float> nc(h), ns(h), qc(qd), qs(qd), kc(kvd), ks(kvd), vc(kvd), vs(kvd);
  std::vector<float> q(qd), ac(qd), as(qd), oc(h), os(h), gc(I), gs(I), uc(I), us(I), xc(I), xs(I);
  std::vector<float> dc(h), ds(h), tmp(std::max(qd, kvd));
  const int Lrun = (n_layers_run > 0 && n_layers_run < m->L) ? n_layers_run : m->L;
  for (int l = 0; l < Lrun; ++l) {
    const OrcLayer& w = m->layers[l];
    const float* mk = masks ? masks + (size_t)l * mask_stride : nullptr;
    // input norm
    orc_rmsnorm_reshare(hc.data(), hs.data(), w.g1, m->eps, variant, mk ? mk : nullptr, nc.data(), ns.data(), h);
    // q/k/v share-wise + RoPE per share
    orc_linear_bf16(w.wq, w.bq, h, qd, nc.data(), ns.data(), qc.data(), qs.data(), 1);
    orc_linear_bf16(w.wk, w.bk, h, kvd, nc.data(), ns.data(), kc.data(), ks.data(), 1);
    orc_linear_bf16(w.wv, w.bv, h, kvd, nc.data(), ns.data(), vc.data(), vs.data(), 1);
    orc_rope_apply(qc.data(), H, d, cosr, sinr, tmp.data());
    std::memcpy(qc.data(), tmp.data(), qd * 4);
    orc_rope_apply(qs.data(), H, d, cosr, sinr, tmp.data());
    std::memcpy(qs.data(), tmp.data(), qd * 4);
    orc_rope_apply(kc.data(), Hkv, d, cosr, sinr, tmp.data());
    std::memcpy(kc.data(), tmp.data(), kvd * 4);
    orc_rope_apply(ks.data(), Hkv, d, cosr, sinr, tmp.data());
    std::memcpy(ks.data(), tmp.data(), kvd * 4);
    // reconstructed K, V appended to this layer's cache; reconstructed Q
    auto& K = m->kcache[l];
    auto& Vv = m->vcache[l];
    K.resize((size_t)(pos + 1) * kvd);
    Vv.resize((size_t)(pos + 1) * kvd);
    for (int i = 0; i < kvd; ++i) {
      K[(size_t)pos * kvd + i] = kc[i] + ks[i];
      Vv[(size_t)pos * kvd + i] = vc[i] + vs[i];
    }
    for (int i = 0; i < qd; ++i) q[i] = qc[i] + qs[i];
    orc_attention(q.data(), K.data(), Vv.data(), pos + 1, H, Hkv, d, attn_variant,
                  mk ? mk + h : nullptr, ac.data(), as.data());
    // o projection on (attn shares), residual per share: o + h
    orc_linear_bf16(w.wo, nullptr, qd, h, ac.data(), as.data(), oc.data(), os.data(), 1);
    for (int i = 0; i < h; ++i) {
      hc[i] = oc[i] + hc[i];
      hs[i] = os[i] + hs[i];
    }
    orc_rmsnorm_reshare(hc.data(), hs.data(), w.g2, m->eps, variant, mk ? mk + 2 * h : nullptr,
                        nc.data(), ns.data(), h);
    orc_linear_bf16(w.wg, nullptr, h, I, nc.data(), ns.data(), gc.data(), gs.data(), 1);
    orc_linear_bf16(w.wu, nullptr, h, I, nc.data(), ns.data(), uc.data(), us.data(), 1);
    orc_swiglu_reshare(gc.data(), gs.data(), uc.data(), us.data(), variant,
                       mk ? mk + 3 * h : nullptr, xc.data(), xs.data(), I);
    orc_linear_bf16(w.wd, nullptr, I, h, xc.data(), xs.data(), dc.data(), ds.data(), 1);
    for (int i = 0; i < h; ++i) {
      hc[i] = dc[i] + hc[i];
      hs[i] = ds[i] + hs[i];
    }
  }
  m->len = pos + 1;
  if (hc_out) std::memcpy(hc_out, hc.data(), h * 4);
  if (hs_out) std::memcpy(hs_out, hs.data(), h * 4);
  if (Lrun == m->L && logits_c && m->lm_head) {
    const float* mk = masks ? masks + (size_t)(m->L - 1) * mask_stride : nullptr;
    orc_rmsnorm_reshare(hc.data(), hs.data(), m->final_norm, m->eps, variant, mk, nc.data(), ns.data(), h);
    orc_linear_bf16(m->lm_head, nullptr, h, m->V, nc.data(), ns.data(), logits_c, logits_s, 1);
  }
  return 0;
}

