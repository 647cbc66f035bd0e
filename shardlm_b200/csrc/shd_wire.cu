// The reference's binary wire format for the prefill and decode routes, decoded and encoded on the
// host, with the model running in between (crates/v2/server/src/routes/binary_protocol.rs:21-81,
// batched_prefill_gpu_v3_binary in secure_inference.rs:2635-2700).
//
// The reference serialises these structs with bincode 1.3.3's default options: fields in
// declaration order, integers little-endian at their full width, a [u8; 16] as its 16 bytes, and a
// Vec<f32> as its length (u64, little-endian) followed by the raw little-endian f32 values.
//   BinaryPrefillRequest  { session_id [u8;16], seq_len u32, hidden_dim u32,
//                           hidden_client Vec<f32> [seq_len*hidden], hidden_server Vec<f32> }
//   BinaryPrefillResponse { final_hidden_client Vec<f32> [hidden], final_hidden_server Vec<f32>,
//                           num_layers u32, kv_dim u32,
//                           k_cache Vec<f32> [num_layers*seq_len*kv_dim], v_cache Vec<f32>,
//                           logits_client Vec<f32> [vocab], logits_server Vec<f32> }
//   BinaryDecodeRequest   { session_id [u8;16], position u32, hidden_client Vec<f32> [hidden],
//                           hidden_server Vec<f32> }
//   BinaryDecodeResponse  { hidden_client Vec<f32>, hidden_server Vec<f32>, logits_client Vec<f32>,
//                           logits_server Vec<f32> }
// The KV cache stays on the device either way (decode reads it there); the prefill response
// carries it as the reference's does unless the caller asks to leave it out (include_kv = 0: empty
// k_cache and v_cache, num_layers and kv_dim still set), which removes the bulk of the response.
// The session id is not interpreted here: the caller maps sessions to model slots.
#include <cstring>
#include <string>
#include <vector>

#include "shd_common.cuh"
#include "shd_model.cuh"

extern "C" int shd_model_prefill_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host, int n,
                                        float* logits_c_host, float* logits_s_host, float* final_c_host,
                                        float* final_s_host, int32_t* next_token_host);
extern "C" int shd_model_read_kv(shd_model* m, int slot, int pos0, int n, float* k_host, float* v_host);
extern "C" int shd_model_forward_host_hidden(shd_model* m, int slot, const float* hc_host, const float* hs_host,
                                             float* logits_c_host, float* logits_s_host, float* hidden_c_host,
                                             float* hidden_s_host);

namespace {

struct Reader {
  const uint8_t* p;
  size_t n, at = 0;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (at + sizeof(T) > n) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + at, sizeof(T));  // little-endian host, as the wire
    at += sizeof(T);
    return v;
  }
  // a Vec<f32>: returns a pointer into the buffer (unaligned is fine for memcpy consumers)
  const uint8_t* vec_f32(uint64_t& count) {
    count = get<uint64_t>();
    if (!ok || count > (n - at) / 4) {
      ok = false;
      return nullptr;
    }
    const uint8_t* q = p + at;
    at += count * 4;
    return q;
  }
};

struct Writer {
  uint8_t* p;
  size_t at = 0;
  template <typename T>
  void put(T v) {
    std::memcpy(p + at, &v, sizeof(T));
    at += sizeof(T);
  }
  void vec_f32(const float* v, uint64_t count) {
    put<uint64_t>(count);
    if (count) std::memcpy(p + at, v, count * 4);
    at += count * 4;
  }
};

int wire_fail(shd_model* m, const std::string& msg) { return shd_fail(m->ctx, SHD_ERR_ARG, msg); }

}  // namespace

extern "C" int shd_bincode_prefill(shd_model* m, int slot, const uint8_t* req, size_t req_len, int include_kv,
                                   uint8_t* resp, size_t resp_cap, size_t* resp_len) {
  if (!m) return SHD_ERR_ARG;
  SHD_REQUIRE(m->ctx, req && resp_len, "shd_bincode_prefill: null pointer");
  SHD_REQUIRE(m->ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_bincode_prefill: slot out of range");
  SHD_REQUIRE(m->ctx, m->ctx->tp_world <= 1, "shd_bincode_prefill: tensor-parallel models are not supported");
  Reader r{req, req_len};
  for (int i = 0; i < 16; ++i) (void)r.get<uint8_t>();  // session id: the caller's slot stands for it
  const uint32_t seq_len = r.get<uint32_t>(), hidden_dim = r.get<uint32_t>();
  uint64_t nc = 0, ns = 0;
  const uint8_t* hc = r.vec_f32(nc);
  const uint8_t* hs = r.ok ? r.vec_f32(ns) : nullptr;
  if (!r.ok || r.at != req_len) return wire_fail(m, "Invalid binary request: truncated or trailing bytes");
  const int h = m->cfg.hidden;
  if ((int)hidden_dim != h)
    return wire_fail(m, "Invalid binary request: hidden_dim " + std::to_string(hidden_dim) + " != " + std::to_string(h));
  if (seq_len == 0) return wire_fail(m, "Invalid binary request: empty prompt");
  if (nc != (uint64_t)seq_len * h || ns != nc)
    return wire_fail(m, "Invalid binary request: hidden states are not seq_len x hidden_dim");
  const int L = m->cfg.n_layers, kvd = m->kvd, V = m->cfg.vocab;
  const uint64_t kv_count = include_kv ? (uint64_t)L * seq_len * kvd : 0;
  const size_t need = 4 * 8 + 2 * (size_t)h * 4 + 8 + 2 * (8 + kv_count * 4) + 2 * (size_t)V * 4;
  *resp_len = need;
  if (!resp || resp_cap < need)
    return wire_fail(m, "shd_bincode_prefill: response needs " + std::to_string(need) + " bytes");
  const int pos0 = m->len[slot];
  std::vector<float> hcv((size_t)nc), hsv((size_t)ns), fc(h), fs(h), lc(V), ls(V);
  std::memcpy(hcv.data(), hc, nc * 4);
  std::memcpy(hsv.data(), hs, ns * 4);
  int rc = shd_model_prefill_hidden(m, slot, hcv.data(), hsv.data(), (int)seq_len, lc.data(), ls.data(), fc.data(),
                                    fs.data(), nullptr);
  if (rc) return rc;
  std::vector<float> k, v;
  if (include_kv) {
    k.resize(kv_count);
    v.resize(kv_count);
    if ((rc = shd_model_read_kv(m, slot, pos0, (int)seq_len, k.data(), v.data()))) return rc;
  }
  Writer w{resp};
  w.vec_f32(fc.data(), h);
  w.vec_f32(fs.data(), h);
  w.put<uint32_t>((uint32_t)L);
  w.put<uint32_t>((uint32_t)kvd);
  w.vec_f32(k.data(), kv_count);
  w.vec_f32(v.data(), kv_count);
  w.vec_f32(lc.data(), V);
  w.vec_f32(ls.data(), V);
  *resp_len = w.at;
  return SHD_OK;
}

extern "C" int shd_bincode_decode(shd_model* m, int slot, const uint8_t* req, size_t req_len, uint8_t* resp,
                                  size_t resp_cap, size_t* resp_len) {
  if (!m) return SHD_ERR_ARG;
  SHD_REQUIRE(m->ctx, req && resp_len, "shd_bincode_decode: null pointer");
  SHD_REQUIRE(m->ctx, slot >= 0 && slot < m->cfg.max_batch, "shd_bincode_decode: slot out of range");
  Reader r{req, req_len};
  for (int i = 0; i < 16; ++i) (void)r.get<uint8_t>();
  const uint32_t position = r.get<uint32_t>();
  uint64_t nc = 0, ns = 0;
  const uint8_t* hc = r.vec_f32(nc);
  const uint8_t* hs = r.ok ? r.vec_f32(ns) : nullptr;
  if (!r.ok || r.at != req_len) return wire_fail(m, "Invalid binary request: truncated or trailing bytes");
  const int h = m->cfg.hidden, V = m->cfg.vocab;
  if (nc != (uint64_t)h || ns != nc) return wire_fail(m, "Invalid binary request: hidden states are not hidden_dim");
  if ((int)position != m->len[slot])
    return wire_fail(m, "Invalid binary request: position " + std::to_string(position) + " but the sequence holds " +
                            std::to_string(m->len[slot]));
  const size_t need = 4 * 8 + 2 * (size_t)h * 4 + 2 * (size_t)V * 4;
  *resp_len = need;
  if (!resp || resp_cap < need)
    return wire_fail(m, "shd_bincode_decode: response needs " + std::to_string(need) + " bytes");
  std::vector<float> hcv(h), hsv(h), oc(h), os(h), lc(V), ls(V);
  std::memcpy(hcv.data(), hc, (size_t)h * 4);
  std::memcpy(hsv.data(), hs, (size_t)h * 4);
  const int rc =
      shd_model_forward_host_hidden(m, slot, hcv.data(), hsv.data(), lc.data(), ls.data(), oc.data(), os.data());
  if (rc) return rc;
  Writer w{resp};
  w.vec_f32(oc.data(), h);
  w.vec_f32(os.data(), h);
  w.vec_f32(lc.data(), V);
  w.vec_f32(ls.data(), V);
  *resp_len = w.at;
  return SHD_OK;
}
