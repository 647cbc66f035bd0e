"""The reference's binary wire format (crates/v2/server/src/routes/binary_protocol.rs:21-81, bincode
1.3.3 default encoding) through shd_bincode_prefill / shd_bincode_decode, against an independent
Python encoder/decoder written here from the bincode rules (little-endian fixed-width integers,
a [u8; 16] as 16 raw bytes, Vec<f32> as a u64 length and the raw values, fields in declaration
order) and against the oracle's layer loop:

* prefill from the client's hidden-state shares (batched_prefill_gpu_v3_binary,
  secure_inference.rs:2635-2700): logits and final hidden state within the logit tolerance of
  test_model.py, the K/V cache rows against the oracle's cache, the response bytes identical to
  the Python encoding of the decoded values, and the KV-less variant;
* one decode position from hidden shares (BinaryDecodeRequest / BinaryDecodeResponse);
* malformed requests rejected as the route's InvalidRequest.
"""
import struct

import numpy as np
import pytest

from test_model import LOGIT_RTOL, _oracle_for

pytestmark = pytest.mark.gpu


def enc_vec(a) -> bytes:
    a = np.ascontiguousarray(a, dtype="<f4").reshape(-1)
    return struct.pack("<Q", a.size) + a.tobytes()


def prefill_request(session: bytes, hc, hs) -> bytes:
    hc, hs = np.asarray(hc, np.float32), np.asarray(hs, np.float32)
    return session + struct.pack("<II", hc.shape[0], hc.shape[1]) + enc_vec(hc) + enc_vec(hs)


def decode_request(session: bytes, position: int, hc, hs) -> bytes:
    return session + struct.pack("<I", position) + enc_vec(hc) + enc_vec(hs)


class _R:
    def __init__(self, b: bytes):
        self.b, self.at = b, 0

    def u32(self):
        v = struct.unpack_from("<I", self.b, self.at)[0]
        self.at += 4
        return v

    def vec(self):
        n = struct.unpack_from("<Q", self.b, self.at)[0]
        v = np.frombuffer(self.b, "<f4", n, self.at + 8).copy()
        self.at += 8 + 4 * n
        return v


def parse_prefill_response(b: bytes) -> dict:
    r = _R(b)
    out = {"final_hidden_client": r.vec(), "final_hidden_server": r.vec(), "num_layers": r.u32(),
           "kv_dim": r.u32(), "k_cache": r.vec(), "v_cache": r.vec(), "logits_client": r.vec(),
           "logits_server": r.vec()}
    assert r.at == len(b), "trailing bytes"
    return out


def encode_prefill_response(d: dict) -> bytes:
    return (enc_vec(d["final_hidden_client"]) + enc_vec(d["final_hidden_server"]) +
            struct.pack("<II", d["num_layers"], d["kv_dim"]) + enc_vec(d["k_cache"]) + enc_vec(d["v_cache"]) +
            enc_vec(d["logits_client"]) + enc_vec(d["logits_server"]))


def parse_decode_response(b: bytes) -> dict:
    r = _R(b)
    out = {"hidden_client": r.vec(), "hidden_server": r.vec(), "logits_client": r.vec(), "logits_server": r.vec()}
    assert r.at == len(b)
    return out


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))


@pytest.fixture(scope="module")
def small_model(ctx):
    from shardlm_b200.model import QWEN2_5_1_5B, SecureModel

    shape = QWEN2_5_1_5B.replace(n_layers=2, vocab=4096)
    m = SecureModel(ctx, shape, max_seq=64, max_batch=2, share_seed=3)
    host = m.load_random_weights(seed=8, host_copy=True)
    yield shape, m, host
    m.close()


def test_binary_prefill_and_decode_match_oracle(ctx, orc, small_model):
    shape, m, host = small_model
    m.reset()
    rng = np.random.default_rng(5)
    toks = rng.integers(0, shape.vocab, 19)  # the reference's benchmark prompt length
    hc, hs = orc.embed_shares_chacha(host["embed"], shape.hidden, toks, bytes(range(16)) + bytes(16))
    session = bytes(range(16))
    resp = m.prefill_binary(prefill_request(session, hc, hs), slot=0, include_kv=True)
    d = parse_prefill_response(resp)
    assert encode_prefill_response(d) == resp  # byte-for-byte the reference's encoding of these values
    assert d["num_layers"] == shape.n_layers and d["kv_dim"] == shape.n_kv_heads * shape.head_dim
    om = _oracle_for(orc, shape, host, 64)
    for p in range(len(toks)):
        oc, os_, lc, ls = om.forward(hc[p], hs[p], variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
    assert _rel(d["logits_client"] + d["logits_server"], lc + ls) < LOGIT_RTOL
    assert _rel(d["final_hidden_client"] + d["final_hidden_server"], oc + os_) < LOGIT_RTOL
    ok, ov = om.get_kv(0, len(toks))
    kv_d = d["kv_dim"]
    k = d["k_cache"].reshape(shape.n_layers, len(toks), kv_d)
    v = d["v_cache"].reshape(shape.n_layers, len(toks), kv_d)
    assert _rel(k, ok) < LOGIT_RTOL and _rel(v, ov) < LOGIT_RTOL
    gk, gv = m.read_kv(0, len(toks))
    assert np.array_equal(gk, k) and np.array_equal(gv, v)

    # one decode position from hidden shares
    nxt = 77
    dc, ds = orc.embed_shares_chacha(host["embed"], shape.hidden, [nxt], session + bytes(16))
    resp = m.decode_binary(decode_request(session, len(toks), dc[0], ds[0]), slot=0)
    dd = parse_decode_response(resp)
    oc, os_, lc, ls = om.forward(dc[0], ds[0], variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
    assert _rel(dd["logits_client"] + dd["logits_server"], lc + ls) < LOGIT_RTOL
    assert _rel(dd["hidden_client"] + dd["hidden_server"], oc + os_) < LOGIT_RTOL
    assert m.seq_len(0) == len(toks) + 1


def test_binary_prefill_without_kv(ctx, orc, small_model):
    shape, m, host = small_model
    m.reset()
    hc = np.random.default_rng(1).standard_normal((3, shape.hidden)).astype(np.float32)
    hs = np.zeros_like(hc)
    resp = m.prefill_binary(prefill_request(bytes(16), hc, hs), slot=1, include_kv=False)
    d = parse_prefill_response(resp)
    assert d["k_cache"].size == 0 and d["v_cache"].size == 0
    assert d["num_layers"] == shape.n_layers and d["logits_client"].size == shape.vocab
    # the cache stayed on the device: decode continues from it
    assert m.seq_len(1) == 3


def test_binary_requests_rejected(ctx, small_model):
    from shardlm_b200._lib import ShdError

    shape, m, _ = small_model
    m.reset()
    h = shape.hidden
    good = prefill_request(bytes(16), np.zeros((2, h), np.float32), np.zeros((2, h), np.float32))
    with pytest.raises(ShdError, match="Invalid binary request"):
        m.prefill_binary(good[:-1], slot=0)  # truncated
    with pytest.raises(ShdError, match="Invalid binary request"):
        m.prefill_binary(good + b"\0", slot=0)  # trailing byte
    wrong = prefill_request(bytes(16), np.zeros((2, h + 4), np.float32), np.zeros((2, h + 4), np.float32))
    with pytest.raises(ShdError, match="hidden_dim"):
        m.prefill_binary(wrong, slot=0)
    m.prefill_binary(good, slot=0)
    with pytest.raises(ShdError, match="position 5"):
        m.decode_binary(decode_request(bytes(16), 5, np.zeros(h, np.float32), np.zeros(h, np.float32)), slot=0)
