"""ctypes binding of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, by __graft_entry__.smoke() as the checker and by
bench.py's CPU-baseline leg; the product library never uses it.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F32 = C.c_float
F64 = C.c_double

NL_APPROX, NL_GPU, NL_MPC = 0, 1, 2

_SIGS = {
    "orc_set_threads": (None, [I32]),
    "orc_max_threads": (I32, []),
    "orc_linear_f32": (None, [P, P, I32, I32, P, P, P, P, I32]),
    "orc_linear_bf16": (None, [P, P, I32, I32, P, P, P, P, I32]),
    "orc_linear_abs_bf16": (None, [P, I32, I32, P, P]),
    "orc_linear_ring": (None, [P, P, I32, I32, P, P, P, P, I32, I32]),
    "orc_plaintext_linear_ring": (None, [P, P, I32, I32, P, P, I32]),
    "orc_fixed_from_f64": (I32, [F64, I32, P]),
    "orc_fixed_mul": (I32, [I32, I32, I32, P]),
    "orc_beaver_f32": (None, [P] * 14 + [I64]),
    "orc_beaver_ring": (None, [P] * 14 + [I64, I32]),
    "orc_philox_words": (None, [U64, U64, U64, P, I64]),
    "orc_fill_uniform": (None, [U64, U64, F32, F32, P, I64]),
    "orc_fill_normal_bf16": (None, [U64, U64, F32, P, I64]),
    "orc_chacha20_words": (None, [P, U64, P, I64]),
    "orc_seed_from_u64": (None, [U64, P]),
    "orc_ring_share_seeded": (None, [P, I64, U64, P, P]),
    "orc_embed_shares_chacha": (None, [P, I32, P, I32, P, P, P]),
    "orc_triples_f32": (None, [U64, U64, I64] + [P] * 9),
    "orc_triples_ring": (None, [U64, U64, I64] + [P] * 6),
    "orc_embed_shares": (None, [P, I32, I32, U64, U64, P, P]),
    "orc_rope_table": (None, [I32, I32, F32, P, P]),
    "orc_rope_apply": (None, [P, I32, I32, P, P, P]),
    "orc_rmsnorm_reshare": (None, [P, P, P, F32, I32, P, P, P, I32]),
    "orc_swiglu_reshare": (None, [P, P, P, P, I32, P, P, P, I32]),
    "orc_silu_reshare": (None, [P, P, I32, P, P, P, I32]),
    "orc_softmax_approx": (None, [P, P, I32, P]),
    "orc_attention": (None, [P, P, P, I32, I32, I32, I32, I32, P, P, P]),
    "orc_argmax_last": (I32, [P, P, I32]),
    "orc_model_create": (P, [I32, I32, I32, I32, I32, I32, I32, F32, F32, I32]),
    "orc_model_destroy": (None, [P]),
    "orc_model_set_layer": (None, [P, I32] + [P] * 12),
    "orc_model_set_head": (None, [P, P, P]),
    "orc_model_reset": (None, [P]),
    "orc_ot_table": (None, [I32, F32, F32, I32, P]),
    "orc_ot_input_to_index": (C.c_uint32, [F32, F32, F32, I32]),
    "orc_model_get_kv": (I32, [P, I32, I32, P, P]),
    "orc_model_set_len": (None, [P, I32]),
    "orc_model_forward": (I32, [P, P, P, I32, I32, P, I64, I32, P, P, P, P]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        srcs = list(HERE.glob("*.cpp"))
        if not LIB.exists() or max(s.stat().st_mtime for s in srcs) > LIB.stat().st_mtime:
            subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
        _lib = C.CDLL(str(LIB))
        for n, (res, args) in _SIGS.items():
            f = getattr(_lib, n)
            f.restype = res
            f.argtypes = args
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    return np.ascontiguousarray(np.asarray(a, dtype=dt))


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return int(lib().orc_max_threads())


def normal_bf16(shape, seed: int, stream: int, std: float = 0.02) -> np.ndarray:
    """N(0, std) values rounded to bf16 (uint16 bit patterns), generated on the oracle's threads."""
    out = np.empty(shape, np.uint16)
    lib().orc_fill_normal_bf16(seed, stream, std, _p(out), out.size)
    return out


def linear_f32(w_in_out, bias, xc, xs):
    """SecureLinear::forward_secure on [M][in] shares; w [in][out] f32."""
    w = _c(w_in_out, np.float32)
    xc, xs = np.atleast_2d(_c(xc, np.float32)), np.atleast_2d(_c(xs, np.float32))
    M, K = xc.shape
    N = w.size // K
    yc, ys = np.empty((M, N), np.float32), np.empty((M, N), np.float32)
    lib().orc_linear_f32(_p(w), _p(None if bias is None else _c(bias, np.float32)), K, N, _p(xc), _p(xs), _p(yc), _p(ys), M)
    return yc, ys


def linear_bf16(w_in_out_u16, bias, xc, xs):
    w = _c(w_in_out_u16, np.uint16)
    xc, xs = np.atleast_2d(_c(xc, np.float32)), np.atleast_2d(_c(xs, np.float32))
    M, K = xc.shape
    N = w.size // K
    yc, ys = np.empty((M, N), np.float32), np.empty((M, N), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().orc_linear_bf16(_p(w), _p(b), K, N, _p(xc), _p(xs), _p(yc), _p(ys), M)
    return yc, ys


def linear_abs_bf16(w_in_out_u16, x):
    w = _c(w_in_out_u16, np.uint16)
    x = _c(x, np.float32).reshape(-1)
    K = x.size
    N = w.size // K
    y = np.empty(N, np.float64)
    lib().orc_linear_abs_bf16(_p(w), K, N, _p(x), _p(y))
    return y


def linear_ring(w_in_out, bias, xc, xs, scale=16):
    w = _c(w_in_out, np.int32)
    xc, xs = np.atleast_2d(_c(xc, np.int32)), np.atleast_2d(_c(xs, np.int32))
    M, K = xc.shape
    N = w.size // K
    yc, ys = np.empty((M, N), np.int32), np.empty((M, N), np.int32)
    b = None if bias is None else _c(bias, np.int32)
    lib().orc_linear_ring(_p(w), _p(b), K, N, _p(xc), _p(xs), _p(yc), _p(ys), M, scale)
    return yc, ys


def plaintext_linear_ring(w_in_out, bias, x, scale=16):
    w = _c(w_in_out, np.int32)
    x = _c(x, np.int32).reshape(-1)
    N = w.size // x.size
    y = np.empty(N, np.int32)
    lib().orc_plaintext_linear_ring(_p(w), _p(None if bias is None else _c(bias, np.int32)), x.size, N, _p(x), _p(y), scale)
    return y


class FixedPointError(ValueError):
    pass


def fixed_from_f64(v: float, scale: int = 16) -> int:
    out = np.zeros(1, np.int32)
    rc = lib().orc_fixed_from_f64(float(v), scale, _p(out))
    if rc == 1:
        raise FixedPointError(f"Overflow {{ value: {v} }}")
    if rc == 2:
        raise FixedPointError(f"Underflow {{ value: {v} }}")
    if rc == 3:
        raise FixedPointError(f"InvalidScale({scale})")
    return int(out[0])


def fixed_mul(a: int, b: int, scale: int = 16) -> int:
    out = np.zeros(1, np.int32)
    if lib().orc_fixed_mul(int(a), int(b), scale, _p(out)) != 0:
        raise FixedPointError("Overflow")
    return int(out[0])


def beaver_f32(xc, xs, yc, ys, ac, as_, bc, bs, cc, cs):
    arrs = [_c(a, np.float32) for a in (xc, xs, yc, ys, ac, as_, bc, bs, cc, cs)]
    n = arrs[0].size
    d, e, zc, zs = (np.empty(n, np.float32) for _ in range(4))
    lib().orc_beaver_f32(*[_p(a) for a in arrs], _p(d), _p(e), _p(zc), _p(zs), n)
    return zc, zs, d, e


def beaver_ring(xc, xs, yc, ys, ac, as_, bc, bs, cc, cs, trunc_shift=0):
    arrs = [_c(a, np.uint32) for a in (xc, xs, yc, ys, ac, as_, bc, bs, cc, cs)]
    n = arrs[0].size
    d, e, zc, zs = (np.empty(n, np.uint32) for _ in range(4))
    lib().orc_beaver_ring(*[_p(a) for a in arrs], _p(d), _p(e), _p(zc), _p(zs), n, trunc_shift)
    return zc, zs, d, e


def philox_words(seed, stream, offset, n):
    out = np.empty(n, np.uint32)
    lib().orc_philox_words(seed, stream, offset, _p(out), n)
    return out


def fill_uniform(seed, offset, lo, hi, n):
    out = np.empty(n, np.float32)
    lib().orc_fill_uniform(seed, offset, lo, hi, _p(out), n)
    return out


def triples_f32(seed, offset, n):
    out = [np.empty(n, np.float32) for _ in range(9)]
    lib().orc_triples_f32(seed, offset, n, *[_p(a) for a in out])
    return out  # a, b, c, a_c, a_s, b_c, b_s, c_c, c_s


def triples_ring(seed, offset, n):
    out = [np.empty(n, np.uint32) for _ in range(6)]
    lib().orc_triples_ring(seed, offset, n, *[_p(a) for a in out])
    return out  # a_c, a_s, b_c, b_s, c_c, c_s


def embed_shares(table_u16, hidden, token, seed, counter):
    t = _c(table_u16, np.uint16)
    hc, hs = np.empty(hidden, np.float32), np.empty(hidden, np.float32)
    lib().orc_embed_shares(_p(t), hidden, int(token), seed, counter, _p(hc), _p(hs))
    return hc, hs


def rope_table(head_dim, max_seq, theta):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty((max_seq, head_dim // 2), np.float32)
    lib().orc_rope_table(head_dim, max_seq, theta, _p(c), _p(s))
    return c, s


def rope_apply(share, n_heads, head_dim, cos_row, sin_row):
    x = _c(share, np.float32)
    out = np.empty_like(x)
    lib().orc_rope_apply(_p(x), n_heads, head_dim, _p(_c(cos_row, np.float32)), _p(_c(sin_row, np.float32)), _p(out))
    return out


def rmsnorm_reshare(xc, xs, gamma, eps, variant, mask=None):
    xc, xs, g = _c(xc, np.float32), _c(xs, np.float32), _c(gamma, np.float32)
    n = xc.size
    yc, ys = np.empty(n, np.float32), np.empty(n, np.float32)
    lib().orc_rmsnorm_reshare(_p(xc), _p(xs), _p(g), eps, variant, _p(None if mask is None else _c(mask, np.float32)), _p(yc), _p(ys), n)
    return yc, ys


def swiglu_reshare(gc, gs, uc, us, variant, mask=None):
    a = [_c(v, np.float32) for v in (gc, gs, uc, us)]
    n = a[0].size
    yc, ys = np.empty(n, np.float32), np.empty(n, np.float32)
    lib().orc_swiglu_reshare(*[_p(v) for v in a], variant, _p(None if mask is None else _c(mask, np.float32)), _p(yc), _p(ys), n)
    return yc, ys


def silu_reshare(xc, xs, variant, mask=None):
    xc, xs = _c(xc, np.float32), _c(xs, np.float32)
    n = xc.size
    yc, ys = np.empty(n, np.float32), np.empty(n, np.float32)
    lib().orc_silu_reshare(_p(xc), _p(xs), variant, _p(None if mask is None else _c(mask, np.float32)), _p(yc), _p(ys), n)
    return yc, ys


def softmax_approx(sc, ss):
    sc, ss = _c(sc, np.float32), _c(ss, np.float32)
    w = np.empty(sc.size, np.float32)
    lib().orc_softmax_approx(_p(sc), _p(ss), sc.size, _p(w))
    return w


def attention(q, kcache, vcache, H, Hkv, d, variant, mask=None):
    q, k, v = _c(q, np.float32), _c(kcache, np.float32), _c(vcache, np.float32)
    kv_len = k.size // (Hkv * d)
    oc, os_ = np.empty(H * d, np.float32), np.empty(H * d, np.float32)
    lib().orc_attention(_p(q), _p(k), _p(v), kv_len, H, Hkv, d, variant, _p(None if mask is None else _c(mask, np.float32)), _p(oc), _p(os_))
    return oc, os_


def argmax_last(lc, ls):
    lc, ls = _c(lc, np.float32), _c(ls, np.float32)
    return int(lib().orc_argmax_last(_p(lc), _p(ls), lc.size))


class Model:
    """CPU layer loop of the reference (oracle_model.cpp); weights bf16 in [in][out] layout."""

    def __init__(self, h, L, H, Hkv, d, I, V, theta=1e6, eps=1e-6, max_seq=2048):
        self.h, self.L, self.H, self.Hkv, self.d, self.I, self.V = h, L, H, Hkv, d, I, V
        self._keep = []
        self.ptr = lib().orc_model_create(h, L, H, Hkv, d, I, V, theta, eps, max_seq)

    def set_layer(self, l, wq, wk, wv, wo, wg, wu, wd, bq, bk, bv, g1, g2):
        arrs = [_c(a, np.uint16) for a in (wq, wk, wv, wo, wg, wu, wd)]
        arrs += [None if a is None else _c(a, np.float32) for a in (bq, bk, bv)]
        arrs += [_c(g1, np.float32), _c(g2, np.float32)]
        self._keep.append(arrs)
        lib().orc_model_set_layer(self.ptr, l, *[_p(a) for a in arrs])

    def set_head(self, lm_head_in_out, final_norm):
        a = [_c(lm_head_in_out, np.uint16), _c(final_norm, np.float32)]
        self._keep.append(a)
        lib().orc_model_set_head(self.ptr, _p(a[0]), _p(a[1]))

    def reset(self):
        lib().orc_model_reset(self.ptr)

    def get_kv(self, pos0: int, n: int):
        """Cached reconstructed K and V rows [L][n][Hkv*d] of positions [pos0, pos0 + n)."""
        k = np.empty((self.L, n, self.Hkv * self.d), np.float32)
        v = np.empty_like(k)
        if lib().orc_model_get_kv(self.ptr, pos0, n, _p(k), _p(v)) != 0:
            raise RuntimeError("oracle model: positions beyond the cache")
        return k, v

    def set_len(self, n: int):
        lib().orc_model_set_len(self.ptr, int(n))

    def forward(self, hc, hs, variant=NL_APPROX, attn_variant=NL_APPROX, masks=None, n_layers=0):
        hc, hs = _c(hc, np.float32), _c(hs, np.float32)
        mk = None if masks is None else _c(masks, np.float32)
        stride = 0 if mk is None else mk.size // self.L
        oc, os_ = np.empty(self.h, np.float32), np.empty(self.h, np.float32)
        want_logits = n_layers in (0, self.L)
        lc = np.empty(self.V, np.float32) if want_logits else None
        ls = np.empty(self.V, np.float32) if want_logits else None
        rc = lib().orc_model_forward(self.ptr, _p(hc), _p(hs), variant, attn_variant, _p(mk), stride,
                                     n_layers, _p(oc), _p(os_), _p(lc), _p(ls))
        if rc != 0:
            raise RuntimeError("oracle model: position beyond max_seq")
        return oc, os_, lc, ls

    def __del__(self):
        try:
            lib().orc_model_destroy(self.ptr)
        except Exception:
            pass


def chacha20_words(seed32: bytes, offset: int, n: int) -> np.ndarray:
    """ChaCha20Rng::from_seed(seed32) next_u32 words [offset, offset + n)."""
    k = np.frombuffer(bytes(seed32), np.uint8).copy()
    assert k.size == 32
    out = np.empty(n, np.uint32)
    lib().orc_chacha20_words(_p(k), offset, _p(out), n)
    return out


def seed_from_u64(seed: int) -> bytes:
    """rand_core 0.6 SeedableRng::seed_from_u64 expansion (PCG32) to a 32-byte seed."""
    out = np.empty(32, np.uint8)
    lib().orc_seed_from_u64(seed, _p(out))
    return out.tobytes()


def ring_share_seeded(x_i32, seed: int):
    """SharePair::from_plaintext_seeded: (client, server) i32 shares."""
    x = _c(x_i32, np.int32).reshape(-1)
    xc, xs = np.empty_like(x), np.empty_like(x)
    lib().orc_ring_share_seeded(_p(x), x.size, seed, _p(xc), _p(xs))
    return xc, xs


def embed_shares_chacha(table_u16, hidden, tokens, seed32: bytes):
    """get_embeddings_direct: [n][hidden] client and server shares of one request."""
    t = _c(table_u16, np.uint16)
    tok = _c(tokens, np.int32).reshape(-1)
    k = np.frombuffer(bytes(seed32), np.uint8).copy()
    hc = np.empty((tok.size, hidden), np.float32)
    hs = np.empty((tok.size, hidden), np.float32)
    lib().orc_embed_shares_chacha(_p(t), hidden, _p(tok), tok.size, _p(k), _p(hc), _p(hs))
    return hc, hs


OT_TABLE_RANGES = ((-8.0, 8.0), (-10.0, 0.0), (0.01, 10.0), (0.01, 100.0))  # silu, exp, rsqrt, reciprocal


def ot_standard_tables(size: int = 4096) -> np.ndarray:
    """StandardOtTables::new(size) values, [4][size] f32 (silu, exp, rsqrt, reciprocal)."""
    out = np.empty((4, size), np.float32)
    for k, (lo, hi) in enumerate(OT_TABLE_RANGES):
        lib().orc_ot_table(k, lo, hi, size, _p(out[k]))
    return out


def ot_input_to_index(x: float, kind: int, size: int = 4096) -> int:
    lo, hi = OT_TABLE_RANGES[kind]
    return int(lib().orc_ot_input_to_index(float(x), lo, hi, size))


# IknpOtExtension's commitment-based query protocol (crates/ot/src/iknp.rs:414-620), restated in
# Python over hashlib's SHA-256 and the `cryptography` package's AES-128: the client's
# generate_query / decode_response and the server's process_query, for checking the device's
# process_query on small batches.
def _ot_prf(key: bytes, ctr: int, n: int) -> bytes:
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms, modes

    enc = Cipher(algorithms.AES(key), modes.ECB()).encryptor()
    blocks = b"".join(ctr.to_bytes(8, "little") + i.to_bytes(8, "little") for i in range((n + 15) // 16))
    return (enc.update(blocks) + enc.finalize())[:n]


def _ot_item_key(commitment: bytes, batch_seed: bytes, j: int, ctr: int) -> bytes:
    import hashlib

    h = hashlib.sha256(b"IKNP-Item-Key-v2" + commitment + batch_seed + j.to_bytes(4, "little") + ctr.to_bytes(8, "little"))
    return h.digest()[:16]


def ot_generate_query(commitment: bytes, ctr: int, indices, batch_seed: bytes, row_keys):
    """The client's query for `indices` with the given batch seed and per-item row keys."""
    q = len(indices).to_bytes(2, "little") + batch_seed
    for j, idx in enumerate(indices):
        k = _ot_item_key(commitment, batch_seed, j, ctr)
        idx_enc = int(idx) ^ int.from_bytes(_ot_prf(k, 0, 4), "little")
        rk = bytes(a ^ b for a, b in zip(row_keys[j], _ot_prf(k, 1, 16)))
        q += idx_enc.to_bytes(4, "little") + rk
    return q


def ot_process_query(commitment: bytes, ctr: int, query: bytes, table: bytes, row_bytes: int) -> bytes:
    m = int.from_bytes(query[:2], "little")
    seed = query[2:34]
    assert len(query) == 34 + 20 * m
    rows = len(table) // row_bytes
    out = b""
    for j in range(m):
        e = query[34 + 20 * j: 54 + 20 * j]
        k = _ot_item_key(commitment, seed, j, ctr)
        idx = int.from_bytes(e[:4], "little") ^ int.from_bytes(_ot_prf(k, 0, 4), "little")
        if idx >= rows:
            raise ValueError(f"InvalidIndex {{ index: {idx}, max: {rows} }}")
        rk = bytes(a ^ b for a, b in zip(e[4:], _ot_prf(k, 1, 16)))
        mask = _ot_prf(rk, ctr * 1000 + j, row_bytes)
        out += bytes(a ^ b for a, b in zip(table[idx * row_bytes:(idx + 1) * row_bytes], mask))
    return out


def ot_decode_response(response: bytes, ctr: int, row_keys, row_bytes: int) -> bytes:
    out = b""
    for j, rk in enumerate(row_keys):
        mask = _ot_prf(rk, ctr * 1000 + j, row_bytes)
        out += bytes(a ^ b for a, b in zip(response[j * row_bytes:(j + 1) * row_bytes], mask))
    return out
