"""Whole-model secret-shared forward pass on libshardlm_cuda (replaces the axum layer loops
batched_prefill_gpu_v3 / batched_full_forward_gpu / generate_token_gpu,
crates/v2/server/src/routes/secure_inference.rs:1553-1796 and :2299-2632).

Weights are random-init (no checkpoints here): N(0, 0.02) bf16 matrices and q/k/v biases, unit
RMSNorm gammas, in the Qwen2.5 architecture shapes the benchmarks name.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import ModelConfigC, NL_APPROX, NL_GPU, ShardInfoC, check, lib
from .runtime import Context, ptr


@dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    qkv_bias: bool = True
    tied: bool = False

    def linear_params(self) -> int:
        """Weight parameters streamed per decoded token (every linear layer + lm_head)."""
        h, d = self.hidden, self.head_dim
        per_layer = h * (self.n_heads * d) + 2 * h * (self.n_kv_heads * d) + (self.n_heads * d) * h + 3 * h * self.intermediate
        return per_layer * self.n_layers + self.vocab * h

    def replace(self, **kw) -> "ModelShape":
        d = dict(self.__dict__)
        d.update(kw)
        return ModelShape(**d)


# Qwen2.5 architectures of the benchmark configs (3, 5).
QWEN2_5_1_5B = ModelShape("qwen2.5-1.5b", 1536, 28, 12, 2, 128, 8960, 151936, tied=True)
QWEN2_5_7B = ModelShape("qwen2.5-7b", 3584, 28, 28, 4, 128, 18944, 152064)
QWEN2_5_14B = ModelShape("qwen2.5-14b", 5120, 48, 40, 8, 128, 13824, 152064)
TINY = ModelShape("tiny", 256, 2, 4, 2, 64, 512, 1000)
SHAPES = {s.name: s for s in (QWEN2_5_1_5B, QWEN2_5_7B, QWEN2_5_14B, TINY)}


def _gen(seed: int, *key: int) -> torch.Generator:
    g = torch.Generator(device="cuda")
    s = seed
    for k in key:
        s = (s * 1000003 + k) & 0x7FFFFFFFFFFFFFFF
    g.manual_seed(s)
    return g


def random_bf16(shape, seed: int, *key: int, std: float = 0.02) -> torch.Tensor:
    t = torch.randn(*shape, device="cuda", dtype=torch.float32, generator=_gen(seed, *key))
    return t.mul_(std).to(torch.bfloat16)


class SecureModel:
    """One rank's secret-shared model (the full model when tp_world == 1)."""

    def __init__(self, ctx: Context, shape: ModelShape, max_seq: int = 2048, max_batch: int = 1,
                 variant_decode: int = NL_APPROX, variant_prefill: int = NL_GPU,
                 variant_attn: int = NL_APPROX, share_seed: int = 0x5EED, tp_rank: int = 0,
                 tp_world: int = 1):
        self.ctx = ctx
        self.shape = shape
        self.max_seq = max_seq
        self.max_batch = max_batch
        self.share_seed = share_seed
        cfg = ModelConfigC(shape.hidden, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.head_dim,
                           shape.intermediate, shape.vocab, shape.rope_theta, shape.rms_eps, max_seq,
                           max_batch, variant_decode, variant_prefill, variant_attn, share_seed, tp_rank,
                           tp_world)
        h = C.c_void_p()
        ctx.bind_stream()
        check(lib().shd_model_create(ctx.ptr, C.byref(cfg), C.byref(h)), ctx.ptr)
        self.handle = h
        info = ShardInfoC()
        check(lib().shd_model_shard_info(self.handle, C.byref(info)), ctx.ptr)
        self.shard = info
        self.tp_rank, self.tp_world = tp_rank, tp_world

    # ---------------------------------------------------------------------------------------
    def _slices(self):
        s, d = self.shard, self.shape.head_dim
        return (slice(s.q_head_begin * d, (s.q_head_begin + s.q_head_count) * d),
                slice(s.kv_head_begin * d, (s.kv_head_begin + s.kv_head_count) * d),
                slice(s.inter_begin, s.inter_begin + s.inter_count),
                slice(s.vocab_begin, s.vocab_begin + s.vocab_count))

    def layer_weights(self, seed: int, l: int) -> dict:
        """Full (unsharded) random-init weights of layer l, device bf16 [out][in]."""
        sh = self.shape
        h, d = sh.hidden, sh.head_dim
        qd, kvd, I = sh.n_heads * d, sh.n_kv_heads * d, sh.intermediate
        w = {
            "wq": random_bf16((qd, h), seed, l, 0), "wk": random_bf16((kvd, h), seed, l, 1),
            "wv": random_bf16((kvd, h), seed, l, 2), "wo": random_bf16((h, qd), seed, l, 3),
            "wg": random_bf16((I, h), seed, l, 4), "wu": random_bf16((I, h), seed, l, 5),
            "wd": random_bf16((h, I), seed, l, 6),
            "g1": torch.ones(h, device="cuda"), "g2": torch.ones(h, device="cuda"),
        }
        if sh.qkv_bias:
            w["bq"] = random_bf16((qd,), seed, l, 7).float()
            w["bk"] = random_bf16((kvd,), seed, l, 8).float()
            w["bv"] = random_bf16((kvd,), seed, l, 9).float()
        else:
            w["bq"] = w["bk"] = w["bv"] = None
        return w

    def set_layer(self, l: int, w: dict) -> None:
        qs, kvs, isl, _ = self._slices()
        c = lambda t: None if t is None else t.contiguous()
        args = [c(w["wq"][qs]), c(w["wk"][kvs]), c(w["wv"][kvs]), c(w["wo"][:, qs]), c(w["wg"][isl]),
                c(w["wu"][isl]), c(w["wd"][:, isl]),
                None if w["bq"] is None else c(w["bq"][qs]), None if w["bk"] is None else c(w["bk"][kvs]),
                None if w["bv"] is None else c(w["bv"][kvs]), c(w["g1"].float()), c(w["g2"].float())]
        self.ctx.bind_stream()
        check(lib().shd_model_set_layer(self.handle, l, *[ptr(a) for a in args]), self.ctx.ptr)

    def head_weights(self, seed: int) -> dict:
        sh = self.shape
        emb = random_bf16((sh.vocab, sh.hidden), seed, 10_000, 0)
        lm = emb if sh.tied else random_bf16((sh.vocab, sh.hidden), seed, 10_000, 1)
        return {"embed": emb, "lm_head": lm, "final_norm": torch.ones(sh.hidden, device="cuda")}

    def set_head(self, w: dict) -> None:
        _, _, _, vs = self._slices()
        self.ctx.bind_stream()
        check(lib().shd_model_set_embedding(self.handle, ptr(w["embed"].contiguous())), self.ctx.ptr)
        check(lib().shd_model_set_head(self.handle, ptr(w["lm_head"][vs].contiguous()),
                                       ptr(w["final_norm"].float().contiguous())), self.ctx.ptr)

    def load_random_weights(self, seed: int = 0, host_copy: bool = False):
        """Random-init every layer (generated on the device, deterministic in `seed`).

        With host_copy, returns the weights as host numpy in the reference's [in][out] layout for the
        CPU oracle (small models only)."""
        host = {"layers": []} if host_copy else None
        for l in range(self.shape.n_layers):
            w = self.layer_weights(seed, l)
            self.set_layer(l, w)
            if host_copy:
                t = lambda x: None if x is None else x.t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
                f = lambda x: None if x is None else x.float().cpu().numpy()
                host["layers"].append({k: (t(v) if k.startswith("w") else f(v)) for k, v in w.items()})
            del w
        hw = self.head_weights(seed)
        self.set_head(hw)
        if host_copy:
            host["embed"] = hw["embed"].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
            host["lm_head_in_out"] = hw["lm_head"].t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
            host["final_norm"] = hw["final_norm"].cpu().numpy()
        torch.cuda.synchronize()
        return host

    # ---------------------------------------------------------------------------------------
    def set_masks(self, masks: torch.Tensor | None) -> None:
        if masks is None:
            check(lib().shd_model_set_masks(self.handle, None, 0), self.ctx.ptr)
            return
        m = masks.float().contiguous()
        check(lib().shd_model_set_masks(self.handle, ptr(m), m.shape[-1]), self.ctx.ptr)

    def reset(self) -> None:
        check(lib().shd_model_reset(self.handle), self.ctx.ptr)

    def prefill(self, tokens, slot: int = 0) -> int:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = C.c_int32()
        self.ctx.bind_stream()
        check(lib().shd_model_prefill(self.handle, slot, t.ctypes.data, t.size, C.byref(out)), self.ctx.ptr)
        return int(out.value)

    def decode_async(self, n_steps: int) -> None:
        self.ctx.bind_stream()
        check(lib().shd_model_decode_async(self.handle, n_steps), self.ctx.ptr)

    def read_tokens(self, count: int, n_active: int) -> np.ndarray:
        out = np.empty((count, n_active), np.int32)
        check(lib().shd_model_read_tokens(self.handle, count, out.ctypes.data), self.ctx.ptr)
        return out

    def decode(self, n_steps: int, n_active: int = 1) -> np.ndarray:
        self.decode_async(n_steps)
        return self.read_tokens(n_steps, n_active)

    def forward_host(self, hc: np.ndarray, hs: np.ndarray, slot: int = 0, out=None):
        """generate_token_gpu: hidden shares (host) in, logit shares (host) out."""
        hc = np.ascontiguousarray(hc, dtype=np.float32)
        hs = np.ascontiguousarray(hs, dtype=np.float32)
        if out is None:
            out = (np.empty(self.shape.vocab, np.float32), np.empty(self.shape.vocab, np.float32))
        self.ctx.bind_stream()
        check(lib().shd_model_forward_host(self.handle, slot, hc.ctypes.data, hs.ctypes.data,
                                           out[0].ctypes.data, out[1].ctypes.data), self.ctx.ptr)
        return out

    def forward_host_rows(self, slots, hc: np.ndarray, hs: np.ndarray, out=None):
        """forward_host for several sequences in one pass: hc/hs [M][hidden], row r at the next
        position of slots[r]; returns logit shares (lc, ls) as [M][vocab]."""
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.int32))
        M = sl.size
        hc = np.ascontiguousarray(hc, dtype=np.float32).reshape(M, self.shape.hidden)
        hs = np.ascontiguousarray(hs, dtype=np.float32).reshape(M, self.shape.hidden)
        if out is None:
            out = (np.empty((M, self.shape.vocab), np.float32), np.empty((M, self.shape.vocab), np.float32))
        self.ctx.bind_stream()
        check(lib().shd_model_forward_host_rows(self.handle, M, sl.ctypes.data, hc.ctypes.data, hs.ctypes.data,
                                                out[0].ctypes.data, out[1].ctypes.data), self.ctx.ptr)
        return out

    def forward_host_hidden(self, hc: np.ndarray, hs: np.ndarray, slot: int = 0):
        """forward_host that also returns the position's output hidden shares:
        (logits_c, logits_s, hidden_c, hidden_s)."""
        hc = np.ascontiguousarray(hc, dtype=np.float32)
        hs = np.ascontiguousarray(hs, dtype=np.float32)
        V, h = self.shape.vocab, self.shape.hidden
        lc, ls = np.empty(V, np.float32), np.empty(V, np.float32)
        oc, os_ = np.empty(h, np.float32), np.empty(h, np.float32)
        self.ctx.bind_stream()
        check(lib().shd_model_forward_host_hidden(self.handle, slot, hc.ctypes.data, hs.ctypes.data, lc.ctypes.data,
                                                  ls.ctypes.data, oc.ctypes.data, os_.ctypes.data), self.ctx.ptr)
        return lc, ls, oc, os_

    def prefill_hidden(self, hc: np.ndarray, hs: np.ndarray, slot: int = 0):
        """batched_prefill_gpu_v3: hidden-state shares [n][h] in; returns (next token, logits_c,
        logits_s, final_hidden_c, final_hidden_s) of the last position."""
        hc = np.ascontiguousarray(hc, dtype=np.float32).reshape(-1, self.shape.hidden)
        hs = np.ascontiguousarray(hs, dtype=np.float32).reshape(-1, self.shape.hidden)
        V, h = self.shape.vocab, self.shape.hidden
        lc, ls = np.empty(V, np.float32), np.empty(V, np.float32)
        fc, fs = np.empty(h, np.float32), np.empty(h, np.float32)
        tok = C.c_int32()
        self.ctx.bind_stream()
        check(lib().shd_model_prefill_hidden(self.handle, slot, hc.ctypes.data, hs.ctypes.data, hc.shape[0],
                                             lc.ctypes.data, ls.ctypes.data, fc.ctypes.data, fs.ctypes.data,
                                             C.byref(tok)), self.ctx.ptr)
        return int(tok.value), lc, ls, fc, fs

    def read_kv(self, pos0: int, n: int, slot: int = 0):
        """Reconstructed K and V rows [n_layers][n][kv_dim] of positions [pos0, pos0 + n)."""
        kvd = self.shard.kv_head_count * self.shape.head_dim
        k = np.empty((self.shape.n_layers, n, kvd), np.float32)
        v = np.empty_like(k)
        check(lib().shd_model_read_kv(self.handle, slot, pos0, n, k.ctypes.data, v.ctypes.data), self.ctx.ptr)
        return k, v

    def _bincode(self, fn: str, req: bytes, *extra) -> bytes:
        buf = np.frombuffer(bytes(req), np.uint8).copy()
        n = C.c_size_t(0)
        self.ctx.bind_stream()
        args = (self.handle,) + extra[:1] + (buf.ctypes.data, buf.size) + extra[1:]
        rc = getattr(lib(), fn)(*args, None, 0, C.byref(n))  # size query (no work is done)
        if rc != _lib.SHD_ERR_ARG or n.value == 0:
            check(rc, self.ctx.ptr)
        out = np.empty(n.value, np.uint8)
        check(getattr(lib(), fn)(*args, out.ctypes.data, out.size, C.byref(n)), self.ctx.ptr)
        return out[: n.value].tobytes()

    def prefill_binary(self, request: bytes, slot: int = 0, include_kv: bool = True) -> bytes:
        """POST /v3/secure/gpu/prefill: a bincode BinaryPrefillRequest in, BinaryPrefillResponse out."""
        return self._bincode("shd_bincode_prefill", request, slot, int(include_kv))

    def decode_binary(self, request: bytes, slot: int = 0) -> bytes:
        """A bincode BinaryDecodeRequest in, BinaryDecodeResponse out."""
        return self._bincode("shd_bincode_decode", request, slot)

    def seq_len(self, slot: int = 0) -> int:
        return int(lib().shd_model_seq_len(self.handle, slot))

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().shd_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def embed_share_counter(slot: int, pos: int) -> int:
    """Counter of the embedding-share generator for a token at `pos` of sequence slot `slot`."""
    return (slot << 32) + pos
