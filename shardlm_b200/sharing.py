"""Host-side mirror of the reference's share-wise layer API, on libshardlm_cuda.

Names, argument meaning and error behaviour follow the Rust crates this path replaces:
  * GpuSecureLinear      -- crates/v2/sharing/src/secure_linear.rs:148-405
  * LinearServer & co.   -- crates/sharing/src/linear.rs:186-274 (v1 Z_2^32 ring shares)
  * Fixed / FixedVector  -- crates/fixed_point/src/fixed.rs:30-49, vector.rs:22-29
  * SharePair / Share    -- crates/sharing/src/share.rs:44-135 (seeded server shares)
  * get_embeddings_direct -- crates/v2/server/src/routes/secure_inference.rs:387-460
  * secure_multiply_*    -- crates/v2/sharing/src/beaver.rs:167-233
  * BeaverTriple(Store)  -- crates/v2/sharing/src/beaver.rs:21-156
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import NL_APPROX
from .runtime import Context, Weight, ptr


class SharingError(ValueError):
    """ShapeMismatch / DimensionMismatch / ScaleMismatch of crates/*/sharing/src/error.rs."""


class ServerContext:
    """Marker that code runs on the server (crates/v2/sharing/src/secure.rs)."""


def _f32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.float32 or not t.is_cuda:
        raise SharingError("expected a float32 CUDA tensor")
    return t.contiguous()


class GpuSecureLinear:
    """Y_c = X_c W^T, Y_s = X_s W^T + b with W streamed once for both shares."""

    def __init__(self, ctx: Context, weight: Weight, bias: torch.Tensor | None):
        self.ctx = ctx
        self.weight = weight
        self.bias = bias
        self._in = weight.in_features
        self._out = weight.out_features

    @classmethod
    def from_cpu(cls, weight, bias, in_features: int, out_features: int, device: Context):
        """weight: host [in][out] row-major f32 (exact bf16 upcasts), as GpuSecureLinear::from_cpu."""
        w = Weight.from_f32_in_out(device, weight, in_features, out_features)
        b = None
        if bias is not None:
            b_np = np.asarray(bias, dtype=np.float32).reshape(-1)
            if b_np.size != out_features:
                raise SharingError(f"ShapeMismatch: bias expected [{out_features}], got [{b_np.size}]")
            b = device.to_device(b_np)
        return cls(device, w, b)

    def in_features(self) -> int:
        return self._in

    def out_features(self) -> int:
        return self._out

    def forward_secure_gpu_tensor(self, client_share: torch.Tensor, server_share: torch.Tensor,
                                  residual: tuple[torch.Tensor, torch.Tensor] | None = None):
        """Device tensors [M, in] (or [in]) -> (Y_c, Y_s) device tensors [M, out]."""
        xc, xs = _f32(client_share), _f32(server_share)
        if xc.numel() % self._in or xc.shape != xs.shape:
            raise SharingError(f"ShapeMismatch: expected [.., {self._in}], got {list(xc.shape)} / {list(xs.shape)}")
        M = xc.numel() // self._in
        out_shape = (M, self._out) if xc.dim() > 1 else (self._out,)
        yc = self.ctx.empty(*out_shape)
        ys = self.ctx.empty(*out_shape)
        rc_ = rs_ = None
        if residual is not None:
            rc_, rs_ = _f32(residual[0]), _f32(residual[1])
        self.ctx.call("shd_linear_dual_f32", self.weight.handle, ptr(self.bias), ptr(xc), ptr(xs),
                      ptr(yc), ptr(ys), M, ptr(rc_), ptr(rs_))
        return yc, ys

    def forward_secure_gpu(self, _ctx: ServerContext | None, client_share, server_share):
        """Host shares in, host shares out (H2D + kernel + D2H), as forward_secure_gpu."""
        c = np.asarray(client_share, dtype=np.float32).reshape(-1)
        s = np.asarray(server_share, dtype=np.float32).reshape(-1)
        if c.size != self._in:
            raise SharingError(f"ShapeMismatch: expected [{self._in}], got [{c.size}]")
        if s.size != self._in:
            raise SharingError(f"ShapeMismatch: expected [{self._in}], got [{s.size}]")
        yc, ys = self.forward_secure_gpu_tensor(self.ctx.to_device(c), self.ctx.to_device(s))
        return yc.cpu().numpy(), ys.cpu().numpy()


# ------------------------------------------------------------------------------------------------
# v1 ring shares (Q16.16 over Z_2^32)
# ------------------------------------------------------------------------------------------------
@dataclass
class Share:
    data: np.ndarray  # int32
    scale: int = 16

    def __len__(self) -> int:
        return int(np.asarray(self.data).size)


@dataclass
class LinearRequestMsg:
    client_share: np.ndarray
    scale: int


@dataclass
class LinearResponseMsg:
    client_output_share: np.ndarray
    server_output_share: np.ndarray
    scale: int


class FixedPointError(ValueError):
    """Overflow / Underflow / InvalidScale of crates/fixed_point/src/error.rs."""


def fixed_from_f64_slice(ctx: Context, values, scale: int = 16) -> torch.Tensor:
    """FixedVector::from_f64_slice on the device: raw = round(v * 2^scale), half away from zero.
    Raises FixedPointError for the first element outside i32 (as the reference's `?` does)."""
    from ._lib import ShdError

    v = values if isinstance(values, torch.Tensor) else torch.as_tensor(np.asarray(values, np.float64))
    v = v.to(device=ctx.torch_device, dtype=torch.float64).contiguous().reshape(-1)
    out = ctx.empty(v.numel(), dtype=torch.int32)
    try:
        ctx.call("shd_fixed_from_f64", ptr(v), v.numel(), scale, ptr(out))
    except ShdError as e:
        raise FixedPointError(str(e)) from None
    return out


def random_share_seeded(ctx: Context, x: torch.Tensor, seed: int):
    """SharePair::from_plaintext_seeded on device i32 plaintext: (client, server) shares with the
    server share = ChaCha20Rng::seed_from_u64(seed) words, client = x wrapping_sub server."""
    x = x.to(device=ctx.torch_device, dtype=torch.int32).contiguous().reshape(-1)
    xc, xs = torch.empty_like(x), torch.empty_like(x)
    ctx.call("shd_ring_share_seeded", ptr(x), x.numel(), seed & 0xFFFFFFFFFFFFFFFF, ptr(xc), ptr(xs))
    return xc, xs


class SharePair:
    """SharePair::from_plaintext_seeded (crates/sharing/src/share.rs:116-135) for host callers."""

    def __init__(self, client: Share, server: Share):
        self.client, self.server = client, server

    @classmethod
    def from_plaintext_seeded(cls, ctx: Context, plaintext_raw, scale: int, seed: int) -> "SharePair":
        xc, xs = random_share_seeded(ctx, torch.as_tensor(np.asarray(plaintext_raw, np.int32)), seed)
        return cls(Share(xc.cpu().numpy(), scale), Share(xs.cpu().numpy(), scale))

    def reconstruct(self) -> np.ndarray:
        if self.client.scale != self.server.scale:
            raise SharingError(f"ScaleMismatch: expected {self.client.scale}, got {self.server.scale}")
        if len(self.client) != len(self.server):
            raise SharingError(f"DimensionMismatch: expected {len(self.client)}, got {len(self.server)}")
        return (self.client.data.astype(np.int64) + self.server.data.astype(np.int64)).astype(np.int32)


def get_embeddings_direct(ctx: Context, table: torch.Tensor, token_ids, session_id: bytes):
    """get_embeddings_direct: shares of the bf16 embedding rows of one request, the server share
    drawn from ChaCha20Rng::from_seed(session id || 16 zero bytes), bit-exact with the reference.
    table: device bf16 [vocab][hidden]; session_id: the 16 UUID bytes."""
    if len(session_id) != 16:
        raise SharingError("InvalidRequest: session id must be 16 bytes")
    vocab, hidden = table.shape
    tok = np.asarray(token_ids, np.int64).reshape(-1)
    bad = tok[(tok < 0) | (tok >= vocab)]
    if bad.size:
        raise SharingError(f"InvalidRequest: Token ID {int(bad[0])} out of range (vocab_size={vocab})")
    t = ctx.to_device(tok.astype(np.int32))
    hc, hs = ctx.empty(tok.size, hidden), ctx.empty(tok.size, hidden)
    sid = np.frombuffer(bytes(session_id), np.uint8).copy()
    ctx.call("shd_embed_shares_session", ptr(table.contiguous()), vocab, hidden, ptr(t), tok.size,
             sid.ctypes.data, ptr(hc), ptr(hs))
    return hc, hs


class LinearServer:
    """LinearServer::new / handle_request on the GPU: bit-exact ring GEMV for both shares."""

    def __init__(self, weight, bias, in_features: int, out_features: int, scale: int, device: Context):
        w = np.asarray(weight, dtype=np.int32).reshape(-1)
        if w.size != in_features * out_features:
            raise SharingError(f"DimensionMismatch: expected {in_features * out_features}, got {w.size}")
        if bias is not None and np.asarray(bias).size != out_features:
            raise SharingError(f"DimensionMismatch: expected {out_features}, got {np.asarray(bias).size}")
        self.ctx = device
        self.weight = Weight.from_i32_in_out(device, w, None if bias is None else np.asarray(bias, np.int32),
                                             in_features, out_features)
        self.in_features = in_features
        self.out_features = out_features
        self.scale = scale

    def forward_tensor(self, xc: torch.Tensor, xs: torch.Tensor):
        """Device int32 shares [M, in] -> (Y_c, Y_s) [M, out]."""
        M = xc.numel() // self.in_features
        yc = self.ctx.empty(M, self.out_features, dtype=torch.int32)
        ys = self.ctx.empty(M, self.out_features, dtype=torch.int32)
        self.ctx.call("shd_linear_dual_ring", self.weight.handle, None, ptr(xc.contiguous()),
                      ptr(xs.contiguous()), ptr(yc), ptr(ys), M, self.scale)
        return yc, ys

    def handle_request(self, request: LinearRequestMsg, server_input_share: Share) -> LinearResponseMsg:
        c = np.asarray(request.client_share, dtype=np.int32).reshape(-1)
        s = np.asarray(server_input_share.data, dtype=np.int32).reshape(-1)
        if c.size != self.in_features:
            raise SharingError(f"DimensionMismatch: expected {self.in_features}, got {c.size}")
        if s.size != self.in_features:
            raise SharingError(f"DimensionMismatch: expected {self.in_features}, got {s.size}")
        if request.scale != self.scale:
            raise SharingError(f"ScaleMismatch: expected {self.scale}, got {request.scale}")
        yc, ys = self.forward_tensor(self.ctx.to_device(c), self.ctx.to_device(s))
        return LinearResponseMsg(yc.cpu().numpy().reshape(-1), ys.cpu().numpy().reshape(-1), self.scale)


# ------------------------------------------------------------------------------------------------
# Beaver triples (V3-MPC)
# ------------------------------------------------------------------------------------------------
@dataclass
class BeaverTriples:
    """A batch of f32 triples as device tensors (BeaverTriple fields, one element per triple)."""
    a: torch.Tensor
    b: torch.Tensor
    c: torch.Tensor
    a_client: torch.Tensor
    a_server: torch.Tensor
    b_client: torch.Tensor
    b_server: torch.Tensor
    c_client: torch.Tensor
    c_server: torch.Tensor

    def __len__(self) -> int:
        return self.a.numel()


def beaver_triples_f32(ctx: Context, n: int, seed: int, offset: int = 0) -> BeaverTriples:
    """BeaverTriple::random_batch (beaver.rs:44-75) from a seeded counter generator."""
    t = [ctx.empty(n) for _ in range(9)]
    ctx.call("shd_beaver_triples_f32", seed, offset, n, *[ptr(x) for x in t[:3]],
             ptr(t[3]), ptr(t[4]), ptr(t[5]), ptr(t[6]), ptr(t[7]), ptr(t[8]))
    return BeaverTriples(*t)


class BeaverTripleStore:
    """BeaverTripleStore (beaver.rs:80-156): per-layer pools with a wrapping cursor."""

    def __init__(self, ctx: Context, num_layers: int, triples_per_layer: int, seed: int = 0):
        self.ctx = ctx
        self.triples_per_layer = triples_per_layer
        self.layers = [beaver_triples_f32(ctx, triples_per_layer, seed, offset=l * triples_per_layer)
                       for l in range(num_layers)]
        self.cursors = [0] * num_layers

    @classmethod
    def pregenerate(cls, ctx: Context, num_layers: int, triples_per_layer: int, seed: int = 0):
        return cls(ctx, num_layers, triples_per_layer, seed)

    def get_layer_triples(self, layer_idx: int) -> BeaverTriples:
        return self.layers[layer_idx]

    def get_triples(self, layer_idx: int, count: int) -> torch.Tensor:
        """Indices of the next `count` triples of a layer (wrapping), advancing the cursor."""
        start = self.cursors[layer_idx]
        self.cursors[layer_idx] += count
        return (torch.arange(count, device=self.ctx.torch_device) + start) % self.triples_per_layer

    def reset(self) -> None:
        self.cursors = [0] * len(self.cursors)

    def memory_usage(self) -> int:
        return len(self.layers) * self.triples_per_layer * 9 * 4


def secure_multiply_batch(ctx: Context, x_client, x_server, y_client, y_server, t: BeaverTriples,
                          return_opened: bool = False):
    """z = x*y on shares (beaver.rs:201-233); returns (z_c, z_s) [, (d, e)]."""
    xs = [_f32(v) for v in (x_client, x_server, y_client, y_server)]
    n = xs[0].numel()
    if any(v.numel() != n for v in xs) or len(t) < n:
        raise SharingError("ShapeMismatch: share and triple lengths differ")
    zc, zs = ctx.empty(n), ctx.empty(n)
    d = ctx.empty(n) if return_opened else None
    e = ctx.empty(n) if return_opened else None
    tr = [t.a_client, t.a_server, t.b_client, t.b_server, t.c_client, t.c_server]
    ctx.call("shd_beaver_mul_f32", *[ptr(v) for v in xs], *[ptr(v) for v in tr], ptr(d), ptr(e),
             ptr(zc), ptr(zs), n)
    return ((zc, zs), (d, e)) if return_opened else (zc, zs)


def secure_multiply_mpc(ctx: Context, x_client: float, x_server: float, y_client: float,
                        y_server: float, triple: BeaverTriples, index: int = 0):
    """Scalar form of secure_multiply_mpc (beaver.rs:167-197) using triple `index` of a batch."""
    dev = ctx.torch_device
    one = lambda v: torch.tensor([v], dtype=torch.float32, device=dev)
    sub = BeaverTriples(*[getattr(triple, f)[index:index + 1].contiguous() for f in BeaverTriples.__dataclass_fields__])
    zc, zs = secure_multiply_batch(ctx, one(x_client), one(x_server), one(y_client), one(y_server), sub)
    return float(zc.item()), float(zs.item())


def beaver_mul_ring(ctx: Context, xc, xs, yc, ys, ac, as_, bc, bs, cc, cs, trunc_shift: int = 0,
                    return_opened: bool = False):
    """Z_2^32 Beaver multiply on uint32/int32 device tensors (wrapping; optional truncation)."""
    ins = [v.contiguous() for v in (xc, xs, yc, ys, ac, as_, bc, bs, cc, cs)]
    n = ins[0].numel()
    zc, zs = ctx.empty(n, dtype=torch.int32), ctx.empty(n, dtype=torch.int32)
    d = ctx.empty(n, dtype=torch.int32) if return_opened else None
    e = ctx.empty(n, dtype=torch.int32) if return_opened else None
    ctx.call("shd_beaver_mul_ring", *[ptr(v) for v in ins], ptr(d), ptr(e), ptr(zc), ptr(zs), n,
             trunc_shift)
    return ((zc, zs), (d, e)) if return_opened else (zc, zs)


def beaver_triples_ring(ctx: Context, n: int, seed: int, offset: int = 0):
    t = [ctx.empty(n, dtype=torch.int32) for _ in range(6)]
    ctx.call("shd_beaver_triples_ring", seed, offset, n, *[ptr(x) for x in t])
    return t  # a_c, a_s, b_c, b_s, c_c, c_s


def fill_uniform(ctx: Context, n: int, seed: int, lo: float, hi: float, offset: int = 0) -> torch.Tensor:
    out = ctx.empty(n)
    ctx.call("shd_fill_uniform_f32", seed, offset, lo, hi, ptr(out), n)
    return out


def reconstruct(ctx: Context, c: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    y = ctx.empty(*c.shape)
    ctx.call("shd_reconstruct_f32", ptr(_f32(c)), ptr(_f32(s)), ptr(y), c.numel())
    return y


def reshare(ctx: Context, y: torch.Tensor, mask: torch.Tensor | None = None):
    oc, os_ = ctx.empty(*y.shape), ctx.empty(*y.shape)
    ctx.call("shd_reshare_f32", ptr(_f32(y)), ptr(mask), ptr(oc), ptr(os_), y.numel())
    return oc, os_


def secure_add_gpu(ctx: Context, a_client, a_server, b_client, b_server):
    """secure_add_gpu (crates/v2/sharing/src/secure_nonlinear_gpu.rs:195-212)."""
    yc, ys = ctx.empty(*a_client.shape), ctx.empty(*a_client.shape)
    ctx.call("shd_add_shares", ptr(_f32(a_client)), ptr(_f32(a_server)), ptr(_f32(b_client)),
             ptr(_f32(b_server)), ptr(yc), ptr(ys), a_client.numel())
    return yc, ys


__all__ = [
    "GpuSecureLinear", "ServerContext", "SharingError", "Share", "LinearRequestMsg",
    "LinearResponseMsg", "LinearServer", "BeaverTriples", "BeaverTripleStore",
    "beaver_triples_f32", "secure_multiply_batch", "secure_multiply_mpc", "beaver_mul_ring",
    "beaver_triples_ring", "fill_uniform", "reconstruct", "reshare", "secure_add_gpu", "NL_APPROX",
]


# ------------------------------------------------------------------------------------------------
# V3-OT function tables and the server's OT query processing
# ------------------------------------------------------------------------------------------------
class StandardOtTables:
    """StandardOtTables::new(table_size) (crates/v2/sharing/src/secure_nonlinear_ot.rs:554-575) on
    the device: silu, exp, rsqrt, reciprocal tables of f32 (4 bytes per row, as the reference's
    as_bytes())."""

    RANGES = {"silu": (-8.0, 8.0), "exp": (-10.0, 0.0), "rsqrt": (0.01, 10.0), "reciprocal": (0.01, 100.0)}

    def __init__(self, ctx: Context, table_size: int = 4096):
        self.ctx, self.size = ctx, table_size
        self.values = ctx.empty(4, table_size)
        ctx.call("shd_ot_standard_tables", table_size, ptr(self.values))
        self.index = {k: i for i, k in enumerate(self.RANGES)}

    def table(self, name: str) -> torch.Tensor:
        """The table of an operation name as the route maps them (rmsnorm/rsqrt, silu/swiglu,
        softmax/exp, reciprocal)."""
        alias = {"rmsnorm": "rsqrt", "swiglu": "silu", "softmax": "exp"}
        return self.values[self.index[alias.get(name, name)]]


class OtFunctionServer:
    """OtFunctionServer (crates/v2/sharing/src/secure_nonlinear_ot.rs:173-235) answering queries on
    the GPU: the session commitment comes from the base-OT handshake (out of scope here), the
    session counter advances by one per query as the reference's does."""

    def __init__(self, ctx: Context, commitment: bytes):
        if len(commitment) != 32:
            raise SharingError("session commitment must be 32 bytes")
        self.ctx, self.commitment, self.session_ctr = ctx, bytes(commitment), 0

    def process_query(self, query: bytes, table: torch.Tensor) -> bytes:
        self.session_ctr += 1
        q = np.frombuffer(bytes(query), np.uint8).copy()
        com = np.frombuffer(self.commitment, np.uint8).copy()
        m = int(q[0]) | (int(q[1]) << 8) if q.size >= 2 else 0
        out = np.empty(max(1, m * 4), np.uint8)
        n = C.c_size_t(0)
        t = table.contiguous()
        self.ctx.call("shd_ot_process_query", com.ctypes.data, self.session_ctr, q.ctypes.data, q.size, ptr(t),
                      t.numel() * t.element_size(), 4, out.ctypes.data, out.size, C.byref(n))
        return out[: n.value].tobytes()
