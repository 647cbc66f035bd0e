"""v1 ring linear (shd_linear_dual_ring) bit-exact vs the oracle's LinearServer::multiply_vector.

Integer arithmetic: every share element must be identical (no tolerance).
"""
import json
import pathlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_known_answers.json").read_text())


def _config1(seed=1):
    """W 1536x1536 ~ N(0,0.02) and x ~ N(0,1) in Q16.16, x_s uniform over Z_2^32."""
    rng = np.random.default_rng(seed)
    w = np.round(rng.standard_normal((1536, 1536)) * 0.02 * 65536).astype(np.int32)  # [in][out]
    x = np.round(rng.standard_normal(1536) * 65536).astype(np.int32)
    xs = rng.integers(0, 2**32, 1536, dtype=np.uint64).astype(np.uint32).view(np.int32)
    xc = (x.astype(np.int64) - xs.astype(np.int64)).astype(np.int32)
    return w, x, xc, xs


def test_config1_bit_exact(ctx, orc):
    from shardlm_b200.sharing import LinearRequestMsg, LinearServer, Share

    w, x, xc, xs = _config1()
    srv = LinearServer(w.reshape(-1), None, 1536, 1536, 16, ctx)
    resp = srv.handle_request(LinearRequestMsg(xc, 16), Share(xs, 16))
    oc, os_ = orc.linear_ring(w, None, xc, xs, 16)
    assert np.array_equal(resp.client_output_share, oc[0])
    assert np.array_equal(resp.server_output_share, os_[0])
    # reconstruction vs plaintext W.x: +-1 LSB except where x_c + x_s wrapped (reported, not failed)
    y = (resp.client_output_share.astype(np.int64) + resp.server_output_share).astype(np.int32)
    p = orc.plaintext_linear_ring(w, None, x, 16)
    wrapped = (xc.astype(np.int64) + xs.astype(np.int64) != x.astype(np.int64))
    if not wrapped.any():
        assert np.max(np.abs(y.astype(np.int64) - p)) <= 1


@pytest.mark.parametrize("K,N,M,bias", [(128, 32, 1, False), (1000, 77, 3, True), (4096, 2048, 8, True), (4, 3, 2, True)])
def test_ring_shapes_bit_exact(ctx, orc, K, N, M, bias):
    from shardlm_b200.sharing import LinearServer

    rng = np.random.default_rng(K + N)
    w = rng.integers(-2**31, 2**31, (K, N), dtype=np.int64).astype(np.int32)
    b = rng.integers(-2**31, 2**31, N, dtype=np.int64).astype(np.int32) if bias else None
    xc = rng.integers(-2**31, 2**31, (M, K), dtype=np.int64).astype(np.int32)
    xs = rng.integers(-2**31, 2**31, (M, K), dtype=np.int64).astype(np.int32)
    srv = LinearServer(w.reshape(-1), b, K, N, 16, ctx)
    yc, ys = srv.forward_tensor(ctx.to_device(xc), ctx.to_device(xs))
    ctx.sync()
    oc, os_ = orc.linear_ring(w, b, xc, xs, 16)
    assert np.array_equal(yc.cpu().numpy(), oc)
    assert np.array_equal(ys.cpu().numpy(), os_)


def test_ring_scales(ctx, orc):
    from shardlm_b200.sharing import LinearServer

    rng = np.random.default_rng(3)
    w = rng.integers(-2**20, 2**20, (512, 64), dtype=np.int64).astype(np.int32)
    xc = rng.integers(-2**31, 2**31, (1, 512), dtype=np.int64).astype(np.int32)
    xs = rng.integers(-2**31, 2**31, (1, 512), dtype=np.int64).astype(np.int32)
    for scale in (0, 8, 16, 30):
        srv = LinearServer(w.reshape(-1), None, 512, 64, scale, ctx)
        yc, ys = srv.forward_tensor(ctx.to_device(xc), ctx.to_device(xs))
        oc, os_ = orc.linear_ring(w, None, xc, xs, scale)
        assert np.array_equal(yc.cpu().numpy(), oc) and np.array_equal(ys.cpu().numpy(), os_)


@pytest.mark.parametrize("name", ["ring_identity", "ring_bias", "ring_matrix_multiply"])
def test_ring_known_answers_gpu(ctx, orc, name):
    from shardlm_b200.sharing import LinearRequestMsg, LinearServer, Share

    c = GOLD[name]
    if "weight_f64_in_out" in c:
        w = np.array([orc.fixed_from_f64(v) for v in c["weight_f64_in_out"]], np.int32)
    else:
        w = np.asarray(c["weight_in_out"], np.int32)
    x = np.array([orc.fixed_from_f64(v) for v in c["x_f64"]], np.int32)
    srv = LinearServer(w, c["bias"], c["in"], c["out"], c["scale"], ctx)
    rng = np.random.default_rng(0)
    xs = rng.integers(-2**31, 2**31, x.size, dtype=np.int64).astype(np.int32)
    xc = (x.astype(np.int64) - xs).astype(np.int32)
    r = srv.handle_request(LinearRequestMsg(xc, 16), Share(xs, 16))
    y = (r.client_output_share.astype(np.int64) + r.server_output_share).astype(np.int32) / 65536.0
    assert np.all(np.abs(y - np.asarray(c["expected"])) < c["tol"])


def test_scale_mismatch_raises(ctx):
    from shardlm_b200.sharing import LinearRequestMsg, LinearServer, Share, SharingError

    srv = LinearServer(np.zeros(4, np.int32), None, 2, 2, 16, ctx)
    with pytest.raises(SharingError, match="ScaleMismatch"):
        srv.handle_request(LinearRequestMsg(np.zeros(2, np.int32), 12), Share(np.zeros(2, np.int32), 12))
    with pytest.raises(SharingError, match="DimensionMismatch"):
        srv.handle_request(LinearRequestMsg(np.zeros(3, np.int32), 16), Share(np.zeros(2, np.int32), 16))
