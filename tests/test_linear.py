"""Dual-share f32 linear (shd_linear_dual_f32) vs the oracle's SecureLinear::matmul order.

Tolerance: the GPU sums the K products of an output in a different order than the reference's
sequential i-outer loop, so results agree within the f32 summation bound
2 * gamma_K * sum_i |x_i||W_ij| (conftest.f32_sum_tolerance), per share, for every element. From 33
rows the tensor-core linear accumulates the three bf16 terms of each activation in one f32
accumulator, a sum of 3K exact products: the bound is then 2 * gamma_3K * sum_i |x_i||W_ij|.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_round, bf16_to_f32, f32_sum_tolerance

pytestmark = pytest.mark.gpu


def _case(rng, K, N, M, with_bias):
    w_f = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w_u16 = bf16_round(w_f)  # [out][in]
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs = rng.uniform(0, 1, (M, K)).astype(np.float32)
    xc = (x - xs).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32) if with_bias else None
    return w_u16, xc, xs, b


def _terms(M):
    """Products summed per output: K, or 3K when the tensor-core linear fuses the terms (M > 32)."""
    return 3 if M > 32 else 1


def _check(orc, w_u16, xc, xs, b, yc, ys, residual=None):
    N, K = w_u16.shape
    KS = K * _terms(xc.shape[0])
    w_in_out = np.ascontiguousarray(w_u16.T)
    oc, os_ = orc.linear_bf16(w_in_out, b, xc, xs)
    if residual is not None:
        oc = (oc + residual[0]).astype(np.float32)
        os_ = (os_ + residual[1]).astype(np.float32)
    for m in range(xc.shape[0]):
        tc = f32_sum_tolerance(KS, orc.linear_abs_bf16(w_in_out, xc[m]))
        ts = f32_sum_tolerance(KS, orc.linear_abs_bf16(w_in_out, xs[m]))
        if b is not None:
            ts = ts + np.abs(b) * 2 ** -23
        if residual is not None:
            tc = tc + np.abs(residual[0][m]) * 2 ** -23
            ts = ts + np.abs(residual[1][m]) * 2 ** -23
        assert np.all(np.abs(yc[m] - oc[m]) <= tc), f"client share row {m}: max {np.max(np.abs(yc[m]-oc[m]))}"
        assert np.all(np.abs(ys[m] - os_[m]) <= ts), f"server share row {m}: max {np.max(np.abs(ys[m]-os_[m]))}"


@pytest.mark.parametrize("K,N,M,bias", [
    (256, 32, 1, False),       # one block
    (1536, 1536, 1, True),     # 1.5B q-projection shape
    (3584, 512, 1, True),      # 7B k/v shape
    (1000, 77, 3, True),       # ragged N and K (K % 4 == 0, not a multiple of 256)
    (8960, 1536, 2, False),    # 1.5B down projection, split-K across CTAs
    (4, 2, 1, True),           # tiny
    # 5 rows and more: tcgen05 tensor-core path (three bf16 terms per f32 share, f32 accumulation
    # in TMEM); up to 8 rows an 8-row token tile, whose one MMA covers both shares
    (520, 4100, 5, False),     # 5 rows, ragged K
    (3584, 3584, 8, True),     # 8 rows, 7B o shape
    (18944, 3584, 6, False),   # 6 rows, 7B down shape: split K and the reduce kernel
    (3584, 4608, 64, True),    # 7B q/k/v shape, one 64-row token tile (terms fused)
    (1000, 77, 9, True),       # ragged N and K, 16-row token tile
    (18944, 3584, 33, False),  # 7B down shape
    (1536, 1536, 130, True),   # two 128-row token tiles (terms fused), ragged last
    (1000, 700, 200, True),    # 128-row token tiles, ragged N, K and M
    (4, 2, 17, True),          # tiny
])
def test_linear_dual_f32_matches_oracle(ctx, orc, K, N, M, bias):
    from shardlm_b200.runtime import Weight
    from shardlm_b200.sharing import GpuSecureLinear

    rng = np.random.default_rng(K * 7 + N + M)
    w_u16, xc, xs, b = _case(rng, K, N, M, bias)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    lin = GpuSecureLinear(ctx, w, None if b is None else ctx.to_device(b))
    yc, ys = lin.forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs))
    ctx.sync()
    _check(orc, w_u16, xc, xs, b, yc.cpu().numpy(), ys.cpu().numpy())


def test_linear_residual_epilogue(ctx, orc):
    from shardlm_b200.runtime import Weight
    from shardlm_b200.sharing import GpuSecureLinear

    rng = np.random.default_rng(5)
    w_u16, xc, xs, _ = _case(rng, 3584, 3584, 1, False)
    rc = rng.standard_normal((1, 3584)).astype(np.float32)
    rs = rng.standard_normal((1, 3584)).astype(np.float32)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    lin = GpuSecureLinear(ctx, w, None)
    yc, ys = lin.forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs),
                                           residual=(ctx.to_device(rc), ctx.to_device(rs)))
    ctx.sync()
    _check(orc, w_u16, xc, xs, None, yc.cpu().numpy(), ys.cpu().numpy(), residual=(rc, rs))


def test_linear_tensor_core_residual_and_determinism(ctx, orc):
    """M > 8 rows through the tensor cores: residual epilogue, and repeated calls bit-identical."""
    from shardlm_b200.runtime import Weight
    from shardlm_b200.sharing import GpuSecureLinear

    rng = np.random.default_rng(6)
    w_u16, xc, xs, _ = _case(rng, 3584, 3584, 40, False)
    rc = rng.standard_normal((40, 3584)).astype(np.float32)
    rs = rng.standard_normal((40, 3584)).astype(np.float32)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    lin = GpuSecureLinear(ctx, w, None)
    res = (ctx.to_device(rc), ctx.to_device(rs))
    outs = [lin.forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs), residual=res) for _ in range(3)]
    ctx.sync()
    _check(orc, w_u16, xc, xs, None, outs[0][0].cpu().numpy(), outs[0][1].cpu().numpy(), residual=(rc, rs))
    for o in outs[1:]:
        assert torch.equal(o[0], outs[0][0]) and torch.equal(o[1], outs[0][1])


def test_linear_deterministic_across_calls(ctx):
    """Split-K partials are combined in a fixed order: repeated calls are bit-identical."""
    from shardlm_b200.runtime import Weight
    from shardlm_b200.sharing import GpuSecureLinear

    rng = np.random.default_rng(11)
    w_u16, xc, xs, _ = _case(rng, 18944, 3584, 1, False)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    lin = GpuSecureLinear(ctx, w, None)
    a = lin.forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs))
    outs = [lin.forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs)) for _ in range(3)]
    ctx.sync()
    for o in outs:
        assert torch.equal(o[0], a[0]) and torch.equal(o[1], a[1])


def test_from_cpu_known_answer(ctx):
    """test_secure_linear_correctness (crates/v2/sharing/src/secure_linear.rs:416-461) on the GPU."""
    from shardlm_b200.sharing import GpuSecureLinear, ServerContext

    weight = [1.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.5, 0.5]
    lin = GpuSecureLinear.from_cpu(weight, [0.1, 0.2], 4, 2, ctx)
    rng = np.random.default_rng(42)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    xs = rng.uniform(-10, 10, 4).astype(np.float32)
    yc, ys = lin.forward_secure_gpu(ServerContext(), x - xs, xs)
    assert np.all(np.abs((yc + ys) - np.array([6.1, 7.2])) < 1e-4)
    assert not np.allclose(yc, [6.1, 7.2]) and not np.allclose(ys, [6.1, 7.2])


def test_from_cpu_rejects_non_bf16_weights(ctx):
    from shardlm_b200._lib import ShdError
    from shardlm_b200.sharing import GpuSecureLinear

    with pytest.raises(ShdError, match="UNSUPPORTED"):
        GpuSecureLinear.from_cpu([0.1, 0.2, 0.3, 0.4], None, 2, 2, ctx)


def test_shape_mismatch_raises(ctx):
    from shardlm_b200.sharing import GpuSecureLinear, ServerContext, SharingError

    lin = GpuSecureLinear.from_cpu([1.0] * 8, None, 4, 2, ctx)
    with pytest.raises(SharingError, match="ShapeMismatch"):
        lin.forward_secure_gpu(ServerContext(), np.zeros(3, np.float32), np.zeros(4, np.float32))
