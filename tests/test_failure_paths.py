"""Failure detection without a GPU fault: a device wait that expires reports SHD_ERR_TIMEOUT through
the context's error word and leaves the context usable.

The self-test kernel waits on a flag that nothing sets, bounded by a short limit of %globaltimer -
the same bound and recording every pipeline wait of the library uses (mbarrier stages, split-tile
exchange, grid barriers, the NVLink all-reduce) - so this exercises the host side of that path: the
error word read and cleared by shd_sync, the message, and the next call succeeding.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_device_wait_reports_timeout_and_recovers(ctx, orc):
    from conftest import bf16_round, f32_sum_tolerance
    from shardlm_b200._lib import SHD_ERR_TIMEOUT, ShdError, check, lib
    from shardlm_b200.runtime import Weight
    from shardlm_b200.sharing import GpuSecureLinear

    ctx.bind_stream()
    check(lib().shd_wait_selftest(ctx.ptr, 50), ctx.ptr)
    with pytest.raises(ShdError) as e:
        ctx.sync()
    assert e.value.code == SHD_ERR_TIMEOUT
    assert "timeout" in str(e.value)
    ctx.sync()  # the word was cleared

    # the context still computes
    rng = np.random.default_rng(0)
    w_u16 = bf16_round((rng.standard_normal((256, 512)) * 0.02).astype(np.float32))
    x = rng.standard_normal((1, 512)).astype(np.float32)
    xs = rng.uniform(0, 1, (1, 512)).astype(np.float32)
    xc = (x - xs).astype(np.float32)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    yc, ys = GpuSecureLinear(ctx, w, None).forward_secure_gpu_tensor(ctx.to_device(xc), ctx.to_device(xs))
    ctx.sync()
    oc, os_ = orc.linear_bf16(np.ascontiguousarray(w_u16.T), None, xc, xs)
    tol = f32_sum_tolerance(512, orc.linear_abs_bf16(np.ascontiguousarray(w_u16.T), xc[0]))
    assert np.all(np.abs(yc.cpu().numpy()[0] - oc[0]) <= tol)


def test_selftest_rejects_unbounded_limits(ctx):
    from shardlm_b200._lib import SHD_ERR_ARG, lib

    assert lib().shd_wait_selftest(ctx.ptr, 0) == SHD_ERR_ARG
    assert lib().shd_wait_selftest(ctx.ptr, 5000) == SHD_ERR_ARG
