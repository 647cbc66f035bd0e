"""The allocation-free linear entry point (shd_linear_dual_f32_noalloc) through the C ABI.

It serves callers that cannot allocate device memory while running a layer (a host framework that
owns the GPU's memory, a request path that must not allocate): the split-K scratch is a static
device array instead of context allocations. Its output must match shd_linear_dual_f32 on the same
weight and shares within the f32 summation tolerance of tests/test_linear.py, on two calls in a row
(the second call reuses the array the first one left behind).

This file is collected last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_round, f32_sum_tolerance

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,N,M", [(3584, 3584, 1), (1000, 4100, 3), (18944, 3584, 2)])
def test_noalloc_linear_matches_linear(ctx, orc, K, N, M):
    from shardlm_b200._lib import check, lib
    from shardlm_b200.runtime import Weight, ptr

    rng = np.random.default_rng(K + N + M)
    w_u16 = bf16_round((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs_h = rng.uniform(0, 1, (M, K)).astype(np.float32)
    xc_h = (x - xs_h).astype(np.float32)
    bias_h = (rng.standard_normal(N) * 0.02).astype(np.float32)
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    xc, xs, bias = ctx.to_device(xc_h), ctx.to_device(xs_h), ctx.to_device(bias_h)

    ref_c, ref_s = ctx.empty(M, N), ctx.empty(M, N)
    ctx.call("shd_linear_dual_f32", w.handle, ptr(bias), ptr(xc), ptr(xs), ptr(ref_c), ptr(ref_s), M, None, None)
    ctx.sync()

    stream = torch.cuda.current_stream().cuda_stream
    abs_c = [orc.linear_abs_bf16(np.ascontiguousarray(w_u16.T), xc_h[m]) for m in range(M)]
    abs_s = [orc.linear_abs_bf16(np.ascontiguousarray(w_u16.T), xs_h[m]) for m in range(M)]
    for call in range(2):
        yc, ys = ctx.empty(M, N), ctx.empty(M, N)
        check(lib().shd_linear_dual_f32_noalloc(w.handle, ptr(bias), ptr(xc), ptr(xs), ptr(yc), ptr(ys), M,
                                                None, None, stream))
        torch.cuda.synchronize()
        for m in range(M):
            tc = f32_sum_tolerance(K, abs_c[m])
            ts = f32_sum_tolerance(K, abs_s[m]) + np.abs(bias_h) * 2.0 ** -23
            dc = np.abs(yc[m].cpu().numpy() - ref_c[m].cpu().numpy())
            ds = np.abs(ys[m].cpu().numpy() - ref_s[m].cpu().numpy())
            assert np.all(dc <= tc), f"call {call} row {m}: client share max diff {dc.max()}"
            assert np.all(ds <= ts), f"call {call} row {m}: server share max diff {ds.max()}"


def test_noalloc_rejects_what_it_cannot_stage(ctx):
    from shardlm_b200._lib import SHD_ERR_ARG, lib
    from shardlm_b200.runtime import Weight, ptr

    w = Weight.from_bf16_out_in(ctx, (torch.randn(64, 6, device="cuda") * 0.02).to(torch.bfloat16))
    x = torch.zeros(1, 6, device="cuda")
    y = torch.zeros(1, 64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # in_features % 4 != 0 would need a staging copy, which this entry point cannot allocate
    assert lib().shd_linear_dual_f32_noalloc(w.handle, None, ptr(x), ptr(x), ptr(y), ptr(y), 1, None, None, stream) == SHD_ERR_ARG
