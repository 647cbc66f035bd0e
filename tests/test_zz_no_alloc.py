"""The allocation-free linear entry point (shd_linear_dual_f32_noalloc) through the C ABI.

It serves callers that cannot allocate device memory while running a layer (a host framework that
owns and freezes the GPU's memory, a request path that must not allocate): the split-K scratch is
a static device array instead of context allocations. Its output must match the oracle's
SecureLinear::matmul order (crates/v2/sharing/src/secure_linear.rs:103-117) within the f32
summation tolerance of tests/test_linear.py, and shd_linear_dual_f32 on the same weight and
shares, on two calls in a row (the second call reuses the array the first one left behind).

Rows are processed 8 per launch, so M = 11 and 17 run several launches in one call whose tile
counters must come back to zero inside the kernel. One case runs on a fresh side stream right
after the weight is created, with no synchronisation in between.

This file is collected last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest
import torch

from conftest import bf16_round, f32_sum_tolerance

pytestmark = pytest.mark.gpu


def _noalloc(w, bias, xc, xs, yc, ys, M, stream):
    from shardlm_b200._lib import check, lib
    from shardlm_b200.runtime import ptr

    check(lib().shd_linear_dual_f32_noalloc(w.handle, ptr(bias), ptr(xc), ptr(xs), ptr(yc), ptr(ys), M,
                                            None, None, stream))


@pytest.mark.parametrize("K,N,M,side_stream", [
    (3584, 3584, 1, False),
    (1000, 4100, 3, False),
    (18944, 3584, 2, False),
    (3584, 4608, 5, False),    # 5-8 rows: one GEMV launch of 5-8 rows (the tensor cores take these
    (1536, 8960, 6, False),    # rows in shd_linear_dual_f32)
    (3584, 512, 7, True),
    (18944, 3584, 8, False),
    (2048, 1000, 11, False),   # two launches
    (1024, 2048, 17, True),    # three launches
])
def test_noalloc_linear_matches_oracle_and_linear(ctx, orc, K, N, M, side_stream):
    from shardlm_b200.runtime import Weight, ptr

    rng = np.random.default_rng(K + N + M)
    w_u16 = bf16_round((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs_h = rng.uniform(0, 1, (M, K)).astype(np.float32)
    xc_h = (x - xs_h).astype(np.float32)
    bias_h = (rng.standard_normal(N) * 0.02).astype(np.float32)
    xc, xs, bias = ctx.to_device(xc_h), ctx.to_device(xs_h), ctx.to_device(bias_h)
    torch.cuda.synchronize()

    s = torch.cuda.Stream() if side_stream else torch.cuda.current_stream()
    w = Weight.from_bf16_out_in(ctx, torch.from_numpy(w_u16.view(np.int16)).view(torch.bfloat16).cuda())
    outs = []
    with torch.cuda.stream(s):
        for call in range(2):
            yc, ys = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
            _noalloc(w, bias, xc, xs, yc, ys, M, s.cuda_stream)
            outs.append((yc, ys))
    s.synchronize()

    ref_c, ref_s = ctx.empty(M, N), ctx.empty(M, N)
    ctx.call("shd_linear_dual_f32", w.handle, ptr(bias), ptr(xc), ptr(xs), ptr(ref_c), ptr(ref_s), M, None, None)
    ctx.sync()
    ref_c, ref_s = ref_c.cpu().numpy(), ref_s.cpu().numpy()

    w_in_out = np.ascontiguousarray(w_u16.T)
    oc, os_ = orc.linear_bf16(w_in_out, bias_h, xc_h, xs_h)
    for call, (yc, ys) in enumerate(outs):
        yc, ys = yc.cpu().numpy(), ys.cpu().numpy()
        for m in range(M):
            tc = f32_sum_tolerance(K, orc.linear_abs_bf16(w_in_out, xc_h[m]))
            ts = f32_sum_tolerance(K, orc.linear_abs_bf16(w_in_out, xs_h[m])) + np.abs(bias_h) * 2.0 ** -23
            for name, got, want_o, want_l, tol in (("client", yc[m], oc[m], ref_c[m], tc),
                                                   ("server", ys[m], os_[m], ref_s[m], ts)):
                d_o = np.abs(got - want_o)
                assert np.all(d_o <= tol), f"call {call} row {m}: {name} share vs oracle, max diff {d_o.max()}"
                d_l = np.abs(got - want_l)
                assert np.all(d_l <= tol), f"call {call} row {m}: {name} share vs shd_linear_dual_f32, max diff {d_l.max()}"


def test_noalloc_rejects_what_it_cannot_stage(ctx):
    from shardlm_b200._lib import SHD_ERR_ARG, lib
    from shardlm_b200.runtime import Weight, ptr

    w = Weight.from_bf16_out_in(ctx, (torch.randn(64, 6, device="cuda") * 0.02).to(torch.bfloat16))
    x = torch.zeros(1, 6, device="cuda")
    y = torch.zeros(1, 64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # in_features % 4 != 0 would need a staging copy, which this entry point cannot allocate
    assert lib().shd_linear_dual_f32_noalloc(w.handle, None, ptr(x), ptr(x), ptr(y), ptr(y), 1, None, None, stream) == SHD_ERR_ARG
    # out_features beyond the static scratch's tile counters (262144)
    big = Weight.from_bf16_out_in(ctx, torch.zeros(262144 + 32, 8, device="cuda", dtype=torch.bfloat16))
    x8 = torch.zeros(1, 8, device="cuda")
    y8 = torch.zeros(1, 262144 + 32, device="cuda")
    assert lib().shd_linear_dual_f32_noalloc(big.handle, None, ptr(x8), ptr(x8), ptr(y8), ptr(y8), 1, None, None, stream) == SHD_ERR_ARG
