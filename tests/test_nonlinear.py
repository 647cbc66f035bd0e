"""Reconstruct-compute-reshare ops, RoPE, attention, embedding shares and greedy sampling vs the
oracle. Bit-exact where the GPU follows the reference's exact operation sequence (RoPE given the
same libm table, reshare masks, embedding shares, argmax); elsewhere within the tolerance stated
per test (reduction order and CUDA expf/rsqrtf vs glibc).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


_LIVE = []


@pytest.fixture(autouse=True)
def _release_staged():
    yield
    torch.cuda.synchronize()
    _LIVE.clear()


def _dev(ctx, a, dtype=np.float32):
    # The raw address goes to the library; keep the tensor alive until the kernels that read it ran.
    t = ctx.to_device(np.ascontiguousarray(a, dtype))
    _LIVE.append(t)
    return t


def _call(ctx, name, *args):
    ctx.call(name, *args)
    ctx.sync()


@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("n", [1536, 3584, 100])
def test_rmsnorm_reshare(ctx, orc, variant, n):
    from shardlm_b200.runtime import ptr

    rng = np.random.default_rng(n + variant)
    M = 3
    x = rng.standard_normal((M, n)).astype(np.float32) * 3
    xs = rng.uniform(0, 1, (M, n)).astype(np.float32)
    xc = (x - xs).astype(np.float32)
    g = rng.uniform(0.5, 1.5, n).astype(np.float32)
    mask = rng.uniform(-1, 1, (M, n)).astype(np.float32) if variant == 2 else None
    yc, ys = ctx.empty(M, n), ctx.empty(M, n)
    # masks are per row here: call row by row so the mask row matches
    for m in range(M):
        ctx.call("shd_rmsnorm_reshare", ptr(_dev(ctx, xc[m])), ptr(_dev(ctx, xs[m])), ptr(_dev(ctx, g)), 1e-6,
                 variant, None if mask is None else ptr(_dev(ctx, mask[m])), ptr(yc[m]), ptr(ys[m]), 1, n)
    ctx.sync()
    for m in range(M):
        oc, os_ = orc.rmsnorm_reshare(xc[m], xs[m], g, 1e-6, variant, None if mask is None else mask[m])
        gc, gs = yc[m].cpu().numpy(), ys[m].cpu().numpy()
        assert np.array_equal(gs, os_)  # the server share is the mask (or 0) exactly
        # sum of squares in another order + rsqrtf (<= 2 ulp): relative 1e-5 of the output scale
        assert np.max(np.abs(gc - oc)) <= 1e-5 * np.max(np.abs(oc)), np.max(np.abs(gc - oc))


@pytest.mark.parametrize("variant", [0, 1, 2])
def test_swiglu_and_silu_reshare(ctx, orc, variant):
    from shardlm_b200.runtime import ptr

    rng = np.random.default_rng(variant)
    n = 18944
    g = (rng.standard_normal(n) * 8).astype(np.float32)
    g[:8] = [30, -30, 20.5, -20.5, 0, -0.0, 1e-30, -50]
    u = rng.standard_normal(n).astype(np.float32)
    gs, us = rng.uniform(0, 1, n).astype(np.float32), rng.uniform(0, 1, n).astype(np.float32)
    gc, uc = (g - gs).astype(np.float32), (u - us).astype(np.float32)
    mask = rng.uniform(-1, 1, n).astype(np.float32) if variant == 2 else None
    yc, ys = ctx.empty(n), ctx.empty(n)
    _call(ctx, "shd_swiglu_reshare", ptr(_dev(ctx, gc)), ptr(_dev(ctx, gs)), ptr(_dev(ctx, uc)), ptr(_dev(ctx, us)),
          variant, None if mask is None else ptr(_dev(ctx, mask)), ptr(yc), ptr(ys), n)
    oc, os_ = orc.swiglu_reshare(gc, gs, uc, us, variant, mask)
    assert np.array_equal(ys.cpu().numpy(), os_)
    # CUDA expf (<= 2 ulp) vs glibc expf: relative 4 ulp per element plus the mask's rounding
    err = np.abs(yc.cpu().numpy() - oc)
    tol = 4 * 2.0 ** -23 * (np.abs(oc) + (np.abs(mask) if mask is not None else 0)) + 1e-30
    assert np.all(err <= tol), np.max(err / tol)
    _call(ctx, "shd_silu_reshare", ptr(_dev(ctx, gc)), ptr(_dev(ctx, gs)), variant, None, ptr(yc), ptr(ys), n)
    oc, _ = orc.silu_reshare(gc, gs, variant)
    err = np.abs(yc.cpu().numpy() - oc)
    assert np.all(err <= 4 * 2.0 ** -23 * np.abs(oc) + 1e-30)


def test_rope_bit_exact(ctx, orc):
    from shardlm_b200.runtime import ptr

    H, d, T = 28, 128, 2048
    ctx.call("shd_rope_init", d, T, 1e6)
    cos_t, sin_t = orc.rope_table(d, T, 1e6)
    rng = np.random.default_rng(0)
    for pos in (0, 1, 511, 2047 - 3):
        M = 3
        xc = rng.standard_normal((M, H * d)).astype(np.float32)
        xs = rng.standard_normal((M, H * d)).astype(np.float32)
        tc, ts = _dev(ctx, xc), _dev(ctx, xs)
        _call(ctx, "shd_rope_shares", ptr(tc), ptr(ts), M, H, d, pos)
        for m in range(M):
            assert np.array_equal(tc[m].cpu().numpy(), orc.rope_apply(xc[m], H, d, cos_t[pos + m], sin_t[pos + m]))
            assert np.array_equal(ts[m].cpu().numpy(), orc.rope_apply(xs[m], H, d, cos_t[pos + m], sin_t[pos + m]))


def test_rope_position_limit_raises(ctx):
    from shardlm_b200._lib import ShdError
    from shardlm_b200.runtime import ptr

    ctx.call("shd_rope_init", 128, 64, 1e6)
    t = ctx.empty(128)
    with pytest.raises(ShdError, match="max_seq"):
        ctx.call("shd_rope_shares", ptr(t), ptr(t), 1, 1, 128, 64)


@pytest.mark.parametrize("variant", [0, 2])
@pytest.mark.parametrize("H,Hkv,kv_len", [(28, 4, 1), (28, 4, 577), (12, 2, 33), (40, 8, 1200)])
def test_attention_decode(ctx, orc, variant, H, Hkv, kv_len):
    from shardlm_b200.runtime import ptr

    d, T = 128, 2048
    rng = np.random.default_rng(H * kv_len + variant)
    q = rng.standard_normal((2, H * d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    pos = np.array([kv_len - 1, max(0, kv_len // 2 - 1)], np.int32)
    mask = rng.uniform(-1, 1, (2, H * d)).astype(np.float32) if variant == 2 else None
    oc, os_ = ctx.empty(2, H * d), ctx.empty(2, H * d)
    for m in range(2):
        ctx.call("shd_attn_decode", ptr(_dev(ctx, q[m])), ptr(_dev(ctx, k)), ptr(_dev(ctx, v)), T, H, Hkv, d,
                 pos[m:m + 1].ctypes.data, 1, variant, None if mask is None else ptr(_dev(ctx, mask[m])),
                 ptr(oc[m]), ptr(os_[m]))
    ctx.sync()
    for m in range(2):
        L = int(pos[m]) + 1
        rc, rs = orc.attention(q[m], k[:L], v[:L], H, Hkv, d, variant, None if mask is None else mask[m])
        assert np.array_equal(os_[m].cpu().numpy(), rs)
        err = np.max(np.abs(oc[m].cpu().numpy() - rc))
        # split softmax + reassociated dot products: 2e-5 of the value scale
        assert err <= 2e-5 * max(1.0, np.max(np.abs(rc))), err


@pytest.mark.parametrize("M", [1, 3, 8, 9])
@pytest.mark.parametrize("H,Hkv,d", [(28, 4, 128), (14, 2, 64), (40, 8, 128), (4, 1, 128)])
def test_attention_decode_rows(ctx, orc, M, H, Hkv, d):
    """Several query rows in one launch, each with its own position (0 to the cache's end): the
    8-CTA cluster of a row and head group splits the row's positions, so short rows leave CTAs
    without positions, and the combine must weigh them out. From 4 rows each kv head's query heads
    form one group (the 8-head kernel, here with groups of 7 and of 5); 4 query heads on 1 kv
    head is a tensor-parallel rank's slice. A second launch must repeat the first bit for bit."""
    from shardlm_b200.runtime import ptr

    T = 2048
    rng = np.random.default_rng(M * 31 + d)
    q = rng.standard_normal((M, H * d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    pos = np.array([(T - 1, 0, 63, 64, 65, 700, 1500, 128, 2000)[i] for i in range(M)], np.int32)
    oc, os_ = ctx.empty(M, H * d), ctx.empty(M, H * d)
    for rep in range(2):
        ctx.call("shd_attn_decode", ptr(_dev(ctx, q)), ptr(_dev(ctx, k)), ptr(_dev(ctx, v)), T, H, Hkv, d,
                 pos.ctypes.data, M, 0, None, ptr(oc), ptr(os_))
        ctx.sync()
        got = oc.cpu().numpy()
        for m in range(M):
            L = int(pos[m]) + 1
            rc, _ = orc.attention(q[m], k[:L], v[:L], H, Hkv, d, 0, None)
            err = np.max(np.abs(got[m] - rc))
            assert err <= 2e-5 * max(1.0, np.max(np.abs(rc))), (rep, m, err)
        if rep == 0:
            first = got.copy()
        else:
            assert np.array_equal(first, got)


@pytest.mark.parametrize("variant", [0, 2])
@pytest.mark.parametrize("H,Hkv,pos0,M", [(28, 4, 0, 512), (28, 4, 384, 128), (12, 2, 33, 100), (40, 8, 0, 2048),
                                          (4, 1, 7, 17)])
def test_attention_prefill_tensor_cores(ctx, orc, variant, H, Hkv, pos0, M):
    """shd_attn_prefill (tcgen05 flash attention over a prompt block) vs the oracle's
    secure_attention_approx / compute_mpc_attention_on_shares row by row: rows m are positions
    pos0 + m attending to [0, pos0 + m]. Ragged blocks (M % 128 != 0), a block after earlier
    positions, a 2048-position prompt, a tensor-parallel slice (4 q heads on 1 kv head); with MPC
    masks the server share is the mask. A second launch repeats the first bit for bit."""
    from shardlm_b200.runtime import ptr

    d = 128
    T = pos0 + M + 5
    rng = np.random.default_rng(H * M + pos0 + variant)
    q = rng.standard_normal((M, H * d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv * d)).astype(np.float32)
    mask = rng.uniform(-1, 1, (M, H * d)).astype(np.float32) if variant == 2 else None
    oc, os_ = ctx.empty(M, H * d), ctx.empty(M, H * d)
    qd, kd, vd = _dev(ctx, q), _dev(ctx, k), _dev(ctx, v)
    md = None if mask is None else _dev(ctx, mask)
    outs = []
    for rep in range(2):
        ctx.call("shd_attn_prefill", ptr(qd), ptr(kd), ptr(vd), T, H, Hkv, d, pos0, M, variant,
                 None if md is None else ptr(md), ptr(oc), ptr(os_))
        ctx.sync()
        outs.append((oc.cpu().numpy().copy(), os_.cpu().numpy().copy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    got_c, got_s = outs[0]
    rows = sorted(set(list(range(0, M, max(1, M // 24))) + [M - 1, min(M - 1, 127), min(M - 1, 128)]))
    for m in rows:
        L = pos0 + m + 1
        rc, rs = orc.attention(q[m], k[:L], v[:L], H, Hkv, d, variant, None if mask is None else mask[m])
        assert np.array_equal(got_s[m], rs)
        err = np.max(np.abs(got_c[m] - rc))
        # f32-accurate products (three-term bf16 split), reassociated sums: 2e-5 of the value scale
        assert err <= 2e-5 * max(1.0, np.max(np.abs(rc))), (m, err)


def test_embed_shares_bit_exact(ctx, orc):
    from shardlm_b200.runtime import ptr

    V, h = 1000, 1536
    rng = np.random.default_rng(1)
    table = torch.randn(V, h, device="cuda").to(torch.bfloat16)
    toks = np.array([0, 999, 17, 17], np.int32)
    hc, hs = ctx.empty(4, h), ctx.empty(4, h)
    counter = (3 << 32) + 100
    _call(ctx, "shd_embed_shares", ptr(table), V, h, ptr(_dev(ctx, toks, np.int32)), 4, 77, counter, ptr(hc), ptr(hs))
    tab = table.view(torch.int16).cpu().numpy().view(np.uint16)
    for m in range(4):
        ec, es = orc.embed_shares(tab, h, toks[m], 77, counter + m)
        assert np.array_equal(hc[m].cpu().numpy(), ec) and np.array_equal(hs[m].cpu().numpy(), es)
        assert np.all((hs[m] >= 0).cpu().numpy()) and np.all((hs[m] < 1).cpu().numpy())
    bad = ctx.to_device(np.array([1000], np.int32))
    ctx.call("shd_embed_shares", ptr(table), V, h, ptr(bad), 1, 77, 0, ptr(hc), ptr(hs))
    from shardlm_b200._lib import ShdError
    with pytest.raises(ShdError):
        ctx.sync()


def test_argmax_last_index_on_ties(ctx, orc):
    from shardlm_b200.runtime import ptr

    V = 152064
    rng = np.random.default_rng(2)
    lc = rng.standard_normal((3, V)).astype(np.float32)
    ls = np.zeros((3, V), np.float32)
    lc[1, [5, 70000, 152063]] = 100.0  # ties: the last index wins
    lc[2, :] = 1.0
    out = ctx.empty(3, dtype=torch.int32)
    _call(ctx, "shd_argmax_reconstruct", ptr(_dev(ctx, lc)), ptr(_dev(ctx, ls)), V, 3, ptr(out))
    got = out.cpu().numpy().tolist()
    assert got == [orc.argmax_last(lc[i], ls[i]) for i in range(3)]
    assert got[1] == 152063 and got[2] == V - 1
