"""Beaver multiply (f32 and Z_2^32), triple/mask generators vs the oracle: bit-exact.

The f32 kernel keeps the reference's operation order without FMA contraction, so every output
element equals the oracle's restatement of beaver.rs:167-197 exactly.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N4 = 512 * 18944  # 9,699,328 elements


def test_triples_and_masks_bit_exact(ctx, orc):
    from shardlm_b200.sharing import beaver_triples_f32, beaver_triples_ring, fill_uniform

    t = beaver_triples_f32(ctx, 1001, seed=9, offset=17)
    ref = orc.triples_f32(9, 17, 1001)
    for got, want in zip([t.a, t.b, t.c, t.a_client, t.a_server, t.b_client, t.b_server, t.c_client, t.c_server], ref):
        assert np.array_equal(got.cpu().numpy(), want)
    r = beaver_triples_ring(ctx, 1001, seed=9, offset=17)
    for got, want in zip(r, orc.triples_ring(9, 17, 1001)):
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want)
    u = fill_uniform(ctx, 4097, seed=3, lo=-1.0, hi=1.0, offset=5)
    assert np.array_equal(u.cpu().numpy(), orc.fill_uniform(3, 5, -1.0, 1.0, 4097))


@pytest.mark.parametrize("n", [1, 7, 4096 + 3, N4])
def test_beaver_f32_bit_exact(ctx, orc, n):
    from shardlm_b200.sharing import beaver_triples_f32, secure_multiply_batch

    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(n, device="cuda", generator=g)
    y = torch.randn(n, device="cuda", generator=g)
    xs = torch.rand(n, device="cuda", generator=g) * 20 - 10
    ys = torch.rand(n, device="cuda", generator=g) * 20 - 10
    xc, yc = x - xs, y - ys
    t = beaver_triples_f32(ctx, n, seed=1)
    (zc, zs), (d, e) = secure_multiply_batch(ctx, xc, xs, yc, ys, t, return_opened=True)
    ctx.sync()
    if n <= 4096 + 3:
        h = lambda v: v.cpu().numpy()
        ozc, ozs, od, oe = orc.beaver_f32(h(xc), h(xs), h(yc), h(ys), h(t.a_client), h(t.a_server),
                                          h(t.b_client), h(t.b_server), h(t.c_client), h(t.c_server))
        assert np.array_equal(h(zc), ozc) and np.array_equal(h(zs), ozs)
        assert np.array_equal(h(d), od) and np.array_equal(h(e), oe)
    else:
        # full config-4 size: compare a strided sample against the oracle, all elements vs x*y
        idx = torch.arange(0, n, 9973, device="cuda")
        h = lambda v: v[idx].cpu().numpy()
        ozc, ozs, _, _ = orc.beaver_f32(h(xc), h(xs), h(yc), h(ys), h(t.a_client), h(t.a_server),
                                        h(t.b_client), h(t.b_server), h(t.c_client), h(t.c_server))
        assert np.array_equal(h(zc), ozc) and np.array_equal(h(zs), ozs)
    err = ((zc + zs) - (xc + xs) * (yc + ys)).abs().max().item()
    assert err < 1e-3


@pytest.mark.parametrize("n", [5, N4])
def test_beaver_ring_exact_product(ctx, orc, n):
    """Z_2^32: z_c + z_s == x*y mod 2^32 for every element; shares equal the oracle's."""
    from shardlm_b200.sharing import beaver_mul_ring, beaver_triples_ring

    g = torch.Generator(device="cuda").manual_seed(n)
    rnd = lambda: torch.randint(-2**31, 2**31 - 1, (n,), device="cuda", dtype=torch.int64, generator=g).to(torch.int32)
    x, y = (torch.randn(n, device="cuda", generator=g) * 65536).round().to(torch.int32), (torch.randn(n, device="cuda", generator=g) * 65536).round().to(torch.int32)
    xs, ys = rnd(), rnd()
    xc = (x.to(torch.int64) - xs).to(torch.int32)
    yc = (y.to(torch.int64) - ys).to(torch.int32)
    ac, as_, bc, bs, cc, cs = beaver_triples_ring(ctx, n, seed=2)
    (zc, zs), (d, e) = beaver_mul_ring(ctx, xc, xs, yc, ys, ac, as_, bc, bs, cc, cs, return_opened=True)
    ctx.sync()
    z = (zc.to(torch.int64) + zs.to(torch.int64)) & 0xFFFFFFFF
    want = (x.to(torch.int64) * y.to(torch.int64)) & 0xFFFFFFFF
    assert torch.equal(z, want)
    m = min(n, 100000)
    h = lambda v: v[:m].cpu().numpy().view(np.uint32)
    ozc, ozs, od, oe = orc.beaver_ring(h(xc), h(xs), h(yc), h(ys), h(ac), h(as_), h(bc), h(bs), h(cc), h(cs))
    assert np.array_equal(h(zc), ozc) and np.array_equal(h(zs), ozs)
    assert np.array_equal(h(d), od) and np.array_equal(h(e), oe)


def test_beaver_ring_truncation_matches_oracle(ctx, orc):
    from shardlm_b200.sharing import beaver_mul_ring, beaver_triples_ring

    n = 100003
    g = torch.Generator(device="cuda").manual_seed(4)
    x = (torch.randn(n, device="cuda", generator=g) * 65536).round().to(torch.int32)
    y = (torch.randn(n, device="cuda", generator=g) * 65536).round().to(torch.int32)
    xs = torch.randint(-2**31, 2**31 - 1, (n,), device="cuda", dtype=torch.int64, generator=g).to(torch.int32)
    ys = torch.randint(-2**31, 2**31 - 1, (n,), device="cuda", dtype=torch.int64, generator=g).to(torch.int32)
    xc, yc = (x.to(torch.int64) - xs).to(torch.int32), (y.to(torch.int64) - ys).to(torch.int32)
    tr = beaver_triples_ring(ctx, n, seed=5)
    zc, zs = beaver_mul_ring(ctx, xc, xs, yc, ys, *tr, trunc_shift=16)
    h = lambda v: v.cpu().numpy().view(np.uint32)
    ozc, ozs, _, _ = orc.beaver_ring(h(xc), h(xs), h(yc), h(ys), *[h(v) for v in tr], trunc_shift=16)
    assert np.array_equal(h(zc), ozc) and np.array_equal(h(zs), ozs)


def test_scalar_secure_multiply_mpc(ctx):
    from shardlm_b200.sharing import beaver_triples_f32, secure_multiply_mpc

    t = beaver_triples_f32(ctx, 100, seed=11)
    rng = np.random.default_rng(1)
    for i in range(100):
        x, y = rng.uniform(-10, 10, 2).astype(np.float32)
        xs_, ys_ = rng.uniform(-10, 10, 2).astype(np.float32)
        zc, zs = secure_multiply_mpc(ctx, float(np.float32(x - xs_)), float(xs_), float(np.float32(y - ys_)), float(ys_), t, i)
        assert abs((zc + zs) - float(x) * float(y)) < 1e-4
