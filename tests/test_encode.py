"""Device encoding and seeded share generation vs the oracle, bit-exact (integer and bit-pattern
work, no tolerance):

* shd_fixed_from_f64 = FixedVector::from_f64_slice (crates/fixed_point/src/vector.rs:22-29,
  fixed.rs:30-49): round half away from zero, first out-of-range element reported;
* shd_ring_share_seeded = SharePair::from_plaintext_seeded (crates/sharing/src/share.rs:116-135)
  with ChaCha20Rng::seed_from_u64;
* shd_embed_shares_session = get_embeddings_direct (crates/v2/server/src/routes/
  secure_inference.rs:387-460) with ChaCha20Rng::from_seed(session id || 0^16);
* BASELINE config 1 end to end through the product: x ~ N(0,1) encoded on the device, seeded
  shares, LinearServer, against the oracle's LinearServer::multiply_vector.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fixed_from_f64_bit_exact(ctx, orc):
    from shardlm_b200.sharing import fixed_from_f64_slice

    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(100_000) * 3.0,
        # exact ties at scale 16 (k + 0.5) / 2^16: half away from zero
        (np.arange(-50, 50) + 0.5) / 65536.0,
        [0.0, -0.0, np.nan, 1.0 / 131072, -1.0 / 131072, 32767.99998474121, -32768.0,
         2147483647.0 / 65536, -2147483648.0 / 65536],
    ])
    got = fixed_from_f64_slice(ctx, x, 16).cpu().numpy()
    want = np.array([orc.fixed_from_f64(v) if not np.isnan(v) else 0 for v in x], np.int32)
    assert np.array_equal(got, want)
    for scale in (0, 8, 30):
        small = rng.uniform(-1.99, 1.99, 1000)  # |v| < 2 fits i32 at scale 30
        got = fixed_from_f64_slice(ctx, small, scale).cpu().numpy()
        assert np.array_equal(got, np.array([orc.fixed_from_f64(v, scale) for v in small], np.int32))


def test_fixed_from_f64_errors(ctx, orc):
    from shardlm_b200.sharing import FixedPointError, fixed_from_f64_slice

    x = np.zeros(5000)
    x[1234] = 40000.0       # 40000 * 2^16 > i32::MAX
    x[4000] = -50000.0
    with pytest.raises(FixedPointError, match=r"Overflow \{ value: 40000 \} at element 1234"):
        fixed_from_f64_slice(ctx, x, 16)
    x[1234] = 0.0
    with pytest.raises(FixedPointError, match=r"Underflow \{ value: -50000 \} at element 4000"):
        fixed_from_f64_slice(ctx, x, 16)
    with pytest.raises(FixedPointError, match="InvalidScale"):
        fixed_from_f64_slice(ctx, np.zeros(3), 31)
    # the boundary itself: 32768 - 2^-16 fits, 32768 does not
    assert fixed_from_f64_slice(ctx, [32768.0 - 2.0 ** -16], 16).cpu().item() == 2**31 - 1
    with pytest.raises(FixedPointError, match="Overflow"):
        fixed_from_f64_slice(ctx, [32768.0], 16)


@pytest.mark.parametrize("n,seed", [(1536, 12345), (17, 42), (1, 0), (10_000_003, 2**64 - 1)])
def test_ring_share_seeded_bit_exact(ctx, orc, n, seed):
    from shardlm_b200.sharing import random_share_seeded

    x = np.random.default_rng(n).integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    xc, xs = random_share_seeded(ctx, torch.from_numpy(x), seed)
    oc, os_ = orc.ring_share_seeded(x, seed)
    assert np.array_equal(xs.cpu().numpy(), os_)
    assert np.array_equal(xc.cpu().numpy(), oc)


def test_share_pair_reconstructs(ctx):
    from shardlm_b200.sharing import SharePair

    x = np.arange(-500, 500, dtype=np.int32) * 65536
    p = SharePair.from_plaintext_seeded(ctx, x, 16, 999)
    assert np.array_equal(p.reconstruct(), x)
    q = SharePair.from_plaintext_seeded(ctx, x, 16, 999)
    assert np.array_equal(p.server.data, q.server.data)
    assert not np.array_equal(SharePair.from_plaintext_seeded(ctx, x, 16, 1000).server.data, p.server.data)


@pytest.mark.parametrize("hidden,n_tokens", [(3584, 5), (1536, 1), (256, 33)])
def test_embed_shares_session_bit_exact(ctx, orc, hidden, n_tokens):
    from shardlm_b200.sharing import get_embeddings_direct

    vocab = 1000
    table = (torch.randn(vocab, hidden, device="cuda") * 0.02).to(torch.bfloat16)
    tu16 = table.view(torch.int16).cpu().numpy().view(np.uint16)
    tokens = np.random.default_rng(hidden).integers(0, vocab, n_tokens).astype(np.int32)
    sid = bytes(range(16, 32))
    hc, hs = get_embeddings_direct(ctx, table, tokens, sid)
    oc, os_ = orc.embed_shares_chacha(tu16, hidden, tokens, sid + bytes(16))
    assert np.array_equal(hs.cpu().numpy().view(np.uint32), os_.view(np.uint32))
    assert np.array_equal(hc.cpu().numpy().view(np.uint32), oc.view(np.uint32))


def test_embed_shares_session_rejects_out_of_range(ctx):
    from shardlm_b200.sharing import SharingError, get_embeddings_direct

    table = torch.zeros(10, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SharingError, match="Token ID 10 out of range"):
        get_embeddings_direct(ctx, table, [1, 10], bytes(16))


def test_config1_end_to_end_through_product_encoding(ctx, orc):
    """Config 1: W 1536x1536 ~ N(0,0.02) and x ~ N(0,1), both encoded by Fixed::from_f64 on the
    device (spot-checked against the oracle's encoder), server input share from seed 7, the ring
    linear on the GPU; output shares bit-exact with the oracle, reconstruction within 1 LSB of
    plaintext_linear where no input share wrapped."""
    from shardlm_b200.sharing import LinearRequestMsg, LinearServer, Share, fixed_from_f64_slice, random_share_seeded

    rng = np.random.default_rng(1)
    w_f = rng.standard_normal((1536, 1536)) * 0.02
    x_f = rng.standard_normal(1536)
    w = fixed_from_f64_slice(ctx, w_f.reshape(-1), 16).cpu().numpy().reshape(1536, 1536)
    assert np.array_equal(w[:4, :4].reshape(-1), [orc.fixed_from_f64(v) for v in w_f[:4, :4].reshape(-1)])
    x = fixed_from_f64_slice(ctx, x_f, 16)
    xc, xs = random_share_seeded(ctx, x, 7)
    srv = LinearServer(w.reshape(-1), None, 1536, 1536, 16, ctx)
    r = srv.handle_request(LinearRequestMsg(xc.cpu().numpy(), 16), Share(xs.cpu().numpy(), 16))
    x_h = x.cpu().numpy()
    oxc, oxs = orc.ring_share_seeded(x_h, 7)
    oc, os_ = orc.linear_ring(w, None, oxc, oxs, 16)
    assert np.array_equal(r.client_output_share, oc[0]) and np.array_equal(r.server_output_share, os_[0])
    y = (r.client_output_share.astype(np.int64) + r.server_output_share).astype(np.int32)
    p = orc.plaintext_linear_ring(w, None, x_h, 16)
    wrapped = oxc.astype(np.int64) + oxs.astype(np.int64) != x_h.astype(np.int64)
    if not wrapped.any():
        assert np.max(np.abs(y.astype(np.int64) - p)) <= 1
