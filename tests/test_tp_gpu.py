"""Tensor parallelism on 2 GPUs (skipped with fewer): every rank holds its slice of a model
(heads, intermediate blocks and vocabulary rows from shd_tp_plan), the library all-reduces the
packed [2][M][h] partial shares after o and down and max-reduces the argmax keys over NCCL.

Checked against the oracle of the full model on identical weights and shares: greedy tokens of
prefill + decode (teacher-forced on the GPU's choice) and the logits of forward_host, whose full
vocabulary is gathered on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
STEPS = 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shape():
    from shardlm_b200.model import QWEN2_5_1_5B

    # 12 query heads, 2 kv heads: the split gives each rank 6 heads of one kv head
    return QWEN2_5_1_5B.replace(name="tp-test", n_layers=2, vocab=4096)


def _rank(rank: int, port: int, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD))
        from datetime import timedelta

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        from shardlm_b200.model import SecureModel
        from shardlm_b200.runtime import Context
        from shardlm_b200.tp import init_tensor_parallel

        ctx = Context(rank)
        init_tensor_parallel(ctx, rank, WORLD)
        from shardlm_b200._lib import check, lib as _l

        # the all-reduce itself: a decode-sized message (peer path when set up) and a prefill-sized
        # one (NCCL); every rank must hold the same sums, equal to the rank-order sum
        sums = []
        for n in (2 * 1536, 2 * 128 * 1536):
            parts = [torch.randn(n, generator=torch.Generator().manual_seed(100 + r)) for r in range(WORLD)]
            buf = parts[rank].cuda()
            ctx.bind_stream()
            check(_l().shd_allreduce_shares(ctx.ptr, buf.data_ptr(), n, 60000), ctx.ptr)
            want = parts[0].clone()
            for r in range(1, WORLD):
                want = want + parts[r]
            sums.append((buf.cpu(), want))
        peer = int(_l().shd_tp_peer_path(ctx.ptr))
        m = SecureModel(ctx, _shape(), max_seq=64, share_seed=321, tp_rank=rank, tp_world=WORLD)
        m.load_random_weights(seed=11)
        prompt = np.arange(9, dtype=np.int32) * 37 % _shape().vocab
        first = m.prefill(prompt)
        toks = m.decode(STEPS)[:, 0]
        rng = np.random.default_rng(3)
        h = _shape().hidden
        x = rng.standard_normal(h).astype(np.float32)
        hs = rng.uniform(0, 1, h).astype(np.float32)
        lc, ls = m.forward_host((x - hs).astype(np.float32), hs)
        q.put((rank, int(first), toks.tolist(), lc.copy(), ls.copy(), peer,
               [(a.numpy(), b.numpy()) for a, b in sums]))
        m.close()
        from shardlm_b200._lib import lib

        lib().shd_tp_destroy(ctx.ptr)
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        import traceback

        q.put((rank, "error", f"{e!r}\n{traceback.format_exc()}", None, None, None, None))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_tp2_tokens_and_logits_match_oracle(orc):
    from test_model import LOGIT_RTOL, _check_token, _oracle_for

    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    peers, sums = {}, {}
    for _ in range(WORLD):
        r, first, toks, lc, ls, peer, sm = q.get(timeout=300)
        assert first != "error", toks
        out[r] = (first, toks, lc, ls)
        peers[r], sums[r] = peer, sm
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # all-reduce: identical on every rank and equal to the rank-order sum (both paths); on NVSwitch
    # nodes the peer-memory path must have been set up
    assert peers[0] == peers[1] == 1
    for i in range(2):
        assert np.array_equal(sums[0][i][0], sums[1][i][0])
        np.testing.assert_allclose(sums[0][i][0], sums[0][i][1], rtol=1e-6, atol=1e-6)
    # every rank returns the same tokens and the same gathered logits
    assert out[0][0] == out[1][0] and out[0][1] == out[1][1]
    assert np.array_equal(out[0][2], out[1][2]) and np.array_equal(out[0][3], out[1][3])

    # the oracle of the full model with the same random-init weights (regenerated on one GPU)
    from shardlm_b200.model import SecureModel
    from shardlm_b200.runtime import Context

    ctx = Context(0)
    shape = _shape()
    ref = SecureModel(ctx, shape, max_seq=64, share_seed=321)
    host = ref.load_random_weights(seed=11, host_copy=True)
    ref.close()
    om = _oracle_for(orc, shape, host, 64)
    prompt = np.arange(9, dtype=np.int32) * 37 % shape.vocab
    for p, t in enumerate(prompt):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 321, p)
        _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
    first, toks, glc, gls = out[0]
    _check_token(first, lc, ls, orc)
    inp = first
    for i in range(STEPS):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 321, len(prompt) + i)
        _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
        _check_token(int(toks[i]), lc, ls, orc)
        inp = int(toks[i])
    rng = np.random.default_rng(3)
    x = rng.standard_normal(shape.hidden).astype(np.float32)
    hs = rng.uniform(0, 1, shape.hidden).astype(np.float32)
    _, _, oc, os_ = om.forward((x - hs).astype(np.float32), hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
    err = np.max(np.abs((glc + gls) - (oc + os_))) / np.max(np.abs(oc + os_))
    assert err < LOGIT_RTOL, err
