"""Host side of tensor parallelism, on the CPU: the shard plan (shd_tp_plan) and world-size-2 gloo
runs of the exchange steps around it.

The plan must cover every query head, intermediate row and vocab row exactly once and give each rank
the kv heads its query heads read. The gloo ranks then check the algebra the NCCL path relies on:
row-parallel partial shares (o and down projections) summed across ranks equal the one-GPU shares,
and the per-rank argmax keys reduced by max give the global last-index argmax. The oracle computes
every rank's slice; the plan and the unique-id exchange are the package's own code.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import bf16_round, f32_sum_tolerance


def _shapes():
    from shardlm_b200.model import QWEN2_5_1_5B, QWEN2_5_7B, QWEN2_5_14B, TINY

    return [QWEN2_5_1_5B, QWEN2_5_7B, QWEN2_5_14B, TINY]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_partitions_every_dimension(world):
    from shardlm_b200.tp import tp_plan

    for sh in _shapes():
        if world > sh.n_heads:
            continue
        plans = [tp_plan(sh, r, world) for r in range(world)]
        group = sh.n_heads // sh.n_kv_heads
        q = [h for p in plans for h in p.q_heads]
        assert q == list(range(sh.n_heads)), (sh.name, world)
        inter = [i for p in plans for i in p.inter]
        assert inter == list(range(sh.intermediate)), (sh.name, world)
        assert all(p.inter.start % 16 == 0 for p in plans)
        vocab = [v for p in plans for v in p.vocab]
        assert vocab == list(range(sh.vocab)), (sh.name, world)
        for p in plans:
            need = sorted({h // group for h in p.q_heads})
            assert list(p.kv_heads) == need, (sh.name, world, p.rank)
        # balanced: query heads differ by at most one between ranks
        counts = [len(p.q_heads) for p in plans]
        assert max(counts) - min(counts) <= 1


def test_plan_rejects_impossible_splits():
    from shardlm_b200._lib import SHD_ERR_ARG, ShdError
    from shardlm_b200.model import TINY
    from shardlm_b200.tp import tp_plan

    with pytest.raises(ShdError) as e:
        tp_plan(TINY, 0, TINY.n_heads + 1)
    assert e.value.code == SHD_ERR_ARG
    with pytest.raises(ShdError):
        tp_plan(TINY, 2, 2)
    with pytest.raises(ShdError):
        tp_plan(TINY.replace(intermediate=520), 0, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SHAPE = dict(hidden=256, n_heads=6, n_kv_heads=2, head_dim=32, intermediate=512, vocab=1000)


def _worker(rank: int, world: int, port: int, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import oracle as orc
        from shardlm_b200.model import TINY
        from shardlm_b200.tp import share_unique_id, tp_plan

        sh = TINY.replace(name="tp-test", **SHAPE)
        plan = tp_plan(sh, rank, world)

        # unique-id exchange: every rank ends with rank 0's bytes
        uid = share_unique_id(rank, "cpu", make_id=lambda: bytes(range(128)))
        ids = [None] * world
        dist.all_gather_object(ids, uid)
        assert all(i == bytes(range(128)) for i in ids)

        rng = np.random.default_rng(7)  # same inputs on every rank
        h, d, I, V = sh.hidden, sh.head_dim, sh.intermediate, sh.vocab
        qd = sh.n_heads * d

        def row_parallel(K, cols):
            w = bf16_round((rng.standard_normal((K, h)) * 0.05).astype(np.float32))  # [in][out]
            xs = rng.uniform(0, 1, K).astype(np.float32)
            xc = (rng.standard_normal(K).astype(np.float32) - xs).astype(np.float32)
            bias = (rng.standard_normal(h) * 0.05).astype(np.float32)
            full_c, full_s = orc.linear_bf16(w, bias, xc, xs)
            # bias belongs to one rank only (rank 0), as the library adds it once
            pc, ps = orc.linear_bf16(np.ascontiguousarray(w[cols]), bias if rank == 0 else np.zeros_like(bias),
                                     np.ascontiguousarray(xc[cols]), np.ascontiguousarray(xs[cols]))
            packed = torch.from_numpy(np.stack([pc, ps]).astype(np.float32))
            dist.all_reduce(packed)
            tol_c = f32_sum_tolerance(K, orc.linear_abs_bf16(w, xc)) * world
            tol_s = f32_sum_tolerance(K, orc.linear_abs_bf16(w, xs)) * world + np.abs(bias) * 2.0 ** -22
            assert np.all(np.abs(packed[0].numpy() - full_c) <= tol_c)
            assert np.all(np.abs(packed[1].numpy() - full_s) <= tol_s)

        q_cols = np.arange(plan.q_heads.start * d, plan.q_heads.stop * d)
        row_parallel(qd, q_cols)                                     # o projection
        row_parallel(I, np.arange(plan.inter.start, plan.inter.stop))  # down projection

        # lm_head by vocab rows: local last-index argmax, then max over (value, index) keys
        lc = rng.standard_normal(V).astype(np.float32)
        ls = rng.standard_normal(V).astype(np.float32)
        lc[[3, 900]] = 50.0  # a tie across the two ranks' slices: the last index wins
        ls[[3, 900]] = 0.0
        sl = slice(plan.vocab.start, plan.vocab.stop)
        local = orc.argmax_last(lc[sl], ls[sl]) + plan.vocab.start
        val = float(lc[local] + ls[local])
        keys = [None] * world
        dist.all_gather_object(keys, (val, local))
        best = max(keys)
        assert best[1] == orc.argmax_last(lc, ls) == 900
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent; the process exits normally
        import traceback

        errq.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")


def test_gloo_world2_row_parallel_and_argmax():
    from shardlm_b200._lib import lib

    lib()  # build once here, not in both ranks
    world = 2
    ctxmp = mp.get_context("spawn")
    errq = ctxmp.Queue()
    port = _free_port()
    procs = [ctxmp.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a gloo rank did not finish"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)


def _leaver(rank: int, world: int, port: int, errq):
    """Rank 1 leaves before the unique-id exchange; rank 0 must get an error, not wait forever."""
    from datetime import timedelta

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        if rank == 1:
            return  # leaves between steps, with nothing in flight
        from shardlm_b200.tp import share_unique_id

        try:
            share_unique_id(rank, "cpu", make_id=lambda: bytes(128))
        except Exception as e:  # the expected outcome
            errq.put(("raised", type(e).__name__))
            return
        errq.put(("no error", ""))
    except Exception as e:
        errq.put(("setup", repr(e)))


def test_gloo_rank_leaving_surfaces_as_error():
    from shardlm_b200._lib import lib

    lib()
    ctxmp = mp.get_context("spawn")
    errq = ctxmp.Queue()
    port = _free_port()
    procs = [ctxmp.Process(target=_leaver, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    outcome = errq.get(timeout=5)
    assert outcome[0] == "raised", outcome
