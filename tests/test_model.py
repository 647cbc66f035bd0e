"""Whole-model secret-shared forward pass (libshardlm_cuda layer loop) vs the oracle's restatement of
the reference layer loop on identical weights and shares.

Token ids: the greedy token at every step must equal the oracle's, except where the oracle's top-2
logit margin is below the float tolerance (then either index is a correct greedy choice of
numerically equal logits). Logits: relative to the logit scale, within LOGIT_RTOL.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 2e-4


def _oracle_for(orc, shape, host, max_seq):
    om = orc.Model(shape.hidden, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.head_dim,
                   shape.intermediate, shape.vocab, shape.rope_theta, shape.rms_eps, max_seq)
    for l, w in enumerate(host["layers"]):
        om.set_layer(l, w["wq"], w["wk"], w["wv"], w["wo"], w["wg"], w["wu"], w["wd"], w["bq"], w["bk"], w["bv"], w["g1"], w["g2"])
    om.set_head(host["lm_head_in_out"], host["final_norm"])
    return om


def _oracle_step(orc, om, host, shape, token, pos, seed, variant, slot=0):
    hc, hs = orc.embed_shares(host["embed"], shape.hidden, token, seed, (slot << 32) + pos)
    return om.forward(hc, hs, variant=variant, attn_variant=orc.NL_APPROX)


def _top2_margin(l):
    s = np.sort(l.astype(np.float64))
    return s[-1] - s[-2]


def _check_token(gpu_tok, lc, ls, orc):
    l = lc + ls
    want = orc.argmax_last(lc, ls)
    if gpu_tok != want:
        margin = abs(float(l[gpu_tok]) - float(l[want]))
        assert margin <= LOGIT_RTOL * np.max(np.abs(l)), f"token {gpu_tok} vs oracle {want}, margin {margin}"
        return False
    return True


@pytest.mark.parametrize("shape_name,n_layers,prompt,steps,max_seq",
                         [("tiny", 2, 11, 12, 64), ("qwen2.5-1.5b", 2, 9, 6, 64), ("tiny", 1, 2450, 3, 2460)])
def test_prefill_decode_tokens_match_oracle(ctx, orc, shape_name, n_layers, prompt, steps, max_seq):
    """Prefill then greedy decode; the long prompt gives the attention kernel many K/V tiles per
    cluster CTA."""
    from shardlm_b200.model import SHAPES, SecureModel

    shape = SHAPES[shape_name].replace(n_layers=n_layers)
    m = SecureModel(ctx, shape, max_seq=max_seq, share_seed=123)
    host = m.load_random_weights(seed=5, host_copy=True)
    om = _oracle_for(orc, shape, host, max_seq)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, shape.vocab, prompt).astype(np.int32)
    nxt = m.prefill(toks)
    for p, t in enumerate(toks):
        _, _, lc, ls = _oracle_step(orc, om, host, shape, int(t), p, 123, orc.NL_GPU)
    _check_token(nxt, lc, ls, orc)
    gpu = m.decode(steps)[:, 0]
    inp = nxt
    exact = 0
    for i in range(steps):
        _, _, lc, ls = _oracle_step(orc, om, host, shape, int(inp), prompt + i, 123, orc.NL_APPROX)
        exact += _check_token(int(gpu[i]), lc, ls, orc)
        inp = int(gpu[i])  # teacher-force the GPU's choice so one near-tie cannot cascade
    assert exact >= steps - 1
    assert m.seq_len() == prompt + steps


@pytest.mark.parametrize("variant", ["v3", "mpc"])
def test_long_prompt_tensor_core_attention(ctx, orc, variant):
    """A 700-token prompt through a one-layer 7B-shaped model: every 128-position block's attention
    runs on the tensor cores (flash prefill), the last block ragged; the next token and three decode
    steps are checked against the oracle (V3-MPC: with reshare masks)."""
    from shardlm_b200._lib import NL_MPC
    from shardlm_b200.model import QWEN2_5_7B, SecureModel
    from shardlm_b200.sharing import beaver_triples_f32

    orc.set_threads(orc.max_threads())
    shape = QWEN2_5_7B.replace(n_layers=1, vocab=4096)
    prompt, steps, max_seq = 700, 3, 712
    mpc = variant == "mpc"
    kw = dict(variant_decode=NL_MPC, variant_prefill=NL_MPC, variant_attn=NL_MPC) if mpc else {}
    m = SecureModel(ctx, shape, max_seq=max_seq, share_seed=31, **kw)
    host = m.load_random_weights(seed=17, host_copy=True)
    masks = None
    if mpc:
        P = 10 * shape.hidden + 20 + 5 * 32
        a = torch.stack([beaver_triples_f32(ctx, P, seed=4, offset=l * P).a for l in range(shape.n_layers)])
        m.set_masks(a)
        masks = a.cpu().numpy()
    om = _oracle_for(orc, shape, host, max_seq)
    toks = np.random.default_rng(3).integers(0, shape.vocab, prompt).astype(np.int32)
    nxt = m.prefill(toks)
    pv = orc.NL_MPC if mpc else orc.NL_GPU
    av = orc.NL_MPC if mpc else orc.NL_APPROX
    for p, t in enumerate(toks):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 31, p)
        _, _, lc, ls = om.forward(hc, hs, variant=pv, attn_variant=av, masks=masks)
    exact = int(_check_token(nxt, lc, ls, orc))
    gpu = m.decode(steps)[:, 0]
    inp = nxt
    for i in range(steps):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 31, prompt + i)
        _, _, lc, ls = om.forward(hc, hs, variant=av, attn_variant=av, masks=masks)
        exact += _check_token(int(gpu[i]), lc, ls, orc)
        inp = int(gpu[i])
    assert exact >= steps
    m.close()


def test_forward_host_logits_match_oracle(ctx, orc):
    """generate_token_gpu semantics: hidden shares in, logit shares out, position by position."""
    from shardlm_b200.model import TINY, SecureModel

    shape = TINY
    m = SecureModel(ctx, shape, max_seq=32)
    host = m.load_random_weights(seed=9, host_copy=True)
    om = _oracle_for(orc, shape, host, 32)
    rng = np.random.default_rng(4)
    for p in range(6):
        x = rng.standard_normal(shape.hidden).astype(np.float32)
        hs = rng.uniform(0, 1, shape.hidden).astype(np.float32)
        hc = (x - hs).astype(np.float32)
        lc, ls = m.forward_host(hc, hs)
        _, _, oc, os_ = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
        ref = oc + os_
        got = lc + ls
        err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
        assert err < LOGIT_RTOL, (p, err)
        # V3 reshares the final norm as (y, 0): the server logit share is exactly zero
        assert np.all(ls == 0) and np.all(os_ == 0)
    assert m.seq_len() == 6


def test_mpc_masks_reshare(ctx, orc):
    """V3-MPC masks: reshares become (y - a, a) with the triple store's a values."""
    from shardlm_b200._lib import NL_MPC
    from shardlm_b200.model import TINY, SecureModel
    from shardlm_b200.sharing import beaver_triples_f32

    shape = TINY
    m = SecureModel(ctx, shape, max_seq=32, variant_decode=NL_MPC, variant_prefill=NL_MPC, variant_attn=NL_MPC)
    host = m.load_random_weights(seed=2, host_copy=True)
    P = 10 * shape.hidden + 20 + 5 * 32  # triples_needed_per_layer(hidden, seq)
    a = torch.stack([beaver_triples_f32(ctx, P, seed=3, offset=l * P).a for l in range(shape.n_layers)])
    m.set_masks(a)
    om = _oracle_for(orc, shape, host, 32)
    masks = a.cpu().numpy()
    rng = np.random.default_rng(5)
    for p in range(4):
        x = rng.standard_normal(shape.hidden).astype(np.float32)
        hs = rng.uniform(0, 1, shape.hidden).astype(np.float32)
        hc = (x - hs).astype(np.float32)
        lc, ls = m.forward_host(hc, hs)
        _, _, oc, os_ = om.forward(hc, hs, variant=orc.NL_MPC, attn_variant=orc.NL_MPC, masks=masks)
        err = np.max(np.abs((lc + ls) - (oc + os_))) / np.max(np.abs(oc + os_))
        assert err < LOGIT_RTOL, err
        # with masks, the server logit share is no longer zero
        assert np.max(np.abs(ls)) > 0


@pytest.mark.parametrize("variant,slots", [("approx", 3), ("mpc", 3), ("approx", 6)])
def test_batched_decode_agrees_with_oracle(ctx, orc, variant, slots):
    """Slots decoded together (M rows per step), each checked against the oracle slot by slot
    (teacher-forced on the GPU's tokens). With 6 rows the layer linears run on the tensor cores."""
    from shardlm_b200._lib import NL_APPROX, NL_GPU, NL_MPC
    from shardlm_b200.model import TINY, SecureModel
    from shardlm_b200.sharing import beaver_triples_f32

    shape = TINY.replace(n_layers=2)
    nl = NL_MPC if variant == "mpc" else NL_APPROX
    nl_pre = NL_MPC if variant == "mpc" else NL_GPU
    prompts = [np.array(p, np.int32) for p in ([5, 17, 300], [9, 2, 44, 11, 7], [999], [1, 2], [640, 3, 3, 8],
                                               [77, 78, 79, 80, 81, 82])][:slots]
    steps = 5
    m = SecureModel(ctx, shape, max_seq=32, max_batch=slots, share_seed=77, variant_decode=nl,
                    variant_prefill=nl_pre, variant_attn=nl)
    host = m.load_random_weights(seed=12, host_copy=True)
    masks = None
    if variant == "mpc":
        P = 10 * shape.hidden + 20 + 5 * 32
        a = torch.stack([beaver_triples_f32(ctx, P, seed=8, offset=l * P).a for l in range(shape.n_layers)])
        m.set_masks(a)
        masks = a.cpu().numpy()
    first = [m.prefill(p, slot=b) for b, p in enumerate(prompts)]
    toks = m.decode(steps, n_active=slots)
    om = [_oracle_for(orc, shape, host, 32) for _ in prompts]
    exact = 0
    for b, p in enumerate(prompts):
        for i, t in enumerate(p):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 77, (b << 32) + i)
            om[b].forward(hc, hs, variant=nl_pre, attn_variant=nl, masks=masks)
        inp = first[b]
        for i in range(steps):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 77, (b << 32) + len(p) + i)
            _, _, lc, ls = om[b].forward(hc, hs, variant=nl, attn_variant=nl, masks=masks)
            exact += _check_token(int(toks[i, b]), lc, ls, orc)
            inp = int(toks[i, b])
    assert exact >= slots * steps - 1


def test_batched_decode_tensor_core_rows(ctx, orc):
    """Three slots of a 7B-shaped layer: gate/up and down (over 48 M weights) run on the tensor cores
    at 3 rows, q/k/v and o on the CUDA-core GEMV; tokens checked against the oracle."""
    from shardlm_b200.model import QWEN2_5_7B, SecureModel

    shape = QWEN2_5_7B.replace(n_layers=1, vocab=4096)
    prompts = [np.array(p, np.int32) for p in ([5, 17, 300], [9, 2, 44, 11, 7], [999])]
    steps = 4
    m = SecureModel(ctx, shape, max_seq=32, max_batch=3, share_seed=5)
    host = m.load_random_weights(seed=21, host_copy=True)
    first = [m.prefill(p, slot=b) for b, p in enumerate(prompts)]
    toks = m.decode(steps, n_active=3)
    exact = 0
    for b, p in enumerate(prompts):
        om = _oracle_for(orc, shape, host, 32)
        for i, t in enumerate(p):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 5, (b << 32) + i)
            om.forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
        inp = first[b]
        for i in range(steps):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 5, (b << 32) + len(p) + i)
            _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
            exact += _check_token(int(toks[i, b]), lc, ls, orc)
            inp = int(toks[i, b])
    assert exact >= 3 * steps - 1


def test_batched_decode_producers_write_planes(ctx, orc):
    """Eight slots of a 14B-shaped layer: every projection runs on the tensor cores with 8-row
    token tiles, and gate/up (K split in 2 by the launcher) writes the down linear's bf16 planes
    from its reduce kernel, so the down input goes through no split kernel. Tokens checked against
    the oracle."""
    from shardlm_b200.model import QWEN2_5_14B, SecureModel

    shape = QWEN2_5_14B.replace(n_layers=1, vocab=4096)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, shape.vocab, 1 + (b % 3)).astype(np.int32) for b in range(8)]
    steps = 3
    m = SecureModel(ctx, shape, max_seq=16, max_batch=8, share_seed=6)
    host = m.load_random_weights(seed=22, host_copy=True)
    first = [m.prefill(p, slot=b) for b, p in enumerate(prompts)]
    toks = m.decode(steps, n_active=8)
    exact = 0
    for b, p in enumerate(prompts):
        om = _oracle_for(orc, shape, host, 16)
        for i, t in enumerate(p):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 6, (b << 32) + i)
            om.forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
        inp = first[b]
        for i in range(steps):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 6, (b << 32) + len(p) + i)
            _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
            exact += _check_token(int(toks[i, b]), lc, ls, orc)
            inp = int(toks[i, b])
    assert exact >= 8 * steps - 1


def test_model_rejects_bad_requests(ctx):
    from shardlm_b200._lib import ShdError
    from shardlm_b200.model import TINY, SecureModel

    m = SecureModel(ctx, TINY, max_seq=8)
    m.load_random_weights(seed=1)
    with pytest.raises(ShdError, match="empty prompt"):
        m.prefill([])
    with pytest.raises(ShdError, match="out of range"):
        m.prefill([TINY.vocab])
    with pytest.raises(ShdError, match="max_seq"):
        m.prefill(list(range(9)))
    m.prefill([1, 2, 3])
    with pytest.raises(ShdError, match="max_seq"):
        m.decode_async(6)


def test_decode_timeline_stamps_every_launch(ctx):
    """The traced step graph (shd_model_set_profiling(m, 2)) stamps every GEMV and attention launch
    in layer order, with consistent times, and decodes the same tokens as the untraced graph."""
    import ctypes as C

    from shardlm_b200._lib import check, lib
    from shardlm_b200.microbench import timeline_summary
    from shardlm_b200.model import SHAPES, SecureModel

    shape = SHAPES["tiny"].replace(n_layers=3)
    toks = np.random.default_rng(1).integers(0, shape.vocab, 7).astype(np.int32)
    runs = []
    for traced in (False, True):
        m = SecureModel(ctx, shape, max_seq=32, share_seed=9)
        m.load_random_weights(seed=2)
        m.prefill(toks)
        if traced:
            check(lib().shd_model_set_profiling(m.handle, 2), ctx.ptr)
        runs.append(m.decode(5)[:, 0])
        if traced:
            n = C.c_int()
            check(lib().shd_model_timeline(m.handle, 0, None, None, C.byref(n)), ctx.ptr)
            kinds = np.zeros(n.value, np.int32)
            st = np.zeros((n.value, 8), np.uint64)
            check(lib().shd_model_timeline(m.handle, n.value, kinds.ctypes.data, st.ctypes.data, C.byref(n)),
                  ctx.ptr)
        m.close()
    assert np.array_equal(runs[0], runs[1])
    assert kinds.tolist() == [0, 5, 1, 2, 3] * shape.n_layers + [4]
    first = st[:, [0, 2, 4]].astype(np.int64)
    last = (~st[:, [1, 3, 5]]).astype(np.int64)
    assert (first > 0).all() and (last > 0).all()
    assert (last[:, 2] >= first[:, 0]).all() and (last[:, 1] >= first[:, 1]).all()
    assert (np.diff(last[:, 2]) >= 0).all()  # each launch ends after the one before it
    summ = timeline_summary(kinds, st)
    assert set(summ) >= {"qkv", "attention", "o", "gateup", "down", "lm_head"}


@pytest.mark.parametrize("rows", [3, 6])
def test_forward_host_rows_match_oracle(ctx, orc, rows):
    """shd_model_forward_host_rows: sequences prefilled with different prompts advance one position
    each in one pass (rows given in reverse slot order); every row's logit shares match the oracle of
    its own sequence, twice in a row. With 6 rows the linears and the lm_head run on the tensor
    cores."""
    from shardlm_b200.model import TINY, SecureModel

    shape = TINY.replace(n_layers=2)
    prompts = [np.array(p, np.int32) for p in ([5, 17, 300], [9, 2, 44, 11, 7], [999], [1, 2], [640, 3, 3, 8],
                                               [77, 78, 79, 80, 81, 82])][:rows]
    m = SecureModel(ctx, shape, max_seq=32, max_batch=rows, share_seed=5)
    host = m.load_random_weights(seed=21, host_copy=True)
    for b, p in enumerate(prompts):
        m.prefill(p, slot=b)
    om = [_oracle_for(orc, shape, host, 32) for _ in prompts]
    for b, p in enumerate(prompts):
        for i, t in enumerate(p):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 5, (b << 32) + i)
            om[b].forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
    slots = list(reversed(range(rows)))
    rng = np.random.default_rng(rows)
    for _ in range(2):
        x = rng.standard_normal((rows, shape.hidden)).astype(np.float32)
        hs = rng.uniform(0, 1, (rows, shape.hidden)).astype(np.float32)
        hc = (x - hs).astype(np.float32)
        lc, ls = m.forward_host_rows(slots, hc, hs)
        for r, b in enumerate(slots):
            _, _, oc, os_ = om[b].forward(hc[r], hs[r], variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
            ref = oc + os_
            err = np.max(np.abs(lc[r] + ls[r] - ref)) / np.max(np.abs(ref))
            assert err < LOGIT_RTOL, (r, b, err)
    for b, p in enumerate(prompts):
        assert m.seq_len(b) == len(p) + 2
