"""Whole models at the benchmark depths (3 and 5) against the oracle's
restatement of the reference layer loop (crates/v2/server/src/routes/secure_inference.rs:1553-1796
decode, :2299-2632 prefill) on identical weights and shares.

* config 2: Qwen2.5-1.5B shape, all 28 layers, 32 seeded uniform prompt ids, 50 greedy tokens;
* config 3: Qwen2.5-7B shape, all 28 layers (the graph bench.py times), a 16-token prompt and
  8 greedy tokens;
* config 5: Qwen2.5-14B shape, all 48 layers, 8 sequences decoded together (every projection on
  the tensor cores), short prompts and 3 greedy steps.

Token ids are compared at every step (greedy = last index among equal maxima,
crates/v2/client/src/lib.rs:604-640); the oracle is teacher-forced with the GPU's token so one
numerical near-tie cannot cascade, and a differing token is accepted only where the two logits are
within LOGIT_RTOL of the logit scale. Logits of the last position are compared whole through
shd_model_forward_host (generate_token_gpu semantics).
"""
import time

import numpy as np
import pytest

from test_model import LOGIT_RTOL, _check_token, _oracle_for

pytestmark = pytest.mark.gpu


def _all_threads(orc):
    orc.set_threads(orc.max_threads())


def _run_single(ctx, orc, shape_name, prompt_len, steps, seed, share_seed, min_exact):
    from shardlm_b200.model import SHAPES, SecureModel

    _all_threads(orc)
    shape = SHAPES[shape_name]
    max_seq = prompt_len + steps + 4
    m = SecureModel(ctx, shape, max_seq=max_seq, share_seed=share_seed)
    host = m.load_random_weights(seed=seed, host_copy=True)
    om = _oracle_for(orc, shape, host, max_seq)
    rng = np.random.default_rng(0)  # seeded uniform prompt ids
    toks = rng.integers(0, shape.vocab, prompt_len).astype(np.int32)
    t0 = time.perf_counter()
    nxt = m.prefill(toks)
    for p, t in enumerate(toks):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), share_seed, p)
        _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
    exact = int(_check_token(nxt, lc, ls, orc))
    gpu = m.decode(steps)[:, 0]
    inp = nxt
    for i in range(steps):
        hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), share_seed, prompt_len + i)
        _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
        exact += _check_token(int(gpu[i]), lc, ls, orc)
        inp = int(gpu[i])
    assert exact >= min_exact, f"{exact} of {steps + 1} tokens equal the oracle's"
    assert m.seq_len() == prompt_len + steps
    # one more position through the host-buffer entry point: the whole logit vector
    hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), share_seed, prompt_len + steps)
    lc_g, ls_g = m.forward_host(hc, hs)
    _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
    ref = lc + ls
    err = float(np.max(np.abs((lc_g + ls_g) - ref)) / np.max(np.abs(ref)))
    assert err < LOGIT_RTOL, err
    m.close()
    print(f"{shape_name}: {exact}/{steps + 1} tokens exact, logit rel err {err:.2e}, "
          f"{time.perf_counter() - t0:.1f} s")


def test_config2_qwen15b_28_layers_32_prompt_50_tokens(ctx, orc):
    """BASELINE config 2 exactly: 28 layers, 32-token seeded prompt, 50 greedy decode tokens."""
    _run_single(ctx, orc, "qwen2.5-1.5b", 32, 50, seed=0, share_seed=0x5EED, min_exact=49)


def test_config3_qwen7b_28_layers(ctx, orc):
    """The 28-layer 7B decode graph that bench.py times (same weight seed and share seed)."""
    _run_single(ctx, orc, "qwen2.5-7b", 16, 8, seed=0, share_seed=0x5EED, min_exact=8)


def test_config5_qwen14b_48_layers_batch8(ctx, orc):
    """Eight sequences of the 48-layer 14B shape decoded together, each checked slot by slot."""
    from shardlm_b200.model import QWEN2_5_14B, SecureModel

    _all_threads(orc)
    shape = QWEN2_5_14B
    B, steps, max_seq = 8, 3, 16
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, shape.vocab, 1 + (b % 3)).astype(np.int32) for b in range(B)]
    m = SecureModel(ctx, shape, max_seq=max_seq, max_batch=B, share_seed=11)
    host = m.load_random_weights(seed=0, host_copy=True)
    first = [m.prefill(p, slot=b) for b, p in enumerate(prompts)]
    toks = m.decode(steps, n_active=B)
    m.close()
    exact = 0
    om = _oracle_for(orc, shape, host, max_seq)
    for b, p in enumerate(prompts):
        om.reset()
        for i, t in enumerate(p):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(t), 11, (b << 32) + i)
            _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_GPU, attn_variant=orc.NL_APPROX)
        exact += _check_token(first[b], lc, ls, orc)
        inp = first[b]
        for i in range(steps):
            hc, hs = orc.embed_shares(host["embed"], shape.hidden, int(inp), 11, (b << 32) + len(p) + i)
            _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
            exact += _check_token(int(toks[i, b]), lc, ls, orc)
            inp = int(toks[i, b])
    assert exact >= B * (steps + 1) - 1, f"{exact} of {B * (steps + 1)} tokens equal the oracle's"
