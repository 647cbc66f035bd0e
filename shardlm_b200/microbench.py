"""Kernel microbenchmarks (CUDA events on the launching stream).

  python -m shardlm_b200.microbench linear [--model qwen2.5-7b] [--kind all|qkv|o|gateup|down|lm_head]
                                           [--rows 1] [--iters 20]
  python -m shardlm_b200.microbench beaver [--n 9699328] [--iters 20]
  python -m shardlm_b200.microbench ring   [--copies 16] [--iters 20]
  python -m shardlm_b200.microbench attn   [--model qwen2.5-7b] [--kv-len 577] [--iters 20]
  python -m shardlm_b200.microbench prefill [--model qwen2.5-7b] [--prompt 512] [--layers 28]
  python -m shardlm_b200.microbench attn-prefill [--model qwen2.5-7b] [--rows 512] [--kv-len 512]
  python -m shardlm_b200.microbench timeline [--model qwen2.5-7b] [--prompt 512] [--rows 1] [--dump f.npz]

--graph times a captured CUDA graph of the launches instead of host-issued launches.
Each weight kind is instantiated in enough copies to exceed the 126 MB L2, and launches rotate over
the copies, so every launch streams its weights from HBM.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .model import SHAPES
from .runtime import Context, Weight, ptr
from .sharing import GpuSecureLinear

L2_BYTES = 126 * 2**20


GRAPH = False  # --graph: time a CUDA graph of `iters` back-to-back launches (no host launch cost)


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    g = None
    if GRAPH:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(iters):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    if g is not None:
        g.replay()
    else:
        for i in range(iters):
            fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def linear(args, ctx: Context):
    sh = SHAPES[args.model]
    h, d = sh.hidden, sh.head_dim
    kinds = {"qkv": (sh.n_heads * d + 2 * sh.n_kv_heads * d, h), "o": (h, sh.n_heads * d),
             "gateup": (2 * sh.intermediate, h), "down": (h, sh.intermediate), "lm_head": (sh.vocab, h)}
    todo = list(kinds) if args.kind == "all" else [args.kind]
    out = {}
    for k in todo:
        N, K = kinds[k]
        copies = max(1, -(-2 * L2_BYTES // (N * K * 2)))
        lins = []
        for c in range(copies):
            w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
            lins.append(GpuSecureLinear(ctx, Weight.from_bf16_out_in(ctx, w), None))
            del w
        M = args.rows
        xc, xs = torch.randn(M, K, device="cuda"), torch.rand(M, K, device="cuda")
        yc, ys = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")

        def run(i):
            ctx.call("shd_linear_dual_f32", lins[i % copies].weight.handle, None, ptr(xc), ptr(xs),
                     ptr(yc), ptr(ys), M, None, None)

        ms = _time(run, args.iters)
        ctx.sync()
        out[k] = {"N": N, "K": K, "rows": M, "us": round(ms * 1e3, 2), "GBps": round(N * K * 2 / ms / 1e6, 1),
                  # 5 rows and more run on the tensor cores: 2 shares x 3 bf16 terms x 2 flops per
                  # weight and row
                  "tensor_TFLOPs": round(12.0 * M * N * K / ms / 1e9, 1) if M >= 5 else None}
        del lins
        torch.cuda.empty_cache()
    print(json.dumps(out))


def beaver(args, ctx: Context):
    from .sharing import beaver_triples_f32, secure_multiply_batch

    n = args.n
    x = [torch.randn(n, device="cuda") for _ in range(4)]
    t = beaver_triples_f32(ctx, n, seed=1)
    res = secure_multiply_batch(ctx, *x, t, return_opened=True)

    def run(i):
        secure_multiply_batch(ctx, *x, t, return_opened=True)

    ms = _time(run, args.iters)
    ctx.sync()
    del res
    print(json.dumps({"beaver_f32": {"n": n, "us": round(ms * 1e3, 2), "GBps": round(56 * n / ms / 1e6, 1)}}))


def ring(args, ctx: Context):
    from .sharing import LinearServer

    rng = np.random.default_rng(0)
    servers = [LinearServer(rng.integers(-2**20, 2**20, 1536 * 1536, dtype=np.int64).astype(np.int32), None,
                            1536, 1536, 16, ctx) for _ in range(args.copies)]
    xc = torch.randint(-2**31, 2**31 - 1, (1, 1536), device="cuda", dtype=torch.int64).to(torch.int32)
    xs = torch.randint(-2**31, 2**31 - 1, (1, 1536), device="cuda", dtype=torch.int64).to(torch.int32)
    yc = torch.empty(1, 1536, device="cuda", dtype=torch.int32)
    ys = torch.empty(1, 1536, device="cuda", dtype=torch.int32)

    def run(i):
        s = servers[i % args.copies]
        ctx.call("shd_linear_dual_ring", s.weight.handle, None, ptr(xc), ptr(xs), ptr(yc), ptr(ys), 1, 16)

    ms = _time(run, args.iters)
    ctx.sync()
    b = 1536 * 1536 * 4
    print(json.dumps({"ring_linear_1536": {"us": round(ms * 1e3, 2), "GBps": round(b / ms / 1e6, 1)}}))


def attn(args, ctx: Context):
    """Decode attention over reconstructed caches: --rows query rows (sequence 0), the last one at
    position kv_len - 1 and each earlier row one position before the next."""
    sh = SHAPES[args.model]
    H, Hkv, d, L = sh.n_heads, sh.n_kv_heads, sh.head_dim, args.kv_len
    M = args.rows
    cap = L + 16
    copies = max(1, -(-2 * L2_BYTES // (2 * cap * Hkv * d * 4)))
    ks = [torch.randn(cap, Hkv * d, device="cuda") for _ in range(copies)]
    vs = [torch.randn(cap, Hkv * d, device="cuda") for _ in range(copies)]
    q = torch.randn(M, H * d, device="cuda")
    oc, os_ = torch.empty(M, H * d, device="cuda"), torch.empty(M, H * d, device="cuda")
    pos = np.array([L - M + i for i in range(M)], np.int32)

    def run(i):
        ctx.call("shd_attn_decode", ptr(q), ptr(ks[i % copies]), ptr(vs[i % copies]), cap, H, Hkv, d,
                 pos.ctypes.data, M, 0, None, ptr(oc), ptr(os_))

    ms = _time(run, args.iters)
    ctx.sync()
    kv_bytes = 2 * int(pos.astype(np.int64).sum() + M) * Hkv * d * 4
    print(json.dumps({"attn": {"H": H, "Hkv": Hkv, "rows": M, "kv_len": L, "us_per_call_incl_host": round(ms * 1e3, 2),
                               "kv_bytes": kv_bytes}}))


def attn_prefill(args, ctx: Context):
    """Prompt-block attention on the tensor cores (shd_attn_prefill): --rows query rows ending at
    position kv_len - 1, every head of the model; reports tensor TFLOP/s (6 bf16 term products per
    f32 multiply-add of QK^T and PV, causal)."""
    sh = SHAPES[args.model]
    H, Hkv, d = sh.n_heads, sh.n_kv_heads, sh.head_dim
    M, L = args.rows, max(args.kv_len, args.rows)
    pos0 = L - M
    q = torch.randn(M, H * d, device="cuda")
    k = torch.randn(L, Hkv * d, device="cuda")
    v = torch.randn(L, Hkv * d, device="cuda")
    oc, os_ = torch.empty(M, H * d, device="cuda"), torch.empty(M, H * d, device="cuda")

    def run(i):
        ctx.call("shd_attn_prefill", ptr(q), ptr(k), ptr(v), L, H, Hkv, d, pos0, M, 0, None, ptr(oc), ptr(os_))

    ms = _time(run, args.iters)
    ctx.sync()
    pairs = M * pos0 + M * (M + 1) // 2  # (query, position) pairs attended
    flops = 24.0 * H * d * pairs
    print(json.dumps({"attn_prefill": {"H": H, "Hkv": Hkv, "rows": M, "kv_len": L,
                                       "us_per_call_incl_host": round(ms * 1e3, 2),
                                       "tensor_TFLOPs": round(flops / ms / 1e9, 1)}}))


def prefill(args, ctx: Context):
    """Whole-model prefill of a seeded prompt: one untimed prefill, then a timed one inside a
    profiler window (cudaProfilerStart/Stop), so `ncu --profile-from-start off` lists exactly the
    timed prefill's launches."""
    from .model import SecureModel

    sh = SHAPES[args.model].replace(n_layers=args.layers) if args.layers else SHAPES[args.model]
    m = SecureModel(ctx, sh, max_seq=args.prompt + 8)
    m.load_random_weights(seed=0)
    toks = np.random.default_rng(0).integers(0, sh.vocab, args.prompt).astype(np.int32)
    m.prefill(toks)
    m.reset()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    m.prefill(toks)
    e.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = s.elapsed_time(e)
    print(json.dumps({"prefill": {"model": sh.name, "layers": sh.n_layers, "tokens": args.prompt,
                                  "ms": round(ms, 3), "tok_s": round(args.prompt / ms * 1e3, 1)}}))
    m.close()


TRACE_KINDS = ["qkv", "o", "gateup", "down", "lm_head", "attention", "exchange"]


def timeline_summary(kinds: np.ndarray, st: np.ndarray) -> dict:
    """Per kind, mean over its launches (microseconds) of: `cost` = its last CTA's exit minus the
    previous traced launch's last exit (these sum to the step); `lead` = how long before that
    previous exit its first CTA was resident; `dep` = from the previous exit to its first return
    from the dependency wait; `prologue` = from that return to the last CTA's end of prologue;
    `body` = from the end of prologue to the last exit; `exit_spread` = last minus first exit."""
    ones = np.uint64(0xFFFFFFFFFFFFFFFF)
    e0, e1 = st[:, 0].astype(np.float64), (~st[:, 1]).astype(np.float64)
    w0, r1 = st[:, 2].astype(np.float64), (~st[:, 3]).astype(np.float64)
    x0, x1 = st[:, 4].astype(np.float64), (~st[:, 5]).astype(np.float64)
    assert not (st[:, [0, 2, 4]] == ones).any(), "a traced launch was not stamped"
    out = {}
    for k in range(len(TRACE_KINDS)):
        idx = [i for i in range(1, len(kinds)) if kinds[i] == k]
        if not idx:
            continue
        prev = np.array([x1[i - 1] for i in idx])
        i = np.array(idx)
        out[TRACE_KINDS[k]] = {
            "n": len(idx),
            "cost": round(float(np.mean(x1[i] - prev)) / 1e3, 2),
            "lead": round(float(np.mean(prev - e0[i])) / 1e3, 2),
            "dep": round(float(np.mean(w0[i] - prev)) / 1e3, 2),
            "prologue": round(float(np.mean(r1[i] - w0[i])) / 1e3, 2),
            "body": round(float(np.mean(x1[i] - r1[i])) / 1e3, 2),
            "exit_spread": round(float(np.mean(x1[i] - x0[i])) / 1e3, 2),
            "entry_spread": round(float(np.mean(e1[i] - e0[i])) / 1e3, 2),
        }
    out["traced_span_us"] = round(float(x1[-1] - e0[0]) / 1e3, 1)
    return out


def timeline(args, ctx: Context):
    """Decode-step timeline from %globaltimer stamps inside the kernels of the captured step
    (shd_model_timeline): where the step's time goes between and inside the launches, with the
    programmatic overlap left intact."""
    import ctypes as C

    from ._lib import check, lib
    from .model import SecureModel

    import os

    sh = SHAPES[args.model].replace(n_layers=args.layers) if args.layers else SHAPES[args.model]
    B = args.rows
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:  # under torchrun: tensor parallel over the ranks, as bench.py
        import torch.distributed as dist
        from datetime import timedelta

        from .tp import init_tensor_parallel

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", torch.cuda.current_device()))
        init_tensor_parallel(ctx, rank, world)
    m = SecureModel(ctx, sh, max_seq=args.prompt + 2 * args.iters + 16, max_batch=B, tp_rank=rank, tp_world=world)
    m.load_random_weights(seed=0)
    rng = np.random.default_rng(0)
    for b in range(B):
        m.prefill(rng.integers(0, sh.vocab, args.prompt).astype(np.int32), slot=b)
    m.decode(4, B)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    m.decode_async(args.iters)
    e.record()
    torch.cuda.synchronize()
    plain_ms = s.elapsed_time(e) / args.iters
    check(lib().shd_model_set_profiling(m.handle, 2), ctx.ptr)
    m.decode(4, B)
    n = C.c_int()
    check(lib().shd_model_timeline(m.handle, 0, None, None, C.byref(n)), ctx.ptr)
    kinds = np.zeros(n.value, np.int32)
    st = np.zeros((n.value, 8), np.uint64)
    check(lib().shd_model_timeline(m.handle, n.value, kinds.ctypes.data, st.ctypes.data, C.byref(n)), ctx.ptr)
    s.record()
    m.decode_async(args.iters)
    e.record()
    torch.cuda.synchronize()
    traced_ms = s.elapsed_time(e) / args.iters
    check(lib().shd_model_set_profiling(m.handle, 0), ctx.ptr)
    summ = timeline_summary(kinds, st)
    if rank == 0:
        print(json.dumps({"timeline": {"model": sh.name, "layers": sh.n_layers, "rows": B, "prompt": args.prompt,
                                       "tp": world, "step_ms": round(plain_ms, 4),
                                       "traced_step_ms": round(traced_ms, 4), "kinds": summ}}))
    if args.dump:
        np.savez(args.dump + (f".rank{rank}" if world > 1 else ""), kinds=kinds, stamps=st)
    m.close()
    if world > 1:
        lib().shd_tp_destroy(ctx.ptr)
        dist.destroy_process_group()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("what", choices=["linear", "beaver", "ring", "attn", "attn-prefill", "prefill", "timeline"])
    p.add_argument("--dump", default="")
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--layers", type=int, default=0)
    p.add_argument("--kv-len", type=int, default=577)
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--kind", default="all")
    p.add_argument("--rows", type=int, default=1)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--n", type=int, default=512 * 18944)
    p.add_argument("--copies", type=int, default=16)
    p.add_argument("--graph", action="store_true")
    args = p.parse_args()
    global GRAPH
    GRAPH = args.graph
    import os

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    ctx = Context(local)
    {"linear": linear, "beaver": beaver, "ring": ring, "attn": attn, "attn-prefill": attn_prefill,
     "prefill": prefill, "timeline": timeline}[args.what](args, ctx)


if __name__ == "__main__":
    main()
