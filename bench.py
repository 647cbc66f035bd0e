#!/usr/bin/env python3
"""Secret-shared decode throughput on B200 (BASELINE metric: "secret-shared decode tok/s
(Qwen2.5-7B shape)"; config 3: 7B architecture, V3 protocol, batch 1, 512-token seeded prompt,
128 decode tokens, tensor parallel over the GPUs given).

A step is one greedy decode token through all layers and the lm_head (one pass of the hot path).
  python bench.py [--gpus N --steps K --warmup W]          # our sm_100a path (libshardlm_cuda)
  python bench.py --impl reference ...                      # the reference's CPU share path
Under torchrun (N > 1) every rank holds its tensor-parallel shard; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "secret-shared decode tok/s (Qwen2.5-7B shape)"


def metric_for(model: str) -> str:
    """The headline metric for the default 7B workload; other shapes name themselves."""
    return METRIC if model == "qwen2.5-7b" else f"secret-shared decode tok/s ({model} shape)"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic (weight) byte of the
# dual-share GEMV, from one ncu capture of each 7B projection at one row: q/k/v 1.0020, o 1.0026,
# gate/up 1.0136, down 1.0290, lm_head 1.0043; weighted by their bytes per step 1.0157.
TRAFFIC_PER_ALGORITHMIC_BYTE_GATEUP = 1.0136
TRAFFIC_PER_ALGORITHMIC_BYTE = 1.0157


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--e2e-steps", type=int, default=24)
    p.add_argument("--cpu-sample-steps", type=int, default=8)
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------
# CPU path: the oracle (restatement of the reference's CPU share arithmetic), bounded sample
# ------------------------------------------------------------------------------------------------
def cpu_decode(shape, prompt: int, n_tokens: int, threads: int, seed: int = 0):
    """Greedy decode of whole tokens on the host cores through the oracle port: the reference's
    CPU share path (crates/v2/server/src/routes/secure_inference.rs:1553-1796 order: embedding
    shares, every layer's norm / q,k,v / RoPE / attention / o / residual / norm / gate,up / SwiGLU /
    down / residual, final norm, lm_head, client reconstruct + greedy argmax) with every linear on
    the CPU (SecureLinear::matmul, crates/v2/sharing/src/secure_linear.rs:103-117).

    Weights: random-init N(0, 0.02) bf16 matrices and q/k/v biases, unit norms, in the model's
    shape, generated on the host (same distribution as the GPU arm, not the same values; the work
    does not depend on them). The KV rows of the prompt's positions are zero-filled rather than
    computed by a CPU prefill, so the decode positions match the GPU arm's. Returns (seconds per
    token for each of the n_tokens decoded, description)."""
    from oracle import oracle as orc

    h, d, I, V = shape.hidden, shape.head_dim, shape.intermediate, shape.vocab
    qd, kvd = shape.n_heads * d, shape.n_kv_heads * d
    orc.set_threads(threads)
    om = orc.Model(h, shape.n_layers, shape.n_heads, shape.n_kv_heads, d, I, V, shape.rope_theta,
                   shape.rms_eps, prompt + n_tokens + 2)
    ones = np.ones(h, np.float32)
    f32 = lambda u16: (u16.astype(np.uint32) << 16).view(np.float32)
    for l in range(shape.n_layers):
        k = 16 * (l + 1)
        # [in][out] layouts: wq [h][qd], wk/wv [h][kvd], wo [qd][h], wg/wu [h][I], wd [I][h]
        ws = [orc.normal_bf16(s_, seed, k + i) for i, s_ in
              enumerate([(h, qd), (h, kvd), (h, kvd), (qd, h), (h, I), (h, I), (I, h)])]
        bs = [f32(orc.normal_bf16(n, seed, k + 8 + i)) if shape.qkv_bias else None
              for i, n in enumerate([qd, kvd, kvd])]
        om.set_layer(l, *ws, *bs, ones, ones)
    embed = orc.normal_bf16((V, h), seed, 1)
    lm = embed.T.copy() if shape.tied else orc.normal_bf16((h, V), seed, 2)
    om.set_head(lm, ones)
    om.set_len(prompt)
    tok = int(np.random.default_rng(0).integers(0, V))
    per_tok = []
    for i in range(n_tokens):
        t0 = time.perf_counter()
        hc, hs = orc.embed_shares(embed, h, tok, 0x5EED, prompt + i)
        _, _, lc, ls = om.forward(hc, hs, variant=orc.NL_APPROX, attn_variant=orc.NL_APPROX)
        tok = orc.argmax_last(lc, ls)
        per_tok.append(time.perf_counter() - t0)
    desc = (f"oracle port (C++, {threads} threads): whole greedy decode tokens of the {shape.n_layers}-layer "
            f"model (embedding shares, every layer, lm_head, argmax) at positions {prompt}.."
            f"{prompt + n_tokens - 1}; prompt KV rows zero-filled")
    return per_tok, desc


def run_reference(args, shape):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the reference arm runs on rank 0 only
    threads = os.cpu_count() or 1
    B = args.batch
    per_tok, desc = cpu_decode(shape, args.prompt, args.warmup + args.steps, threads)
    t = per_tok[args.warmup:] or per_tok
    sec = float(np.sum(t)) / len(t)  # one sequence decoded: a step is one token of it
    v = 1.0 / sec
    desc += f"; {len(t)} timed tokens after {len(per_tok) - len(t)} warm-up tokens, mean"
    if B > 1:
        desc += f"; one sequence of the {B}-sequence batch (the CPU path decodes sequences one by one)"
    line = {
        "impl": "reference", "metric": metric_for(shape.name), "value": round(v, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, shape, args.gpus, "cpu"),
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args, shape, world: int, parallelism: str) -> dict:
    """The workload both arms name (same string, so the driver can pair them)."""
    B = args.batch
    return {"workload": f"{shape.name} V3 greedy decode, prompt {args.prompt}, batch {B}, "
                        f"positions {args.prompt}..{args.prompt + args.warmup + args.steps}",
            "model": shape.name, "global_batch": B, "seq_len": args.prompt, "parallelism": parallelism}


# ------------------------------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device: int):
        self.samples, self.reasons, self.ok = [], 0, False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            # one query before the timed region: the first ones after nvmlInit are the slow ones
            pynvml.nvmlDeviceGetClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.ok = True
        except Exception:
            self.max = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": ["nvml unavailable"]}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": int(np.median(self.samples)), "sm_max_mhz": int(self.max), "reasons": names,
                "samples": len(self.samples)}

    @staticmethod
    def merge(per_rank: list) -> dict:
        """Every rank's summary in one: the lowest median SM clock, the union of throttle reasons."""
        ok = [c for c in per_rank if c.get("sm_mhz") is not None]
        if not ok:
            return per_rank[0]
        low = min(ok, key=lambda c: c["sm_mhz"])
        reasons = sorted({r for c in per_rank for r in c.get("reasons", [])})
        return {"sm_mhz": low["sm_mhz"], "sm_max_mhz": low["sm_max_mhz"], "reasons": reasons,
                "samples": sum(c.get("samples", 0) for c in ok), "ranks": len(per_rank),
                "sm_mhz_per_rank": [c.get("sm_mhz") for c in per_rank]}


# ------------------------------------------------------------------------------------------------
# Our path
# ------------------------------------------------------------------------------------------------
def run_ours(args, shape):
    import torch
    import torch.distributed as dist

    from shardlm_b200 import _lib
    from shardlm_b200.model import SecureModel
    from shardlm_b200.runtime import Context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    ctx = Context(local)
    if world > 1:
        from shardlm_b200.tp import init_tensor_parallel

        init_tensor_parallel(ctx, rank, world)

    B = args.batch
    e2e_steps = args.e2e_steps
    prof_steps = 3
    max_seq = args.prompt + args.warmup + args.steps + 2 * prof_steps + e2e_steps + 8
    model = SecureModel(ctx, shape, max_seq=max_seq, max_batch=B, share_seed=0x5EED, tp_rank=rank, tp_world=world)
    model.load_random_weights(seed=0)
    rng = np.random.default_rng(0)  # seeded uniform prompt token ids
    prompts = [rng.integers(0, shape.vocab, args.prompt).astype(np.int32) for _ in range(B)]
    # prefill throughput (config 3/5 report it beside decode): the first slot's prompt warms up the
    # kernels, the others (or, with one slot, a second prefill after a reset) are timed
    model.prefill(prompts[0], slot=0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_pf = time.perf_counter()
    if B > 1:
        for b in range(1, B):
            model.prefill(prompts[b], slot=b)
        n_pf = (B - 1) * args.prompt
    else:
        model.reset()
        model.prefill(prompts[0], slot=0)
        n_pf = args.prompt
    torch.cuda.synchronize()
    pf_s = time.perf_counter() - t_pf
    if world > 1:
        t = torch.tensor([pf_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pf_s = float(t.item())
    # tensor-pipe work of the timed prefill: the seven layer linears at 12 FLOPs per weight and token
    # (2 shares x 3 bf16 terms x multiply-add) and the prompt attention at 24 FLOPs per score and
    # per weighted value (6 bf16 term products x multiply-add), per rank
    h, d = shape.hidden, shape.head_dim
    per_layer = (h * shape.n_heads * d + 2 * h * shape.n_kv_heads * d + shape.n_heads * d * h
                 + 3 * h * shape.intermediate)
    n_prompts = max(1, B - 1) if B > 1 else 1
    P = args.prompt
    tc_flops = (12.0 * per_layer * shape.n_layers * n_pf
                + 24.0 * shape.n_heads * d * shape.n_layers * n_prompts * P * (P + 1) / 2) / world
    sustained = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            sustained = float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        sustained = 1400.0
    tc_tflops = tc_flops / pf_s / 1e12
    prefill = {"tokens": n_pf, "seconds": round(pf_s, 4), "tok_s": round(n_pf / pf_s, 1),
               "tensor_tflops": round(tc_tflops, 1), "tensor_flops_per_gpu": tc_flops,
               "tensor_frac_of_sustained_bf16": round(tc_tflops / sustained, 4),
               "sustained_bf16_tflops": sustained,
               "path": "shd_model_prefill: prompt chunks through the tcgen05 linears and the tcgen05 "
                       "prefill attention (host-synchronous, wall time around the call)"}
    lib = _lib.lib()
    model.decode_async(args.warmup)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync = torch.zeros(1, device="cuda")
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        # profiler capture window (ncu --profile-from-start off sees exactly the timed launches)
        torch.cuda.profiler.start()
        if world > 1:
            # a device-side rendezvous right before the start event: every rank's timed region starts
            # when the last rank's stream reaches it, so a rank whose host launches late does not
            # stretch the others' first exchange inside their timed region
            dist.all_reduce(sync)
        start.record(stream)
        model.decode_async(args.steps)
        end.record(stream)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        barrier()
    ms = start.elapsed_time(end)
    clock_summary = clocks.summary()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        per_rank = [None] * world
        dist.all_gather_object(per_rank, clock_summary)
        clock_summary = ClockSampler.merge(per_rank)
    toks = model.read_tokens(args.steps, B)
    launches_per_step = int(lib.shd_model_step_launches(model.handle))
    # per-kernel timing of the share-wise linears: the same step graph re-captured with CUDA events
    # around every linear launch, replayed right after the timed region (event nodes are kept out of
    # the timed graph itself)
    lib.shd_model_set_profiling(model.handle, 1)
    model.decode_async(prof_steps)
    ms5 = np.zeros(6, np.float32)
    by5 = np.zeros(6, np.float64)
    _lib.check(lib.shd_model_linear_times(model.handle, ms5.ctypes.data, by5.ctypes.data), ctx.ptr)
    lib.shd_model_set_profiling(model.handle, 0)
    # the same step with the overlap intact: %globaltimer stamps inside the kernels of the graph
    # (shd_model_timeline), per kind the mean time from the previous launch's end to its own
    timeline = in_graph_timeline(lib, _lib, model, ctx, prof_steps, by5)

    # e2e: generate_token_gpu semantics with host buffers (H2D hidden shares, D2H logit shares),
    # server-side embedding shares and client-side reconstruct + greedy sampling on the host; with
    # several sequences, one shd_model_forward_host_rows call serves all of them per step
    e2e = None
    if e2e_steps > 0:
        embed_host = None
        hw = model.head_weights(0)
        embed_host = hw["embed"].float().cpu().numpy()
        del hw
        torch.cuda.empty_cache()
        hrng = np.random.default_rng(1)
        cur = [int(t) for t in toks[-1, :B]]

        # pinned host buffers, reused every step: the hidden shares going in, the logit shares out
        def pinned(*shp):
            return torch.empty(*shp, dtype=torch.float32, pin_memory=True).numpy()

        c_buf, s_buf = pinned(B, shape.hidden), pinned(B, shape.hidden)
        out = (pinned(B, shape.vocab), pinned(B, shape.vocab))
        l_buf = np.empty(shape.vocab, np.float32)
        slots = np.arange(B, dtype=np.int32)

        def greedy(lc, ls):
            # client reconstruct + greedy: the LAST index among equal maxima (Iterator::max_by)
            l = np.add(lc, ls, out=l_buf)
            i = int(np.argmax(l))
            ties = np.flatnonzero(l[i + 1:] == l[i])
            return i + 1 + int(ties[-1]) if ties.size else i

        def one(cur):
            hrng.random(out=s_buf, dtype=np.float32)
            for b in range(B):
                np.subtract(embed_host[cur[b]], s_buf[b], out=c_buf[b])
            if B == 1:
                lc, ls = model.forward_host(c_buf[0], s_buf[0], slot=0, out=(out[0][0], out[1][0]))
                return [greedy(lc, ls)]
            lc, ls = model.forward_host_rows(slots, c_buf, s_buf, out=out)
            return [greedy(lc[b], ls[b]) for b in range(B)]

        for _ in range(2):
            cur = one(cur)
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps - 2):
            cur = one(cur)
        el = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([el], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        e2e = {"value": round(B * (e2e_steps - 2) / el, 3), "unit": "tok/s",
               "h2d_bytes_per_step": 2 * B * shape.hidden * 4 + (8 * B if B > 1 else 8),
               "d2h_bytes_per_step": 2 * B * shape.vocab * 4,
               "path": ("shd_model_forward_host (host shares in, host logit shares out, pinned host buffers), "
                        "host argmax") if B == 1 else
                       ("shd_model_forward_host_rows: the %d sequences' hidden shares in, their logit shares "
                        "out in one call per step (pinned host buffers), host argmax per sequence" % B)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        n, nw = args.cpu_sample_steps, 2
        per_tok, desc = cpu_decode(shape, args.prompt, nw + n, threads)
        sec = float(np.sum(per_tok[nw:])) / n
        desc += f"; {n} timed tokens after {nw} warm-up tokens, mean (one sequence)"
        cpu = {"value": round(1.0 / sec, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        peak, src = peaks()
        lin_ms = float(ms5[:5].sum())
        lin_bytes = float(by5[:5].sum())
        n_lin = 4 * shape.n_layers + 1
        achieved = lin_bytes / (lin_ms * 1e-3) / 1e9 if lin_ms > 0 else None
        gu_bytes = float(by5[2]) / shape.n_layers
        gu_us = float(ms5[2]) * 1e3 / shape.n_layers if ms5[2] > 0 else None
        gu_achieved = gu_bytes / (gu_us * 1e-6) / 1e9 if gu_us else None
        ms_step = ms / args.steps
        weight_bytes = shape.linear_params() * 2 / world
        value = B * args.steps / (ms * 1e-3)
        line = {
            "metric": metric_for(shape.name), "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {**workload_config(args, shape, world, f"tp{world}"),
                       "allreduce": (("nvlink peer-memory one-shot" if lib.shd_tp_peer_path(ctx.ptr) else "nccl")
                                     if world > 1 else None),
                       "l2": "weights streamed per step (>= 1.7 GB per GPU) exceed the 126 MB L2"},
            # the dominant kernel of the step (about 40 % of it in the ncu launch list): the gate/up
            # GEMV with its RMSNorm prologue and SwiGLU reshare epilogue, one launch per layer
            "roofline": {"bound": "hbm",
                         "kernel": "gemv_f32_kernel<1, 2, 1, 2> (gate/up: RMSNorm prologue, dual-share "
                                   "linear, SwiGLU reshare epilogue)",
                         "achieved": round(gu_achieved, 1) if gu_achieved else None, "peak": peak,
                         "peak_source": src, "unit": "GB/s",
                         "frac": round(gu_achieved / peak, 4) if gu_achieved else None,
                         "traffic": round(TRAFFIC_PER_ALGORITHMIC_BYTE_GATEUP * gu_bytes),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one gate/up "
                                           "launch (profiles/gemv_dual_share_7b.md): 1.0136 x the "
                                           "algorithmic bytes",
                         "algorithmic_bytes_per_launch": round(gu_bytes),
                         "avg_launch_us": round(gu_us, 2) if gu_us else None,
                         "all_gemv": {"achieved": round(achieved, 1) if achieved else None,
                                      "frac": round(achieved / peak, 4) if achieved else None,
                                      "algorithmic_bytes_per_launch": round(lin_bytes / n_lin),
                                      "avg_launch_us": round(lin_ms * 1e3 / n_lin, 2),
                                      "traffic": round(TRAFFIC_PER_ALGORITHMIC_BYTE * lin_bytes / n_lin)},
                         "per_kind_GBps": {k: round(by5[i] / (ms5[i] * 1e-3) / 1e9, 1) if ms5[i] > 0 else None
                                           for i, k in enumerate(["qkv", "o", "gateup", "down", "lm_head"])},
                         "per_kind_us_per_step": {k: round(float(ms5[i]) * 1e3, 1) for i, k in
                                                  enumerate(["qkv", "o", "gateup", "down", "lm_head", "attention"])},
                         "timing": "CUDA events around each launch in a profiled replay of the step graph "
                                   "right after the timed region (events cut programmatic-launch overlap)",
                         "in_graph": timeline},
            "step_roofline": {"weight_bytes_per_token_per_gpu": int(weight_bytes),
                              "frac_of_hbm": round(weight_bytes / (ms_step * 1e-3) / 1e9 / peak, 4)},
            "e2e": e2e,
            "prefill": prefill,
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clock_summary,
            "tokens_head": toks[:8, 0].tolist(),
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        _lib.lib().shd_tp_destroy(ctx.ptr)
        dist.destroy_process_group()


def in_graph_timeline(lib, _lib, model, ctx, steps: int, by5) -> dict | None:
    """Per kind (q/k/v, o, gate/up, down, lm_head, attention, TP exchange): the mean in-graph cost
    (the launch's last CTA exit minus the previous launch's) over the step's launches, and for the
    linears the weight bytes of one launch over that cost. None when some launch of the step runs
    on a path that is not stamped (the tensor-core linear of batched decode)."""
    import ctypes as C

    from shardlm_b200.microbench import TRACE_KINDS, timeline_summary

    lib.shd_model_set_profiling(model.handle, 2)
    try:
        model.decode_async(steps)
        n = C.c_int()
        _lib.check(lib.shd_model_timeline(model.handle, 0, None, None, C.byref(n)), ctx.ptr)
        kinds = np.zeros(n.value, np.int32)
        st = np.zeros((n.value, 8), np.uint64)
        _lib.check(lib.shd_model_timeline(model.handle, n.value, kinds.ctypes.data, st.ctypes.data, C.byref(n)),
                   ctx.ptr)
    finally:
        lib.shd_model_set_profiling(model.handle, 0)
    if (st[:, [0, 2, 4]] == np.uint64(0xFFFFFFFFFFFFFFFF)).any():
        return None
    summ = timeline_summary(kinds, st)
    out = {"us_per_launch": {}, "GBps": {}, "frac": {}}
    peak = peaks()[0]
    for i, k in enumerate(TRACE_KINDS):
        if k not in summ:
            continue
        cost = summ[k]["cost"]
        out["us_per_launch"][k] = cost
        if i < 5 and cost > 0:
            per_launch = by5[i] / max(1, int((kinds == i).sum()))
            out["GBps"][k] = round(per_launch / (cost * 1e-6) / 1e9, 1)
            out["frac"][k] = round(out["GBps"][k] / peak, 4)
    out["span_us"] = summ["traced_span_us"]
    out["timing"] = ("%globaltimer stamps inside every GEMV, attention and exchange launch of a traced replay "
                     "of the step graph (shd_model_timeline); cost = last CTA exit minus the previous launch's")
    return out


def main():
    args = parse()
    from shardlm_b200.model import SHAPES

    shape = SHAPES[args.model]
    if args.impl == "reference":
        run_reference(args, shape)
    else:
        run_ours(args, shape)


if __name__ == "__main__":
    main()
