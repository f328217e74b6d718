#!/usr/bin/env python
"""Decode throughput of the device-resident llmdot path (BASELINE.json metric:
decode tok/s at batch 1 / 32 on 1..8 B200, achieved HBM GB/s vs peak).

Default workload: Llama-3.2-1B-shape synthetic Q4_K_M
GGUF, batch 1, 512-token random prompt, greedy decode, fp16 KV of 4096
positions.  A "step" is one greedy decode token for every session of the GPU.

    python bench.py [--gpus N --steps K --warmup W] [--batch B] [--config NAME]
    python bench.py --impl reference ...   # the reference's CPU algorithm (oracle port)

Under torchrun each rank drives its own GPU with its own sessions (session
data parallelism, no collective on the data path: weak scaling); rank 0 prints
one JSON line with value = all ranks' tokens / the slowest rank's device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from typing import Optional

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from dotllm_b200 import synth  # noqa: E402

WORKLOADS = {
    "llama1b": "Llama-3.2-1B-shape synthetic Q4_K_M GGUF (16 layers, d2048, 32q/8kv heads, hd64, FFN 8192, "
               "vocab 128256 tied; Q4_K, attn_v/ffn_down Q6_K), {prompt}-token random prompt, greedy decode, "
               "{kv} KV cache of {ctx} positions, batch {batch} per GPU",
    "tiny": "tiny LLaMA-like synthetic GGUF (6 layers, d512), {prompt}-token prompt, greedy decode, {kv} KV, batch {batch}",
    "phi3mini": "Phi-3-mini-shape synthetic Q4_K_M GGUF, {prompt}-token prompt, greedy decode, {kv} KV, batch {batch}",
    "gemma2b": "Gemma-2-2B-shape synthetic Q4_K_M GGUF, {prompt}-token prompt, greedy decode, {kv} KV, batch {batch}",
    "llama8b": "Llama-3-8B-shape synthetic Q4_K_M GGUF, {prompt}-token prompt, greedy decode, {kv} KV, batch {batch}",
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Clock / throttle sampling during the timed region: an NVML polling thread (read-only
    queries every 10 ms) and, as a fallback, `nvidia-smi -lms 200`.  The summary uses the NVML
    samples when there are any."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    PERIOD_S = 0.01

    def __init__(self, gpu_index: int, uuid: Optional[str] = None):
        self.idx = gpu_index
        self.uuid = uuid  # the CUDA device's UUID: NVML's order need not be CUDA's
        self.proc = None
        self.samples = []  # (sm_mhz, sm_max_mhz, [reason names]) from NVML
        self._stop = threading.Event()
        self._thread = None

    def _nvml_loop(self, nv):
        try:
            nv.nvmlInit()
        except Exception:
            return
        try:
            h = None
            if self.uuid:
                want = self.uuid.lower().replace("gpu-", "")
                for i in range(int(nv.nvmlDeviceGetCount())):
                    hi = nv.nvmlDeviceGetHandleByIndex(i)
                    u = nv.nvmlDeviceGetUUID(hi)
                    u = u.decode() if isinstance(u, bytes) else str(u)
                    if u.lower().replace("gpu-", "") == want:
                        h = hi
                        break
            if h is None:
                h = nv.nvmlDeviceGetHandleByIndex(self.idx)
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            bits = {name: getattr(nv, "nvmlClocksEventReason" + tag, None) or getattr(nv, "nvmlClocksThrottleReason" + tag)
                    for name, tag in zip(self.REASONS, ("HwSlowdown", "HwThermalSlowdown", "SwThermalSlowdown",
                                                        "SwPowerCap"))}
            while not self._stop.is_set():
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                r = int(get_reasons(h))
                self.samples.append((sm, mx, [n for n, b in bits.items() if r & int(b)]))
                self._stop.wait(self.PERIOD_S)
        except Exception:
            pass
        finally:
            try:
                nv.nvmlShutdown()
            except Exception:
                pass

    def __enter__(self):
        if self.idx < 0:
            return self
        try:
            import pynvml
            self._thread = threading.Thread(target=self._nvml_loop, args=(pynvml,), daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.samples:
            sm = [s[0] for s in self.samples]
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                    "reasons": sorted({n for s in self.samples for n in s[2]}), "samples": len(self.samples),
                    "source": "nvml"}
        rows = [r.split(",") for r in (getattr(self, "out", "") or "").strip().splitlines()]
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({self.REASONS[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


def cpu_baseline_sample(path: str, cfg, threads: int, n_prompt: int, n_decode: int):
    """Time the oracle (C restatement of the reference's managed CPU path) on a bounded sample:
    n_prompt prefill tokens then n_decode greedy steps; returns decode tok/s."""
    from oracle import oracle as O
    O.set_threads(threads)
    m = O.Model(path)
    s = O.Session(m)
    prompt = synth.prompt_tokens(cfg, n_prompt)
    t0 = time.perf_counter()
    logits = None
    for i, t in enumerate(prompt):
        logits = s.process_token(int(t), i)
    t1 = time.perf_counter()
    tok = int(np.argmax(logits))
    for j in range(n_decode):
        logits = s.process_token(tok, n_prompt + j)
        tok = int(np.argmax(logits))
    t2 = time.perf_counter()
    s.close()
    m.close()
    return {"decode_tok_s": n_decode / (t2 - t1), "prefill_tok_s": n_prompt / (t1 - t0),
            "decode_s_per_tok": (t2 - t1) / n_decode}


def run_reference(args, rank):
    if rank != 0:
        return
    cfg = synth.get(args.config)
    path = synth.build_model(cfg)
    from oracle import oracle as O
    O.build()
    threads = max(1, O.max_threads())
    n_prompt = 8
    # warm-up: W decode steps (bounded), then K decode steps sized to a few minutes of CPU time
    probe = cpu_baseline_sample(path, cfg, threads, n_prompt, max(1, min(args.warmup, 3)))
    budget_s = 120.0
    k = max(1, min(args.steps, int(budget_s / max(probe["decode_s_per_tok"], 1e-6))))
    res = cpu_baseline_sample(path, cfg, threads, n_prompt, k)
    v = res["decode_tok_s"]
    line = {
        "impl": "reference", "metric": f"decode tok/s (batch {args.batch})", "value": v, "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": k, "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOADS.get(args.config, args.config).format(prompt=n_prompt, kv="f32", ctx="its",
                                                                              batch=1),
                   "model": args.config, "note": "the reference decodes one session at a time on the host cores"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n_prompt}-token prompt then {k} greedy decode steps of the {args.config} model "
                                   f"(C restatement of llmdot's managed CPU path, row-parallel OpenMP, {threads} threads)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "prefill_tok_s": res["prefill_tok_s"],
    }
    print(json.dumps(line), flush=True)


# dram__bytes_read.sum + dram__bytes_write.sum over the four matvec launches of one decode layer
# (profiles/gemv_mma_kernel_llama1b_b1.md) divided by their quantised weight bytes
DRAM_PER_ALGORITHMIC_BYTE = (2.431232 + 18.949632 + 13.859072 + 3.880960) / (2.359296 + 18.874368 + 13.762560 + 3.813376)


def measure(m, cfg, args, B, n_prompt, ctx, rank, steps, dist, local, clocks=False):
    """Prefill B sessions, warm up, then time `steps` device-resident greedy steps of all of them
    (max over ranks).  Returns the sessions, the device ms, kernels per step, prefill seconds and
    the clock record."""
    import torch
    from dotllm_b200.engine import decode_steps
    # one untimed prompt first: the first calls of a process load kernels and build graphs
    warm = m.session(max_ctx=ctx, kv=args.kv)
    warm.prefill(synth.prompt_tokens(cfg, min(n_prompt, 64), session=10_000))
    warm.close()
    sessions = [m.session(max_ctx=ctx, kv=args.kv) for _ in range(B)]
    # under tensor parallelism every rank decodes the same sessions; under DP, distinct ones
    sid = 0 if args.tp else rank * B
    prompts = [synth.prompt_tokens(cfg, n_prompt, session=sid + i) for i in range(B)]
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    first = [s.prefill(p)[0] for s, p in zip(sessions, prompts)]
    prefill_s = time.perf_counter() - t0
    toks, _, _ = decode_steps(sessions, first, args.warmup)
    cur = toks[-1]
    if dist:
        dist.barrier()
        torch.cuda.synchronize()
    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except ValueError:
            pass
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clk = ClockSampler(gpu_index if clocks else -1, uuid)
    if clocks:
        with clk:
            out, dev_ms, kps = decode_steps(sessions, cur, steps)
    else:
        out, dev_ms, kps = decode_steps(sessions, cur, steps)
    if dist:
        t = torch.tensor([dev_ms, prefill_s], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, prefill_s = float(t[0].item()), float(t[1].item())
    return sessions, out[-1], dev_ms, kps, prefill_s, clk


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="llama1b")
    ap.add_argument("--batch", type=int, default=1, help="sessions per GPU (per TP group with --tp)")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--kv", choices=["f16", "f32"], default="f16")
    ap.add_argument("--tp", action="store_true", help="the torchrun ranks form ONE tensor-parallel group")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch32", action="store_true", help="skip the sharded batch-32 measurement")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world == 1:
        args.tp = False

    if args.impl == "reference":
        run_reference(args, rank)
        return

    cfg = synth.get(args.config)
    n_prompt = args.prompt if args.prompt is not None else cfg.prompt_len
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    # rank 0 writes the synthetic GGUF (spawned workers, before any CUDA work), the others reuse it
    if rank == 0:
        path = synth.build_model(cfg)
    if dist:
        dist.barrier()
    path = synth.build_model(cfg)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # single-threaded, like the reference (no threading in its src/): ~10-30 s of CPU work
        n_pre, n_dec = (2, 3) if cfg.hidden >= 2048 else (8, 16)
        r = cpu_baseline_sample(path, cfg, 1, n_pre, n_dec)
        cpu = {"value": r["decode_tok_s"], "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"{n_pre}-token prompt then {n_dec} greedy decode steps of the same model, C restatement of "
                         f"llmdot's managed CPU path (oracle/), 1 thread"}

    from dotllm_b200.engine import CudaModel, decode_batch, tp_unique_id
    t_load = time.perf_counter()
    if args.tp:
        m = CudaModel.load_tp(path, world, rank, device=local)
        uid = [tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        m.tp_init(uid[0])
    else:
        m = CudaModel.load(path, device=local)
    load_s = time.perf_counter() - t_load
    ctx = min(cfg.context, 4096) if args.config == "llama1b" else cfg.context
    B = args.batch
    sessions, cur, dev_ms, kps, prefill_s, clk = measure(m, cfg, args, B, n_prompt, ctx, rank, args.steps, dist,
                                                         local, clocks=True)

    # end to end through the public per-step API: host tokens in, host ids out, every step
    if dist:
        dist.barrier()
    e2e_steps = args.steps
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        cur, _ = decode_batch(sessions, cur)
    e2e_s = time.perf_counter() - t0
    if dist:
        import torch
        t = torch.tensor([e2e_s], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    for s in sessions:
        s.close()

    # roofline of the dominant kernel family: the quantised matvec launches of one step,
    # each timed live with CUDA events (profile_matvec), aggregated over the step's launches
    c = m.config
    per_layer = ["attn_qkv"] if c["qkv_fused"] else ["attn_q", "attn_k", "attn_v"]
    per_layer += ["attn_output", "ffn_gate", "ffn_up", "ffn_down"]
    tot_ms, tot_bytes, launches = 0.0, 0, 0
    for name in per_layer:
        ms, nb = m.profile_matvec(f"blk.*.{name}.weight", B, 5)
        tot_ms += ms * c["layers"]
        tot_bytes += nb * c["layers"]
        launches += c["layers"]
    head = "output.weight" if (args.tp or not c["tied"]) else "token_embd.weight"
    ms, nb = m.profile_matvec(head, B, 10)
    tot_ms += ms
    tot_bytes += nb
    launches += 1
    peak, peak_kind = peaks()
    achieved = tot_bytes / (tot_ms * 1e-3) / 1e9

    # sessions sharded over the GPUs: 32 in total (the north star's scaling workload)
    b32 = None
    if not args.tp and not args.no_batch32 and 32 % world == 0 and 32 // world != B:
        per = 32 // world
        k32 = min(args.steps, 64)
        ss, _, ms32, _, pre32, _ = measure(m, cfg, args, per, n_prompt, ctx, rank, k32, dist, local)
        for s in ss:
            s.close()
        b32 = {"global_batch": 32, "sessions_per_gpu": per, "steps": k32, "value": per * world * k32 / (ms32 * 1e-3),
               "unit": "tok/s", "ms_per_step": ms32 / k32, "prefill_tok_s": per * world * n_prompt / pre32}

    # Generate with Sampler.Sample on the device against greedy Generate, same prompt and length:
    # the difference is the sampler and its per-token history upload (one GPU only)
    sampled = None
    if world == 1 and not args.tp:
        try:
            from dotllm_b200.native import LlmdotSampling
            ss = m.session(max_ctx=ctx, kv=args.kv)
            sp = synth.prompt_tokens(cfg, n_prompt, session=20_000)
            ntok = min(args.steps, 256)
            opts = LlmdotSampling(seed=42)  # the reference's defaults: top-k 40, T 0.8, penalty 1.1 over 64
            ss.generate(sp, 4)
            ss.generate_sampled(sp, 4, opts)
            t0 = time.perf_counter()
            ng = len(ss.generate(sp, ntok))
            tg = time.perf_counter() - t0
            t0 = time.perf_counter()
            ns = len(ss.generate_sampled(sp, ntok, opts))
            ts = time.perf_counter() - t0
            ss.close()
            sampled = {"prompt": n_prompt, "tokens": ntok, "greedy_generate_s": tg, "sampled_generate_s": ts,
                       "sampler_us_per_token": (ts - tg) / max(ntok, 1) * 1e6, "tokens_out": [ng, ns],
                       "options": "top_k 40, top_p 0.95 (unused with top_k), temperature 0.8, repeat penalty 1.1 "
                                  "over 64 tokens, seed 42; wall clock of the public calls, prefill included in both"}
        except Exception as e:  # recorded, never allowed to drop the measurement line
            sampled = {"error": str(e)[:300]}

    K = args.steps
    step_ms = dev_ms / K
    layer_b, head_b = m.weight_bytes()
    kv_bytes_per_elem = 2 if args.kv == "f16" else 4
    kv_dim = c["heads_kv"] * c["head_dim"] // (world if args.tp else 1)
    mean_pos = n_prompt + args.warmup + K / 2.0
    kv_read = B * c["layers"] * 2 * kv_dim * kv_bytes_per_elem * mean_pos
    step_bytes = layer_b + head_b + kv_read
    ranks_tokens = 1 if args.tp else world  # a TP group decodes one set of sessions
    value = B * K * ranks_tokens / (dev_ms * 1e-3)
    par = f"tp{world} (one tensor-parallel group, NCCL all-reduce after attn-out and ffn-down)" if args.tp else \
        f"dp{world} (independent sessions per GPU)"
    line = {
        "metric": f"decode tok/s (batch {B})", "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "strong" if args.tp else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_K/Q6_K, uniform random prompt ids",
        "config": {"workload": WORKLOADS.get(args.config, args.config).format(prompt=n_prompt, kv=args.kv, ctx=ctx,
                                                                              batch=B),
                   "model": args.config, "global_batch": B * ranks_tokens, "seq_len": n_prompt, "kv": args.kv,
                   "parallelism": par,
                   "l2": f"weights ({(layer_b + head_b) / 1e6:.0f} MB per GPU) exceed L2 (126 MB): inputs larger "
                         f"than L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": tot_bytes * DRAM_PER_ALGORITHMIC_BYTE,
                     "traffic_note": "DRAM bytes per step scaled from the ncu capture in "
                                     "profiles/gemv_mma_kernel_llama1b_b1.md (read+write / algorithmic = 1.008)",
                     "kernel": "quantised matvec (all launches of one step)",
                     "launches_per_step": launches, "bytes_per_step": tot_bytes,
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind},
        "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (step_ms * 1e-3) / 1e9,
                          "frac": step_bytes / (step_ms * 1e-3) / 1e9 / peak,
                          "note": "per GPU: quantised weights + KV reads at the mean position / device step time"},
        "cpu_baseline": cpu,
        "e2e": {"value": B * e2e_steps * ranks_tokens / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": B * (4 + 4 + 32),
                "d2h_bytes_per_step": B * 4},
        "gpu_launches": kps * K,
        "kernels_per_step": kps,
        "clocks": clk.summary(),
        "prefill_tok_s": B * ranks_tokens * n_prompt / prefill_s,
        "load_s": load_s,
        "sharded_batch32": b32,
        "sampled": sampled,
    }
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
