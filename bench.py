#!/usr/bin/env python
"""Benchmark: greedy generation on a synthetic model through libstrasgpt.so.

One step = one request of the workload: a P-token prompt (prefill) followed
by S greedy decode steps, batch 1, on the benchmark shape (default: the
Qwen3-0.6B-shaped configuration, P=512, S=128). Printed on rank 0 as ONE
JSON line:
  value       decode tok/s, whole job, device time (CUDA events on the
              library's stream), weights resident in HBM;
  prefill     prefill tok/s, same timing;
  e2e         decode tok/s through the reference-facing C ABI
              (transformer_predict with host token/logits buffers, host
              argmax as strasgpt.c does), host wall clock;
  roofline    the decode matvec kernels' algorithmic bytes / their CUDA-event
              time, against the measured HBM copy bandwidth;
  cpu_baseline the reference's own forward pass (oracle/_ref, OpenMP, all
              host cores) on a bounded sample of the same workload.
`--impl reference` times the reference CPU implementation alone (rank 0).
Launch with N>1 GPUs through torch.distributed.run (tensor parallel).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL_CACHE = os.environ.get("STRASGPT_MODEL_CACHE", "/tmp/strasgpt_models")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["strasgpt", "reference"], default="strasgpt")
    p.add_argument("--config", default="c2_qwen3_0p6b")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


class Dist:
    """Rank placement from torch.distributed.run's environment; host-side
    barrier and max-reduce over gloo (the timings are device measurements)."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", str(self.rank)))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, values):
        if not self.pg:
            return list(values)
        import torch
        t = torch.tensor(list(values), dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return t.tolist()

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi samples during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def profiled_dram_bytes_per_step(kernel: str, config: str):
    """DRAM bytes (read + write) per decode step of `kernel` on `config`,
    from the committed ncu summary profiles/<kernel>_<config>.md (line
    `dram_bytes_per_step: N`), or None."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("dram_bytes_per_step:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


def golden_tokens(name: str):
    path = os.path.join(ROOT, "tests", "golden", f"{name}.json")
    if not os.path.exists(path):
        return None
    return json.load(open(path)).get("tokens")


def cpu_reference_run(model_dir: str, prompt, decode_steps: int, steps: int,
                      warmup: int):
    """Time the reference's own forward pass (oracle/_ref) on the host cores:
    per step a full prefill of `prompt` then `decode_steps` greedy steps."""
    import numpy as np
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    os.environ.setdefault("OMP_WAIT_POLICY", "ACTIVE")
    os.environ.setdefault("OMP_PROC_BIND", "close")
    import oracle
    if oracle.reference_available():
        m, kind = oracle.Reference(model_dir), "reference"
    else:
        m, kind = oracle.Restatement(model_dir), "port"
    pre, dec = 0.0, 0.0
    for i in range(warmup + steps):
        m.reset()
        t0 = time.perf_counter()
        logits = m.predict(prompt, 1)[0]
        t1 = time.perf_counter()
        tok = int(np.argmax(logits))
        for _ in range(decode_steps):
            tok = int(np.argmax(m.predict([tok], 1)[0]))
        t2 = time.perf_counter()
        if i >= warmup:
            pre += t1 - t0
            dec += t2 - t1
    m.free()
    return {"kind": kind, "cores": int(os.environ["OMP_NUM_THREADS"]),
            "prefill_tok_s": steps * len(prompt) / pre,
            "decode_tok_s": steps * decode_steps / dec}


def main():
    args = parse_args()
    dist = Dist()
    from strasgpt_b200 import configs, synth
    cfg = configs.get(args.config)
    mdir = os.path.join(MODEL_CACHE, f"{cfg.name}_s0")
    workload = {"workload": f"{cfg.name}: prompt {cfg.prompt_len} + {cfg.steps} greedy "
                            f"decode steps, batch 1",
                "model": cfg.name, "global_batch": 1, "seq_len": cfg.prompt_len + cfg.steps,
                "parallelism": f"tp{args.gpus}" if args.gpus > 1 else "tp1",
                "l2": "weights (>= 1.1 GB) exceed the 126 MB L2 between steps"}
    if dist.rank == 0:
        synth.write_model(mdir, cfg, seed=0)
    dist.barrier()
    prompt = synth.prompt_tokens(cfg, seed=0)

    if args.impl == "reference":
        if dist.rank != 0:
            dist.close()
            return
        dec_steps = min(cfg.steps, 8)
        r = cpu_reference_run(mdir, prompt, dec_steps, args.steps, args.warmup)
        sample = (f"per step: prefill {cfg.prompt_len} tokens + {dec_steps} greedy "
                  f"decode steps (of {cfg.steps})")
        print(json.dumps({
            "impl": "reference", "metric": "decode tok/s", "value": r["decode_tok_s"],
            "unit": "tok/s", "higher_is_better": True, "n_gpus": 0, "steps": args.steps,
            "warmup": args.warmup, "dtype": "f32", "data": "synthetic",
            "prefill": {"value": r["prefill_tok_s"], "unit": "tok/s"},
            "config": workload,
            "cpu_baseline": {"value": r["decode_tok_s"], "unit": "tok/s",
                             "cores": r["cores"], "kind": r["kind"], "sample": sample},
            "e2e": {"value": r["decode_tok_s"], "unit": "tok/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        dist.close()
        return

    import numpy as np
    from strasgpt_b200 import Transformer
    m = Transformer(mdir, rank=dist.rank, world=dist.world, device=dist.local)
    S, P = cfg.steps, cfg.prompt_len
    toks = None
    for _ in range(args.warmup):
        m.reset()
        toks, _ = m.generate_greedy(prompt, S)
    dist.barrier()
    clocks = Clocks(dist.local)
    clocks.start()
    pre_ms = dec_ms = 0.0
    launches = dec_launches = 0
    for _ in range(args.steps):
        m.reset()
        toks, tm = m.generate_greedy(prompt, S)
        pre_ms += tm.prefill_ms
        dec_ms += tm.decode_ms
        launches += tm.kernel_launches
        dec_launches = tm.decode_launches
    clk = clocks.stop()
    dist.barrier()
    pre_ms, dec_ms = dist.max([pre_ms, dec_ms])
    value = args.steps * S / (dec_ms / 1e3)
    prefill = args.steps * P / (pre_ms / 1e3)

    peaks = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    # Whole decode step: algorithmic bytes (weights once + KV read/write at
    # the mean position) / device time per token.
    mean_pos = P + (S - 1) / 2.0
    step_bytes = (cfg.decode_weight_bytes() + cfg.kv_bytes(int(mean_pos))) / args.gpus
    step_gbs = step_bytes / (dec_ms / 1e3 / (args.steps * S)) / 1e9

    # Per-kernel-family device time of eager decode steps (CUDA events
    # around every launch): explains the step when no persistent kernel runs.
    m.reset()
    first = int(np.argmax(m.predict(prompt, 1)[0]))
    prof = m.profile_decode(first, 16)
    mv = prof["matvec"]
    mv_gbs = mv["bytes"] / (mv["ms"] / 1e3) / 1e9 if mv["ms"] > 0 else None
    total_ms = sum(v["ms"] for v in prof.values())
    peak_source = "measured" if "fallback" not in peaks else "fallback"
    if dec_launches == 1:
        # One persistent kernel ran all S decode steps: its algorithmic bytes
        # per launch (S x step_bytes) over its CUDA-event duration.
        per_step_traffic = profiled_dram_bytes_per_step("k_mega_decode", cfg.name)
        roofline = {"bound": "hbm", "kernel": "k_mega_decode", "achieved": step_gbs,
                    "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                    "peak_source": peak_source,
                    "bytes_per_launch": step_bytes * S,
                    "launch_ms": dec_ms / args.steps,
                    "traffic": per_step_traffic * S if per_step_traffic else None,
                    "traffic_source": "profiles/k_mega_decode_" + cfg.name + ".md"
                    if per_step_traffic else None,
                    "share_of_decode": 1.0}
    else:
        roofline = {"bound": "hbm", "kernel": "decode matvec family", "achieved": mv_gbs,
                    "peak": hbm, "unit": "GB/s", "frac": (mv_gbs / hbm) if mv_gbs else None,
                    "peak_source": peak_source, "traffic": None,
                    "share_of_decode": mv["ms"] / total_ms if total_ms else None,
                    "launches_per_token": mv["launches"] / 16.0}

    e2e = None
    if not args.no_e2e:
        # The reference-facing API: transformer_predict with host token ids
        # and host logits every step, host argmax (as strasgpt.c samples).
        m.reset()
        dist.barrier()
        t0 = time.perf_counter()
        tok = int(np.argmax(m.predict(prompt, 1)[0]))
        t1 = time.perf_counter()
        for _ in range(S):
            tok = int(np.argmax(m.predict([tok], 1)[0]))
        t2 = time.perf_counter()
        pre_s, dec_s = dist.max([t1 - t0, t2 - t1])
        e2e = {"value": S / dec_s, "unit": "tok/s",
               "prefill_tok_s": P / pre_s,
               "h2d_bytes_per_step": (P + S) * 4,
               "d2h_bytes_per_step": (S + 1) * cfg.vocab * 4}

    cpu = None
    if not args.no_cpu_baseline and dist.world == 1 and dist.rank == 0:
        r = cpu_reference_run(mdir, prompt, 8, 1, 0)
        cpu = {"value": r["decode_tok_s"], "unit": "tok/s", "cores": r["cores"],
               "kind": r["kind"], "prefill_tok_s": r["prefill_tok_s"],
               "sample": f"one request: prefill {P} tokens + 8 greedy decode steps"}

    gold = golden_tokens(cfg.name)
    if dist.rank == 0:
        line = {
            "metric": "decode tok/s", "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": (pre_ms + dec_ms) / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (random-init bf16 weights, seeded prompt)",
            "config": workload,
            "prefill": {"value": prefill, "unit": "tok/s",
                        "tflops": P * cfg.prefill_flops_per_token() / (pre_ms / args.steps / 1e3) / 1e12},
            "decode_step": {"achieved_gbs": step_gbs, "peak_gbs": hbm,
                            "frac": step_gbs / hbm, "bytes_per_token": step_bytes},
            "roofline": roofline,
            "eager_decode_profile": {
                "note": "per-launch CUDA events of 16 eager decode steps (no persistent kernel)",
                "matvec_gbs": mv_gbs,
                "ms_per_token": {k: v["ms"] / 16.0 for k, v in prof.items()}},
            "e2e": e2e, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": launches,
            "tokens_match_golden": (list(toks) == gold) if gold else None,
        }
        print(json.dumps(line), flush=True)
    m.free()
    dist.close()


if __name__ == "__main__":
    main()
