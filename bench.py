#!/usr/bin/env python
"""Benchmark: greedy decode of a synthetic model through libstrasgpt.so.

Workload (default): the Llama-3.1-8B-shaped configuration C3 (2048-token
prompt, greedy decode, batch 1), the configuration the headline metric is
quoted on "at 1/2/4/8 GPUs" that fits one GPU. One STEP is one greedy decode
token at the positions right after the prompt. Printed on rank 0 as ONE
JSON line:
  value        decode tok/s, whole job (every rank works on the same token
               under tensor parallelism), device time: CUDA events on the
               library's stream around ONE persistent-kernel launch that runs
               exactly --steps tokens, weights resident in HBM;
  prefill      tok/s of the timed request's 2048-token prompt (CUDA events);
  e2e          decode tok/s through the reference-facing C ABI:
               transformer_predict with the token id in host memory and the
               full-vocabulary logits copied back to host memory every step,
               host argmax (as strasgpt.c samples), host wall clock;
  roofline     the persistent decode kernel's algorithmic bytes (weights once
               + KV cache at the timed positions) / its CUDA-event time,
               against the measured HBM copy bandwidth;
  cpu_baseline the reference's own forward pass (oracle/_ref, OpenMP, all
               host cores) on a bounded sample: a prefill of the prompt's
               first 128 tokens, then 8 greedy decode tokens.
`--impl reference` times the reference CPU implementation alone on rank 0:
one prefill of the prompt (reported as `prefill`), --warmup untimed decode
tokens, then --steps timed decode tokens (`value`).
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
CPU_DECODE_TOKENS = 8
CPU_PREFILL_TOKENS = 128


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["strasgpt", "reference"], default="strasgpt")
    p.add_argument("--config", default="c3_llama8b")
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
    """nvidia-smi samples (every 50 ms) while the GPU works."""
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
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # nvidia-smi takes a moment to start sampling; the GPU work that
            # follows must fall inside its window.
            time.sleep(1.0)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, loaded, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                if float(f[3]) > 250.0:
                    loaded.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        use = loaded or sm
        return {"sm_mhz": statistics.median(use) if use else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "samples_under_load": len(loaded),
                "window": "warm-up + timed request (prefill and decode)"}


def measured_peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def profiled_traffic_ratio(kernel: str, config: str):
    """DRAM bytes (read + write) over algorithmic bytes of `kernel` on
    `config`, from the committed ncu summary profiles/<kernel>_<config>.md
    (line `traffic_over_algorithmic: R`), or None."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_over_algorithmic:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


def golden_tokens(name: str):
    path = os.path.join(ROOT, "tests", "golden", f"{name}.json")
    if not os.path.exists(path):
        return None
    return json.load(open(path)).get("tokens")


def cpu_threads() -> int:
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    os.environ.setdefault("OMP_WAIT_POLICY", "ACTIVE")
    os.environ.setdefault("OMP_PROC_BIND", "close")
    return int(os.environ["OMP_NUM_THREADS"])


def cpu_reference_run(model_dir: str, prompt, warmup: int, steps: int) -> dict:
    """The reference's own forward pass (oracle/_ref) on the host cores: one
    prefill of `prompt`, `warmup` untimed greedy decode tokens, then `steps`
    timed ones (the restatement, kind "port", if the reference library is
    absent)."""
    import numpy as np
    cores = cpu_threads()
    import oracle
    if oracle.reference_available():
        m, kind = oracle.Reference(model_dir), "reference"
    else:
        m, kind = oracle.Restatement(model_dir), "port"
    m.reset()
    t0 = time.perf_counter()
    tok = int(np.argmax(m.predict(prompt, 1)[0]))
    t1 = time.perf_counter()
    for _ in range(warmup):
        tok = int(np.argmax(m.predict([tok], 1)[0]))
    t2 = time.perf_counter()
    for _ in range(steps):
        tok = int(np.argmax(m.predict([tok], 1)[0]))
    t3 = time.perf_counter()
    m.free()
    return {"kind": kind, "cores": cores, "prefill_tok_s": len(prompt) / (t1 - t0),
            "prefill_s": t1 - t0, "decode_tok_s": steps / (t3 - t2),
            "ms_per_token": (t3 - t2) / steps * 1e3}


def main():
    args = parse_args()
    dist = Dist()
    from strasgpt_b200 import configs, synth
    cfg = configs.get(args.config)
    mdir = os.path.join(MODEL_CACHE, f"{cfg.name}_s0")
    P, K, W = cfg.prompt_len, args.steps, args.warmup
    workload = {"workload": f"{cfg.name}: {P}-token prompt, then greedy decode, batch 1; "
                            f"one step = one decode token at positions {P}..{P + K - 1}",
                "model": cfg.name, "global_batch": 1, "seq_len": P + K,
                "prompt_len": P, "parallelism": f"tp{args.gpus}",
                "l2": f"weights ({cfg.decode_weight_bytes() / 1e9:.1f} GB per token) "
                      "exceed the 126 MB L2 between steps"}
    if dist.rank == 0:
        synth.write_model(mdir, cfg, seed=0)
    dist.barrier()
    prompt = synth.prompt_tokens(cfg, seed=0)

    if args.impl == "reference":
        if dist.rank != 0:
            dist.close()
            return
        r = cpu_reference_run(mdir, prompt, W, K)
        sample = (f"one prefill of the {P}-token prompt ({r['prefill_s']:.1f} s), {W} untimed "
                  f"and {K} timed greedy decode tokens")
        print(json.dumps({
            "impl": "reference", "metric": "decode tok/s", "value": r["decode_tok_s"],
            "unit": "tok/s", "higher_is_better": True, "n_gpus": 0, "steps": K,
            "warmup": W, "ms_per_step": r["ms_per_token"], "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
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
    clocks = Clocks(dist.local)
    clocks.start()
    # W untimed warm-up decode tokens after the prompt.
    m.reset()
    m.generate_greedy(prompt, W)
    # The timed request: the prompt (its own events: `prefill`), then ONE
    # persistent launch of exactly K decode tokens between two events.
    m.reset()
    dist.barrier()
    toks, tm = m.generate_greedy(prompt, K)
    dist.barrier()
    clk = clocks.stop()
    pre_ms, dec_ms = dist.max([tm.prefill_ms, tm.decode_ms])
    value = K / (dec_ms / 1e3)
    prefill = P / (pre_ms / 1e3)

    peaks = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_source = "measured" if "fallback" not in peaks else "fallback"
    # Algorithmic bytes per token on one rank: its weight shard once, its
    # KV heads' cache rows [0, pos] read and row pos written, at the mean
    # timed position.
    mean_pos = P + (K - 1) / 2.0
    step_bytes = (cfg.decode_weight_bytes() + cfg.kv_bytes(int(round(mean_pos)))) / args.gpus
    step_gbs = step_bytes / (dec_ms / 1e3 / K) / 1e9
    ratio = profiled_traffic_ratio("k_mega_decode", cfg.name)
    roofline = {"bound": "hbm", "kernel": "k_mega_decode", "achieved": step_gbs,
                "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                "peak_source": peak_source,
                "bytes_per_launch": step_bytes * K, "launch_ms": dec_ms,
                "traffic": ratio * step_bytes * K if ratio else None,
                "traffic_source": (f"profiles/k_mega_decode_{cfg.name}.md: DRAM bytes / "
                                   "algorithmic bytes of a captured launch" if ratio else None),
                "launches_in_timed_region": int(tm.decode_launches)}

    e2e = None
    if not args.no_e2e:
        # The reference-facing API: one transformer_predict per token, the
        # token id from host memory, the logits [V] back into host memory,
        # host argmax (as strasgpt.c samples).
        m.reset()
        t0 = time.perf_counter()
        tok = int(np.argmax(m.predict(prompt, 1)[0]))
        t1 = time.perf_counter()
        for _ in range(W):
            tok = int(np.argmax(m.predict([tok], 1)[0]))
        dist.barrier()
        t2 = time.perf_counter()
        for _ in range(K):
            tok = int(np.argmax(m.predict([tok], 1)[0]))
        t3 = time.perf_counter()
        pre_s, dec_s = dist.max([t1 - t0, t3 - t2])
        e2e = {"value": K / dec_s, "unit": "tok/s", "prefill_tok_s": P / pre_s,
               "h2d_bytes_per_step": 4, "d2h_bytes_per_step": cfg.vocab * 4,
               "path": "transformer_predict(1 token, 1 logits row) + host argmax"}
    m.free()

    cpu = None
    if not args.no_cpu_baseline and dist.world == 1 and dist.rank == 0:
        n = min(P, CPU_PREFILL_TOKENS)
        r = cpu_reference_run(mdir, prompt[:n], 0, CPU_DECODE_TOKENS)
        cpu = {"value": r["decode_tok_s"], "unit": "tok/s", "cores": r["cores"],
               "kind": r["kind"], "prefill_tok_s": r["prefill_tok_s"],
               "sample": f"a prefill of the prompt's first {n} tokens ({r['prefill_s']:.1f} s), "
                         f"then {CPU_DECODE_TOKENS} greedy decode tokens at positions "
                         f"{n}..{n + CPU_DECODE_TOKENS - 1} (weights read once per token: "
                         f"{cfg.decode_weight_bytes() / 1e9:.2f} GB of the "
                         f"{(cfg.decode_weight_bytes() + cfg.kv_bytes(P)) / 1e9:.2f} GB a "
                         f"token at position {P} reads); `--impl reference` times the "
                         f"full prompt"}

    gold = golden_tokens(cfg.name)
    if dist.rank == 0:
        line = {
            "metric": "decode tok/s", "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": K, "warmup": W,
            "ms_per_step": dec_ms / K,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (random-init bf16 weights, seeded prompt)",
            "config": workload,
            "prefill": {"value": prefill, "unit": "tok/s", "ms": pre_ms,
                        "tflops": P * cfg.prefill_flops_per_token() / (pre_ms / 1e3) / 1e12,
                        "launches": int(tm.kernel_launches - tm.decode_launches)},
            "decode_step": {"achieved_gbs": step_gbs, "peak_gbs": hbm,
                            "frac": step_gbs / hbm, "bytes_per_token": step_bytes,
                            "frac_of_8tbs": step_gbs / 8000.0},
            "roofline": roofline,
            "e2e": e2e, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": int(tm.decode_launches),
            "tokens_match_golden": (list(toks) == gold[:K + 1]) if gold else None,
        }
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
