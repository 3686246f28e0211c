"""Greedy generation on a synthetic configuration:

    python -m strasgpt_b200 --config c2_qwen3_0p6b --steps 128 --repeat 2

writes the random-init model once (cached under $STRASGPT_MODEL_CACHE,
default /tmp/strasgpt_models), then runs `--repeat` requests of prompt +
`--steps` greedy decode steps through transformer_generate_greedy and prints
one JSON line per request with the device times. `--steps 0` runs the
prompt (prefill) alone."""
import argparse
import json
import os

from . import configs, synth
from .runtime import Transformer


def main():
    p = argparse.ArgumentParser(prog="python -m strasgpt_b200")
    p.add_argument("--config", default="c2_qwen3_0p6b")
    p.add_argument("--steps", type=int, default=None, help="decode steps (default: the config's)")
    p.add_argument("--repeat", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args()
    cfg = configs.get(args.config)
    cache = os.environ.get("STRASGPT_MODEL_CACHE", "/tmp/strasgpt_models")
    mdir = synth.write_model(os.path.join(cache, f"{cfg.name}_s{args.seed}"), cfg, seed=args.seed)
    steps = cfg.steps if args.steps is None else args.steps
    prompt = synth.prompt_tokens(cfg, seed=args.seed)
    m = Transformer(mdir)
    for i in range(args.repeat):
        m.reset()
        toks, tm = m.generate_greedy(prompt, steps)
        print(json.dumps({
            "request": i, "config": cfg.name, "prompt": len(prompt), "steps": steps,
            "prefill_ms": tm.prefill_ms, "decode_ms": tm.decode_ms,
            "prefill_tok_s": len(prompt) / (tm.prefill_ms / 1e3) if tm.prefill_ms else None,
            "decode_tok_s": steps / (tm.decode_ms / 1e3) if steps and tm.decode_ms else None,
            "kernel_launches": tm.kernel_launches, "tokens": [int(t) for t in toks[:16]],
        }), flush=True)
    m.free()


if __name__ == "__main__":
    main()
