"""Time the upstream megakernel (built unmodified into oracle/_ref/) on a GPU.

Records, for the two batch-1 workloads of the benchmark configuration, the
upstream implementation's own decode throughput through its own ops:

* config 1: seeded 16-token prompt, upstream ``decode`` for the first 15
  tokens, then ``generate_nosync(prompt[-1], 64)`` at position 15 (timed);
* config 2: seeded 1920-token prompt prefilled with upstream ``decode`` steps
  (untimed), then ``generate_nosync(first, 128)`` at position 1920 (timed).

Times are CUDA events around the op call plus a synchronisation (the upstream
launcher already synchronises once per step).  Prints one JSON line.
Usage: python tests/golden/time_reference_gpu.py
"""
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import RefDecoder, _load_ref  # noqa: E402


def main():
    mk = _load_ref("qwen_megakernel_C")
    dec = RefDecoder(mk, seed=0, num_layers=28)
    out = {}
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 151936, (16,), generator=g).tolist()
    for i, t in enumerate(prompt[:-1]):
        dec.step(t, i)
    for _ in range(2):
        dec.gen(prompt[-1], 15, 64)
    t0 = time.perf_counter()
    dec.gen(prompt[-1], 15, 64)
    dt = time.perf_counter() - t0
    out["config1_generate64_tok_s"] = 64 / dt
    # single decode-step latency at position 16
    t0 = time.perf_counter()
    for i in range(20):
        dec.step(prompt[-1], 16 + i)
    out["decode_step_ms"] = (time.perf_counter() - t0) / 20 * 1000
    # config 2
    dec.kc.zero_()
    dec.vc.zero_()
    g = torch.Generator().manual_seed(1)  # same stream as bench.py's prompt
    g.manual_seed(0 + 1)
    prompt = torch.randint(0, 151936, (1920,), generator=g).tolist()
    t0 = time.perf_counter()
    first = None
    for i, t in enumerate(prompt):
        first = dec.step(t, i)
    out["prefill1920_s"] = time.perf_counter() - t0
    dec.gen(first, 1920, 128)
    t0 = time.perf_counter()
    toks = dec.gen(first, 1920, 128)
    dt = time.perf_counter() - t0
    out["config2_generate128_tok_s"] = 128 / dt
    out["config2_first_tokens"] = [int(x) for x in toks[:8]]
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
