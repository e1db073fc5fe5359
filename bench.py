"""Benchmark of the B200 batch-1 greedy decode path (one JSON line on rank 0).

Workload: Qwen3-0.6B architecture with seeded
random-init fp16 weights, one sequence, a seeded uniform-random 1920-token
prompt prefilled with decode steps (untimed), then greedy decode at positions
1920..2047.  One bench "step" = one ``generate_nosync`` of 128 tokens from
position 1920 (the KV cache of the prompt stays resident; positions
1920..2047 are rewritten with identical values every step).  Weights are
1.19 GB per token, far larger than the 126 MB L2, so no L2 flush is needed.

``value``  tokens/s of the whole job (all ranks), device-timed with CUDA
           events on the launching stream, max over ranks.
``e2e``    the same metric through the public Python API
           (``Decoder.generate_nosync`` + a device->host read of the 128 output
           tokens), host wall clock, the first token passed from the host.
``roofline`` algorithmic bytes per launch (weights + KV read per token, summed
           over the 128 tokens) / average launch duration, against the measured
           HBM copy bandwidth.
``cpu_baseline`` the CPU oracle (a C restatement of the upstream algorithm)
           on this host's cores, on a bounded sample of the same workload.
``cpu_baseline_hf`` the comparator upstream's own benchmark uses: HF
           transformers Qwen3ForCausalLM in fp32 on the host cores (thread
           count and torch.get_num_threads() recorded), a bounded sample.
``batched`` the config-4 result (below) at the same number of GPUs, measured
           after the decode workload in the same run, so that every default
           run -- the 1/2/4/8-GPU scaling runs included -- carries the batched
           tok/s; ``--no-batched`` skips it.

Multi-GPU: single-sequence decode does not shard; ``--gpus N`` runs N
independent replicas (one process per GPU) and reports their aggregate.

``--workload batched``: 256 independent sequences per
GPU, seeded prompt lengths uniform in [32, 512] and uniform token ids,
prefilled with batched steps (untimed); one bench step = one batched greedy
step of all 256 sequences (256 tokens).  Sequences are sharded per GPU (seeds
offset by rank) with no collective; ``value`` is the aggregate tok/s.  Its CPU
figures (``cpu_baseline``: the C oracle; ``cpu_baseline_hf``: HF fp32) decode
one sequence at the workload's mean position and are marked extrapolated.
``--workload ops`` also reports ``cpu_baseline_torch``: the same chain as fp32
torch ops on the host cores.
``--impl reference`` times the upstream algorithm's CPU restatement (the C
oracle, kind "port") with all host threads, rank 0 only; each of its steps is a
sample of 16 consecutive tokens of config 2's per-token work.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen0.6b_b200")
sys.path.insert(0, PKG)

PROMPT_LEN = 1920
GEN = 128
SEED = 0
W_BYTES = 2 * (440_466_432 + 1_024) + 2 * 155_582_464   # weights streamed per token
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 2                   # K+V bytes per cached position
METRIC = "batch-1 decode tok/s + % HBM roofline; batched tok/s at 1/2/4/8 B200"


def algorithmic_bytes(start: int, n: int) -> int:
    """Bytes one launch of n greedy steps from `start` must read: all weights
    once per token plus the K/V of every attended position (pos+1 per step)."""
    return sum(W_BYTES + KV_BYTES_PER_POS * (p + 1) for p in range(start, start + n))


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def profile_traffic() -> float | None:
    """DRAM bytes per decode-kernel launch from the committed ncu summary, scaled
    to one 128-token launch (the line 'traffic_bytes_per_token: X')."""
    path = os.path.join(ROOT, "profiles", "decode_kernel_longctx.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_token:"):
                return float(line.split(":", 1)[1]) * GEN
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return self._one_shot()
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}

    def _one_shot(self) -> dict | None:
        """A timed region shorter than the sampling interval: one reading right
        after it (marked as such)."""
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,"
                                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                                  "--format=csv,noheader,nounits", "-i", str(self.gpu)],
                                 capture_output=True, text=True, timeout=20).stdout.strip().split(",")
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            return {"sm_mhz": float(out[0]), "sm_max_mhz": float(out[1]),
                    "reasons": [n for n, v in zip(names, out[2:6]) if v.strip().lower() == "active"],
                    "samples": 1, "note": "timed region shorter than the sampling interval: read right after it"}
        except (OSError, ValueError, IndexError, subprocess.TimeoutExpired):
            return None


def cpu_baseline(weights_cpu: dict, seconds: float = 12.0, start: int = PROMPT_LEN) -> dict:
    """CPU oracle, 28 layers at positions start.. over a seeded random KV cache
    of `start` positions (the per-token work equals the GPU workload's)."""
    from oracle.oracle import OracleModel

    threads = len(os.sched_getaffinity(0))
    orc = OracleModel(weights_cpu, nthreads=threads)
    g = torch.Generator().manual_seed(1)
    orc.k_cache[:, :, :start] = torch.randn(28, 8, start, 128, generator=g).half()
    orc.v_cache[:, :, :start] = torch.randn(28, 8, start, 128, generator=g).half()
    orc.position = start
    tok, n = 1, 0
    orc.step(tok)  # warm-up
    t0 = time.perf_counter()
    while (time.perf_counter() - t0 < seconds or n < 3) and orc.position < 2048:
        tok = orc.step(tok)["token"]
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} greedy steps of the 28-layer CPU oracle at positions {start + 1}.."
                      f"{start + n} over a seeded random {start}-position KV cache ({dt:.1f} s)"}


REF_TOKENS_PER_STEP = 16


def run_reference_arm(args, rank: int) -> None:
    """The upstream algorithm's CPU restatement (the C oracle, all host
    threads) on config 2's per-token work.  One reference "step" is a sample of
    REF_TOKENS_PER_STEP consecutive greedy tokens at positions 1920.. over a
    seeded 1920-position KV cache: the line's steps, ms_per_step and value
    describe exactly those timed tokens (the GPU arm's step is 128 tokens)."""
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    from oracle.oracle import OracleModel
    from qwen_weights import synthetic_weights

    w = synthetic_weights(seed=SEED)
    threads = len(os.sched_getaffinity(0))
    orc = OracleModel(w, nthreads=threads)
    g = torch.Generator().manual_seed(1)
    orc.k_cache[:, :, :PROMPT_LEN] = torch.randn(28, 8, PROMPT_LEN, 128, generator=g).half()
    orc.v_cache[:, :, :PROMPT_LEN] = torch.randn(28, 8, PROMPT_LEN, 128, generator=g).half()

    def sample(step: int) -> float:
        # Positions wrap inside the 128-token range, so any K stays in bounds.
        orc.position = PROMPT_LEN + (step * REF_TOKENS_PER_STEP) % (GEN - REF_TOKENS_PER_STEP + 1)
        tok = 1
        t0 = time.perf_counter()
        for _ in range(REF_TOKENS_PER_STEP):
            tok = orc.step(tok)["token"]
        return time.perf_counter() - t0

    for i in range(args.warmup):
        sample(i)
    secs = [sample(args.warmup + i) for i in range(args.steps)]
    total = sum(secs)
    v = REF_TOKENS_PER_STEP * args.steps / total
    desc = (f"{args.steps} samples of {REF_TOKENS_PER_STEP} consecutive greedy tokens of the 28-layer "
            f"C oracle at positions {PROMPT_LEN}..{PROMPT_LEN + GEN - 1} over a seeded random "
            f"{PROMPT_LEN}-position KV cache, {threads} threads ({total:.1f} s timed)")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config 2 per-token work: batch-1 greedy decode at positions "
                                   f"1920..2047; one step = a sample of {REF_TOKENS_PER_STEP} tokens "
                                   "(the GPU arm's step is 128 tokens)",
                       "batch": 1, "prompt_len": PROMPT_LEN, "gen_steps": GEN,
                       "tokens_per_step": REF_TOKENS_PER_STEP, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def hf_cpu_baseline(weights_cpu: dict, start: int = PROMPT_LEN, seconds: float = 10.0) -> dict:
    """The comparator upstream's own benchmark uses (Model/benchmark.py:48-84):
    HF transformers Qwen3ForCausalLM in fp32 on the host cores, greedy decode
    with the KV cache after an untimed prefill of a seeded `start`-token
    prompt; a bounded sample of decode steps is timed."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from qwen_weights import hf_state_dict

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                      num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True,
                      max_position_embeddings=2048, attention_bias=False)
    # Built on the meta device (no random init of 0.6 B parameters), then
    # materialised and filled from the seeded weights; the rotary table is a
    # non-persistent buffer, so it is rebuilt rather than loaded.
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    with torch.device("meta"):
        m = Qwen3ForCausalLM(cfg)
    m.load_state_dict(hf_state_dict(weights_cpu), strict=False, assign=True)
    m.model.rotary_emb = Qwen3RotaryEmbedding(config=cfg)
    m = m.float().eval()
    g = torch.Generator().manual_seed(SEED + 1)
    ids = torch.randint(0, 151936, (1, start), generator=g)
    with torch.no_grad():
        t0 = time.perf_counter()
        out = m(ids, use_cache=True)
        prefill_s = time.perf_counter() - t0
        past, tok = out.past_key_values, out.logits[:, -1:].argmax(-1)
        n, t0 = 0, time.perf_counter()
        while (time.perf_counter() - t0 < seconds or n < 3) and start + n < 2048:
            out = m(tok, past_key_values=past, use_cache=True)
            past, tok = out.past_key_values, out.logits[:, -1:].argmax(-1)
            n += 1
        dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "torch_threads": torch.get_num_threads(),
            "kind": "hf-fp32",
            "sample": f"{n} greedy decode steps of HF Qwen3ForCausalLM fp32 (transformers "
                      f"{__import__('transformers').__version__}) at positions {start}..{start + n - 1} "
                      f"after a {start}-token prefill ({prefill_s:.1f} s, untimed), {dt:.1f} s timed"}


def batched_cpu_baseline(weights_cpu: dict, pos: int, seconds: float = 10.0) -> dict:
    """CPU oracle on one sequence at the batched workload's mean position (the
    oracle decodes one sequence at a time; its tok/s is the CPU rate for this
    per-token work), a bounded sample."""
    cb = cpu_baseline(weights_cpu, seconds=seconds, start=pos)
    cb["sample"] = ("one sequence, " + cb["sample"] + f" (batched workload mean position {pos}); "
                    "extrapolated to the batch: the CPU decodes the sequences one after another, "
                    "so its tok/s for the batch is this one sequence's rate")
    cb["extrapolated"] = True
    return cb


def run_batched(args, world: int, rank: int, local: int, dev, dist) -> None:
    line = batched_line(args, world, rank, local, dev, dist)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def batched_line(args, world: int, rank: int, local: int, dev, dist, with_cpu: bool = True) -> dict:
    """Config 4: batched greedy decode of independent sequences per GPU."""
    from batched import BatchedDecoder
    from qwen_weights import synthetic_weights

    n = args.seqs
    w_cpu = synthetic_weights(seed=SEED, num_layers=args.layers)
    g = torch.Generator().manual_seed(1000 + rank)
    lengths = torch.randint(32, 513, (n,), generator=g).tolist()
    prompts = [torch.randint(0, 151936, (ln,), generator=g).tolist() for ln in lengths]
    total_steps = args.warmup + args.steps
    num_pages = sum((ln + total_steps + 127) // 128 for ln in lengths) if args.paged else None
    bd = BatchedDecoder(w_cpu, num_seqs=n, max_rows=n, device=dev, num_layers=args.layers,
                        paged=args.paged, num_pages=num_pages)
    kv_bytes = 2 * bd.k_pool.numel() * 2
    bd.prefill(prompts)
    for i, ln in enumerate(lengths):
        bd.reserve(i, ln - 1 + total_steps - 1)
    ids = torch.arange(n, dtype=torch.int32, device=dev)
    pos0 = torch.tensor([ln - 1 for ln in lengths], dtype=torch.int32, device=dev)
    tok0 = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
    start_max = max(lengths) - 1
    assert start_max + 2 * total_steps < 2048

    # Device-timed run: warm-up steps, then the timed steps, continuing the generation.
    outs = [torch.empty(n, dtype=torch.int32, device=dev) for _ in range(total_steps)]
    stream = torch.cuda.current_stream(dev)
    pos, tok = pos0.clone(), tok0.clone()
    for s in range(args.warmup):
        tok = bd.step(ids, pos, tok, start_max + s, out=outs[s])
        pos = pos + 1
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos_list = []
    if args.profile:
        torch.cuda.cudart().cudaProfilerStart()
    t_start.record(stream)
    for i in range(args.steps):
        s = args.warmup + i
        ev[i][0].record(stream)
        tok = bd.step(ids, pos, tok, start_max + s, out=outs[s])
        ev[i][1].record(stream)
        pos_list.append(pos)
        pos = pos + 1
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStop()
    clk = clocks.stop()
    if dist is not None:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    assert bd.status() == 0, "device-side error in the batched steps"
    ref_tokens = [o.cpu() for o in outs]

    # End to end through BatchedDecoder.step: inputs from pinned host memory,
    # tokens back to the host, every step (same positions: the cache rows are
    # rewritten with identical values, so the tokens must repeat exactly).
    h_in = torch.empty(3, n, dtype=torch.int32).pin_memory()
    h_out = torch.empty(n, dtype=torch.int32).pin_memory()
    d_in = torch.empty(3, n, dtype=torch.int32, device=dev)
    pos, tok_h = pos0.cpu(), tok0.cpu()
    for s in range(args.warmup):
        pos = pos + 1
        tok_h = ref_tokens[s]
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    h_in[0].copy_(ids.cpu())
    for i in range(args.steps):
        s = args.warmup + i
        h_in[1].copy_(pos)
        h_in[2].copy_(tok_h)
        d_in.copy_(h_in, non_blocking=True)
        out = bd.step(d_in[0], d_in[1], d_in[2], start_max + s)
        h_out.copy_(out, non_blocking=True)
        stream.synchronize()
        tok_h = h_out.clone()
        assert torch.equal(tok_h, ref_tokens[s]), "e2e tokens differ from the device-timed run"
        pos = pos + 1
    e2e_ms = 1000.0 * (time.perf_counter() - t0)

    if dist is not None:
        t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = world * n * args.steps / (total_ms / 1000.0)
    e2e_value = world * n * args.steps / (e2e_ms / 1000.0)
    # Algorithmic bytes per step: every weight once (layers + tied lm_head)
    # plus the K/V of every attended position of every sequence.
    w_bytes = W_BYTES if args.layers == 28 else W_BYTES - 2 * (28 - args.layers) * 15_728_640 - 2 * (28 - args.layers) * 2304
    kv_pos = KV_BYTES_PER_POS * args.layers // 28
    alg = [w_bytes + kv_pos * int((p + 1).sum()) for p in pos_list]
    avg_alg = statistics.mean(alg)
    avg_step_s = statistics.mean(step_ms) / 1000.0
    peaks = measured_peaks()
    achieved = avg_alg / avg_step_s / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded random-init weights, uniform-random token ids)",
        "config": {"workload": f"config 4: batched greedy decode, {n} independent sequences per GPU, "
                               "prompt lengths uniform in [32, 512] (prefill untimed), one step = "
                               f"one token for each of the {n} sequences",
                   "batch": n, "prompt_len": "uniform [32, 512]", "gen_steps": args.steps,
                   "layers": args.layers if args.layers != 28 else None,
                   "parallelism": f"sequence shards x{world}" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2 ({avg_alg / 1e9:.1f} GB of weights + KV read per step); no flush",
                   "kv": (f"paged: {bd.num_pages} pages of 128 tokens, {kv_bytes / 1e9:.1f} GB "
                          f"(contiguous pools: {2 * n * args.layers * 8 * 2048 * 128 * 2 / 1e9:.1f} GB)"
                          if args.paged else f"contiguous per-sequence pools, {kv_bytes / 1e9:.1f} GB")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_src": peaks["src"], "traffic": None,
                     "algorithmic_bytes_per_step": avg_alg, "avg_step_ms": avg_step_s * 1000.0},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 3 * 4 * n,
                "d2h_bytes_per_step": 4 * n},
        "gpu_launches": args.steps * (args.layers * 9 + 3),  # 9 kernels per layer, 3 per step
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and with_cpu:
        mean_pos = int(statistics.mean(int(p.float().mean()) for p in pos_list))
        line["cpu_baseline"] = batched_cpu_baseline(w_cpu, mean_pos)
        if not args.no_hf_baseline and args.layers == 28:
            hf = hf_cpu_baseline(w_cpu, start=mean_pos, seconds=5.0)
            hf["sample"] = ("one sequence, " + hf["sample"] + f" (batched workload mean position {mean_pos}); "
                            "extrapolated to the batch: the CPU decodes the sequences one after another")
            hf["extrapolated"] = True
            line["cpu_baseline_hf"] = hf
    bd.close()
    return line


def torch_ops_cpu_baseline(x, w, wg, wu, wd, eps: float, seconds: float = 5.0) -> dict:
    """The config-3 chain as fp32 torch ops on the host cores: RMSNorm, then
    silu(x Wg) * (x Wu) and the down projection (weights in the upstream
    [H, I] / [I, H] layout), a bounded sample of calls."""
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    xf, wf, g, u, d = (t.float() for t in (x, w, wg, wu, wd))

    def call():
        xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * wf
        return (torch.nn.functional.silu(xn @ g) * (xn @ u)) @ d

    call()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 3:
        call()
        n += 1
    dt = time.perf_counter() - t0
    rows = x.shape[0]
    return {"value": rows * n / dt, "unit": "rows/s", "cores": threads, "torch_threads": torch.get_num_threads(),
            "kind": "torch-fp32",
            "sample": f"{n} calls of RMSNorm + SwiGLU + down projection as fp32 torch ops on {rows} rows ({dt:.1f} s)"}


def run_ops(args, world: int, rank: int, local: int, dev, dist) -> None:
    """Config 3: RMSNorm over [B, 1024] followed by the fused SwiGLU + down
    projection (the upstream Tools/rmsnorm + Tools/swiglu forward chain, fp16
    accumulation reproduced bit for bit).  One step = one call on B rows; 8
    weight sets rotate so that more than the L2 capacity is in play."""
    import swiglu_fused
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    from inputs import OPS_CASE, ops_inputs

    B = args.batch
    x, w, _, wg, wu, wd = (t.to(dev) for t in ops_inputs(B))
    sets = [(wg.clone(), wu.clone(), wd.clone()) for _ in range(8)]
    eps = OPS_CASE["eps"]
    stream = torch.cuda.current_stream(dev)
    exact = True if args.exact else None  # None: tensor cores from 64 rows on
    for i in range(args.warmup):
        swiglu_fused.rmsnorm_forward_down(x, w, eps, *sets[i % 8], exact=exact)
    ref = swiglu_fused.rmsnorm_forward_down(x, w, eps, *sets[0], exact=exact)[0].clone()
    torch.cuda.synchronize(dev)
    # The calls are timed as a CUDA graph of 8 calls (one per weight set), as a
    # serving loop would issue them: eager calls from Python are bound by the
    # host (~35 us per call), the kernels are not.  e2e below stays eager.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(8):
            swiglu_fused.rmsnorm_forward_down(x, w, eps, *sets[i], exact=exact)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(1, -(-args.steps // 8))
    steps = 8 * reps
    if dist is not None:
        dist.barrier()
    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStart()
    t_start.record(stream)
    for i in range(reps):
        ev[i][0].record(stream)
        graph.replay()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStop()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) / 8.0 for a, b in ev]
    h_x = x.cpu().pin_memory()
    h_y = torch.empty(B, 1024, dtype=torch.float16).pin_memory()
    d_x = torch.empty_like(x)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        d_x.copy_(h_x, non_blocking=True)
        h_y.copy_(swiglu_fused.rmsnorm_forward_down(d_x, w, eps, *sets[0], exact=exact)[0], non_blocking=True)
        stream.synchronize()
    e2e_ms = 1000.0 * (time.perf_counter() - t0)
    assert torch.equal(h_y, ref.cpu()), "non-deterministic operator output"
    if dist is not None:
        t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = world * B * steps / (total_ms / 1000.0)
    e2e_value = world * B * args.steps / (e2e_ms / 1000.0)
    alg = 3 * 1024 * 3072 * 2 + 1024 * 2 + 4 * B * 1024
    tc = not args.exact and B >= 64
    avg_step_s = statistics.mean(step_ms) / 1000.0
    peaks = measured_peaks()
    achieved = alg / avg_step_s / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": total_ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (x ~ N(0,1), norm weight ~ N(1,0.1), W ~ N(0,0.02))",
        "config": {"workload": f"config 3: RMSNorm + SwiGLU + down projection on [{B}, 1024], "
                               + ("tcgen05 GEMMs with fp32 accumulation" if tc else
                                  "upstream fp16 accumulation order reproduced (bit-exact)"),
                   "batch": B, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "8 weight sets of 18.9 MB rotate (151 MB > L2)",
                   "launch": "CUDA graph of 8 calls (one per weight set), replayed steps / 8 times"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_src": peaks["src"], "traffic": None,
                     "algorithmic_bytes_per_step": alg, "avg_step_ms": avg_step_s * 1000.0,
                     "note": ("two tcgen05 GEMMs (gate|up with the SwiGLU epilogue, down with K split "
                              "over a cluster) after the RMSNorm kernel" if tc else
                              "the serial fp16 chains (1024 + 3072 dependent adds) bound small batches")},
        "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": B * 2048,
                "d2h_bytes_per_step": B * 2048},
        "gpu_launches": steps * (4 if tc else 3),  # RMSNorm, gate|up, down (+ split-K reduction on the tensor cores)
        "clocks": clk,
    }
    if tc:
        line["tflops"] = 2 * 3 * 1024 * 3072 * B / avg_step_s / 1e12
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        threads = len(os.sched_getaffinity(0))
        xs, ws_ = x.cpu(), w.cpu()
        wgc, wuc, wdc = wg.cpu(), wu.cpu(), wd.cpu()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 or n < 1:
            nrm, _ = O.rmsnorm_forward(xs, ws_, eps)
            O.swiglu_forward_down(nrm.view(B, 1, 1024), wgc, wuc, wdc, nthreads=threads)
            n += 1
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": B * n / dt, "unit": "rows/s", "cores": threads, "kind": "port",
                                "sample": f"{n} calls of the C restatement (same fp16 chain) on {B} rows "
                                          f"({dt:.1f} s)"}
        line["cpu_baseline_torch"] = torch_ops_cpu_baseline(xs, ws_, wgc, wuc, wdc, eps)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_sample(args, world: int, rank: int, local: int, dev, dist) -> None:
    """Sampling on logits rows (no upstream counterpart; upstream is greedy
    only): temperature 0.8, top-k 50, top-p 0.9 over [B, 151936] fp32 logits,
    the transformers warpers' semantics, one token per row.  One step = one
    call on B rows; 4 logits buffers rotate."""
    from sampling import SamplingParams, sample
    B, V = args.batch, 151936
    params = SamplingParams(0.8, 50, 0.9, seed=7)
    g = torch.Generator(device=dev).manual_seed(SEED + rank)
    bufs = [3.0 * torch.randn(B, V, generator=g, device=dev) for _ in range(4)]
    out = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        sample(bufs[i % 4], params, offset=i, out=out)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        sample(bufs[i % 4], params, offset=i, out=out)
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    h_l = bufs[0].cpu().pin_memory()
    h_t = torch.empty(B, dtype=torch.int32).pin_memory()
    d_l = torch.empty_like(bufs[0])
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        d_l.copy_(h_l, non_blocking=True)
        h_t.copy_(sample(d_l, params, offset=i, out=out), non_blocking=True)
        stream.synchronize()
    e2e_ms = 1000.0 * (time.perf_counter() - t0)
    if dist is not None:
        t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = world * B * args.steps / (total_ms / 1000.0)
    alg = B * V * 4
    avg_step_s = statistics.mean(step_ms) / 1000.0
    peaks = measured_peaks()
    achieved = alg / avg_step_s / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (logits ~ 3 N(0,1))",
        "config": {"workload": f"sampling (temperature 0.8, top-k 50, top-p 0.9) of {B} rows x {V} logits",
                   "batch": B, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "4 logits buffers rotate" + (" (> L2 each)" if B * V * 4 > 126e6 else
                                                      " (L2-resident, as right after the lm_head)")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_src": peaks["src"], "traffic": None,
                     "algorithmic_bytes_per_step": alg, "avg_step_ms": avg_step_s * 1000.0,
                     "note": "algorithmic bytes = one read of the logits; with top-k or top-p the "
                             "one-CTA path reads each row three times (max, window statistics, "
                             "window collection)"},
        "e2e": {"value": world * B * args.steps / (e2e_ms / 1000.0), "unit": "rows/s",
                "h2d_bytes_per_step": B * V * 4, "d2h_bytes_per_step": B * 4},
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from transformers.generation.logits_process import (TemperatureLogitsWarper, TopKLogitsWarper,
                                                            TopPLogitsWarper)
        threads = torch.get_num_threads()
        x = bufs[0][: min(B, 16)].cpu()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 or n < 1:
            sc = TopPLogitsWarper(0.9)(None, TopKLogitsWarper(50)(None, TemperatureLogitsWarper(0.8)(None, x)))
            torch.multinomial(torch.softmax(sc, -1), 1)
            n += 1
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": x.shape[0] * n / dt, "unit": "rows/s", "cores": threads,
                                "kind": "port",
                                "sample": f"{n} calls of the transformers warpers + torch.multinomial on "
                                          f"{x.shape[0]} rows on the host ({dt:.1f} s)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_lmhead(args, world: int, rank: int, local: int, dev, dist) -> None:
    line = lmhead_line(args, world, rank, local, dev, dist, args.batch)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def lmhead_line(args, world: int, rank: int, local: int, dev, dist, B: int, with_cpu: bool = True) -> dict:
    """Config 5: tied lm_head + greedy argmax with the vocabulary split over the
    ranks (one contiguous row block each), the per-row (max, index) pairs
    exchanged through peer memory (one kernel per rank, default) or an NCCL
    all-gather (--exchange nccl).  One step = the argmax of B hidden rows over
    the whole vocabulary; total work is fixed, so scaling is strong."""
    from lmhead_shard import HIDDEN, VOCAB, ShardedLMHead

    g = torch.Generator(device=dev).manual_seed(SEED)
    emb = (0.02 * torch.randn(VOCAB, HIDDEN, generator=g, device=dev)).half()
    x = torch.randn(B, HIDDEN, generator=g, device=dev).half()
    # The unsharded argmax on this GPU: the sharded tokens must equal it bit for bit.
    unsharded = ShardedLMHead(emb, 1, 0, device=dev, max_rows=B).argmax(x).clone() if world > 1 else None
    head = ShardedLMHead(emb, world, rank, device=dev, max_rows=B, exchange=args.exchange)
    del emb
    torch.cuda.empty_cache()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        ref = head.argmax(x).clone()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStart()
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        tok = head.argmax(x)
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStop()
    clk = clocks.stop()
    assert torch.equal(tok, ref), "non-deterministic sharded argmax"
    if unsharded is not None:
        assert torch.equal(tok, unsharded), "sharded argmax differs from the unsharded one"
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    # End to end: hidden rows from pinned host memory, tokens back to the host.
    h_x = x.cpu().pin_memory()
    h_tok = torch.empty(B, dtype=torch.int32).pin_memory()
    d_x = torch.empty_like(x)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        d_x.copy_(h_x, non_blocking=True)
        h_tok.copy_(head.argmax(d_x), non_blocking=True)
        stream.synchronize()
    e2e_ms = 1000.0 * (time.perf_counter() - t0)
    assert torch.equal(h_tok, ref.cpu())
    if dist is not None:
        t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = B * args.steps / (total_ms / 1000.0)
    e2e_value = B * args.steps / (e2e_ms / 1000.0)
    shard_bytes = (head.hi - head.lo) * HIDDEN * 2 + B * HIDDEN * 2
    avg_step_s = statistics.mean(step_ms) / 1000.0
    peaks = measured_peaks()
    achieved = shard_bytes / avg_step_s / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,0.02) embedding, N(0,1) hidden rows)",
        "config": {"workload": f"config 5: tied lm_head + greedy argmax of {B} hidden rows, vocabulary "
                               f"split over {world} GPU(s), (max, index) pairs "
                               + ("stored into every rank's buffer through peer memory (one kernel)"
                                  if head.exchange == "peer" else "all-gathered over NCCL"),
                   "batch": B, "parallelism": f"vocab shards x{world}" if world > 1 else "single GPU",
                   "l2": f"weights of a shard ({(head.hi - head.lo) * HIDDEN * 2 / 1e6:.1f} MB) are re-read "
                         "each step; no flush" + (" (a shard fits in L2 at 8 GPUs)" if world >= 4 else ""),
                   "tokens": "equal to the unsharded argmax on every rank" if world > 1 else "single shard"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_src": peaks["src"], "traffic": None,
                     "algorithmic_bytes_per_step": shard_bytes, "avg_step_ms": avg_step_s * 1000.0},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": B * HIDDEN * 2,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": args.steps * (2 if (world == 1 or head.exchange == "peer") else 3),
        "clocks": clk,
    }
    if head.exchange == "peer" and head.device_status() != 0:
        raise RuntimeError(f"peer exchange wait gave up: status {head.device_status():#x}")
    head.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline and with_cpu:
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        e_cpu = (0.02 * torch.randn(VOCAB, HIDDEN, generator=torch.Generator().manual_seed(2))).float()
        x_cpu = x.float().cpu()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 or n < 2:
            (x_cpu @ e_cpu.t()).argmax(dim=1)
            n += 1
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": B * n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{n} fp32 torch matmul + argmax of {B} rows over the full "
                                          f"vocabulary on the host ({dt:.1f} s)"}
    return line


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-hf-baseline", action="store_true",
                    help="skip the HF transformers fp32 CPU figure of the default line")
    ap.add_argument("--no-batched", action="store_true",
                    help="default workload: skip the config-4 (batched) sub-record")
    ap.add_argument("--prompt-len", type=int, default=PROMPT_LEN,
                    help="prefilled tokens before the timed steps (workload: 1920)")
    ap.add_argument("--gen", type=int, default=GEN, help="tokens per step (workload: 128)")
    ap.add_argument("--workload", default="decode", choices=["decode", "ops", "batched", "lmhead", "sample"],
                    help="decode: config 2 (default); ops: config 3; batched: config 4; lmhead: config 5")
    ap.add_argument("--batch", type=int, default=256, help="rows per step (ops, lmhead workloads)")
    ap.add_argument("--layers", type=int, default=28,
                    help="model depth of the batched workload; fewer layers only for profiling captures")
    ap.add_argument("--paged", action="store_true",
                    help="batched workload: paged KV pools (128-token pages) instead of contiguous ones")
    ap.add_argument("--sampled", action="store_true",
                    help="decode workload: sample (temperature 0.8, top-k 50, top-p 0.9) instead of greedy")
    ap.add_argument("--profile", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--seqs", type=int, default=256, help="sequences per GPU (batched workload)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="lmhead workload: how the ranks exchange their (max, index) pairs")
    ap.add_argument("--exact", action="store_true",
                    help="ops workload: upstream's fp16 accumulation chains (bit-exact) at every batch size")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "batched":
        run_batched(args, world, rank, local, dev, dist)
        return
    if args.workload == "lmhead":
        run_lmhead(args, world, rank, local, dev, dist)
        return
    if args.workload == "ops":
        run_ops(args, world, rank, local, dev, dist)
        return
    if args.workload == "sample":
        run_sample(args, world, rank, local, dev, dist)
        return

    from Qwen06B_architecture import Decoder
    from qwen_weights import synthetic_weights

    w_cpu = synthetic_weights(seed=SEED)
    w_gpu = {k: ([t.to(dev) for t in v] if isinstance(v, list) else v.to(dev))
             for k, v in w_cpu.items() if k != "lm_head_weight"}
    w_gpu["lm_head_weight"] = w_gpu["embed_weight"]
    dec = Decoder(weights=w_gpu, verbose=False)

    plen, gen = args.prompt_len, args.gen
    cfg_name = {(16, 64): "config 1", (1920, 128): "config 2"}.get((plen, gen), "config 2 shape")
    g = torch.Generator().manual_seed(SEED + 1)
    prompt = torch.randint(0, 151936, (plen,), generator=g).tolist()
    first = None
    for t in prompt:                       # untimed prefill, positions 0..plen-1
        first = dec.step(t)
    assert dec.position == plen

    stream = torch.cuda.current_stream(dev)

    def one_step():
        dec._position = plen
        if args.sampled:
            return dec.sample_nosync(first, gen, temperature=0.8, top_k=50, top_p=0.9, seed=7)
        return dec.generate_nosync(first, gen)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize(dev)
    ref_tokens = one_step().cpu().tolist()
    assert all(t >= 0 for t in ref_tokens), "device-side failure in warm-up"

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStart()
    t_start.record(stream)
    outs = []
    for i in range(args.steps):
        ev[i][0].record(stream)
        outs.append(one_step())
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if args.profile:
        torch.cuda.cudart().cudaProfilerStop()
    clk = clocks.stop()
    if dist is not None:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    for o in outs:
        assert o.cpu().tolist() == ref_tokens, "non-deterministic or failed decode"

    # End to end through the public API: host token in, host tokens out.
    e2e_ms = []
    for i in range(args.steps):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        toks = one_step().cpu()
        e2e_ms.append(1000.0 * (time.perf_counter() - t0))
        assert toks.tolist() == ref_tokens

    if dist is not None:
        t = torch.tensor([total_ms, sum(e2e_ms)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_total = float(t[0]), float(t[1])
    else:
        e2e_total = sum(e2e_ms)

    value = world * gen * args.steps / (total_ms / 1000.0)
    e2e_value = world * gen * args.steps / (e2e_total / 1000.0)
    avg_launch_s = statistics.mean(launch_ms) / 1000.0
    alg = algorithmic_bytes(plen, gen)
    peaks = measured_peaks()
    achieved = alg / avg_launch_s / 1e9
    traffic = profile_traffic() if (plen, gen) == (PROMPT_LEN, GEN) else None
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded random-init weights, uniform-random token ids)",
        "config": {"workload": f"{cfg_name}: batch-1 {'sampled (temperature 0.8, top-k 50, top-p 0.9)' if args.sampled else 'greedy'}"
                               f" decode, {plen}-token seeded prompt "
                               f"prefilled (untimed), {gen} steps at positions {plen}..{plen + gen - 1}"
                               " per step",
                   "batch": 1, "prompt_len": plen, "gen_steps": gen,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (1.19 GB of weights read per token); no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_src": peaks["src"], "traffic": traffic,
                     "algorithmic_bytes_per_launch": alg, "avg_launch_ms": avg_launch_s * 1000.0},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * gen},
        "gpu_launches": args.steps * (2 * gen if args.sampled else 1),
        "clocks": clk,
    }
    if args.sampled:
        line["roofline"]["note"] = "per token: one decode launch (logits written) + one sampling launch"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w_cpu)
        if not args.no_hf_baseline:
            line["cpu_baseline_hf"] = hf_cpu_baseline(w_cpu)
    if not args.no_batched and (plen, gen) == (PROMPT_LEN, GEN) and not args.sampled:
        # Config 4 at the same N (BASELINE's "batched tok/s at 1/2/4/8"), so
        # every default run -- the driver's scaling runs included -- records it.
        del dec, w_gpu
        torch.cuda.empty_cache()
        b = batched_line(args, world, rank, local, dev, dist, with_cpu=True)
        keep = ("value", "unit", "ms_per_step", "steps", "warmup", "scaling", "config", "roofline",
                "e2e", "gpu_launches", "clocks", "cpu_baseline", "cpu_baseline_hf")
        line["batched"] = {k: b[k] for k in keep if k in b}
        torch.cuda.empty_cache()
        # Config 5 (vocabulary-sharded lm_head, B = 256) at the same N.
        lm = lmhead_line(args, world, rank, local, dev, dist, 256, with_cpu=False)
        line["lmhead"] = {k: lm[k] for k in ("value", "unit", "ms_per_step", "steps", "scaling", "config",
                                             "roofline", "e2e", "gpu_launches", "clocks") if k in lm}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
