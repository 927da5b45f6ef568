"""Decode throughput of the B200 decoder on the headline configuration.

Default workload (the configuration the north
star's target is quoted on): a Qwen3-0.6B-shaped decoder with seeded
synthetic Q8_0 weights, batch 1 per GPU, a 64-token prompt of uniform
random ids, 128 greedy tokens. One step = one generation.
With --gpus N (torchrun, one process per GPU) every rank runs its own
independent stream: data parallel over streams, no collective in the data
path (weak scaling). Timing: a barrier + device synchronize on both sides
of the K timed steps, the maximum over ranks.

  value : decode tokens/s of the whole job, from CUDA events around the
          greedy-step phase inside the library (inputs resident in HBM).
  e2e   : tokens/s through the public C ABI call trit_lm_generate with the
          prompt ids in host memory and the tokens copied back, prefill
          included, wall clock between barriers.
The weights (633 MB) are larger than the 126 MB L2, so no L2 flush is done
between steps.

--impl reference runs the CPU restatement of the reference decoder (the
oracle, all host threads) on the same workload, rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

PROMPT = 64
MAX_NEW = 128
CONFIG_NAME = "c1_qwen3_0.6b_q8_0"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(config: dict, fmt: str, positions: list[int], kv_bytes: int) -> dict:
    """Bytes one greedy step must move: every weight once, the KV cache read
    up to the step's position, one KV row written."""
    d, ffn, L = config["hidden_size"], config["intermediate_size"], config["num_hidden_layers"]
    hd, H, KV, V = config["head_dim"], config["num_attention_heads"], config["num_key_value_heads"], config["vocab_size"]
    qd, kvd = H * hd, KV * hd
    mats = [(qd + 2 * kvd, d), (d, qd), (2 * ffn, d), (d, ffn)]

    def mat_bytes(n, k):
        if fmt == "q8_0":
            return n * k * 34 // 32
        if fmt == "int8":
            return n * k + 4 * n
        return n * k // 4 + 4 * n * (k // 128)

    layers = L * sum(mat_bytes(n, k) for n, k in mats) + L * 4 * (2 * d + 2 * hd)
    table = V * d * 34 // 32 if fmt != "int8" else V * d + V * (d // 32) * 4
    if not config.get("tie_word_embeddings", False):
        table = table  # the output projection is read; the embedding row is negligible
    kv_row = L * 2 * kvd * kv_bytes
    kv = sum(kv_row * (p + 1) for p in positions) / max(1, len(positions)) + kv_row
    return {"weights": layers + table, "kv": kv, "total": layers + table + kv}


class Clocks:
    """nvidia-smi samples of one GPU while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier_sync(world: int):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompts(vocab: int, count: int, seed: int) -> list[list[int]]:
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, size=PROMPT).tolist() for _ in range(count)]


def cpu_baseline(model_dir: str, threads: int | None, decode_tokens: int, reps: int) -> dict:
    """The oracle (a C++ port of the reference CPU decoder) on the host cores."""
    from oracle import oracle as O

    if threads:
        O.lib().oracle_set_threads(threads)
    oracle = O.Oracle(model_dir)
    per_token = []
    prefill = []
    for r in range(reps):
        p = prompts(oracle.vocab, 1, 1000 + r)[0]
        res = oracle.generate(p, decode_tokens + 1, timing=True)
        per_token.extend(res["seconds"][1:].tolist())
        prefill.append(res["prefill_seconds"])
    med = statistics.median(per_token)
    return {"value": 1.0 / med, "unit": "tok/s", "cores": int(O.lib().oracle_threads()), "kind": "port",
            "isa": O.lib().oracle_isa().decode(),
            "sample": f"{reps} x ({PROMPT}-token prompt + {decode_tokens} greedy tokens), median per-token time; "
                      f"prefill median {statistics.median(prefill) * 1e3:.0f} ms"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    from trit_b200 import presets

    model_dir = presets.model_path(CONFIG_NAME)
    config, fmt, _ = presets.CONFIGS[CONFIG_NAME]
    warm = cpu_baseline(model_dir, None, 2, max(1, min(args.warmup, 1)))
    del warm
    t0 = time.perf_counter()
    base = cpu_baseline(model_dir, None, 8, max(1, args.steps))
    wall = time.perf_counter() - t0
    line = {
        "impl": "reference", "metric": "decode tok/s (batch 1 per GPU)", "value": base["value"], "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3 / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> i32, f32",
        "data": "synthetic (seeded weights N(0,0.02) -> Q8_0, uniform random prompt ids)",
        "config": {"workload": "C1: Qwen3-0.6B-shaped Q8_0, batch 1, 64-token prompt, greedy decode",
                   "model": CONFIG_NAME, "global_batch": world, "seq_len": PROMPT + MAX_NEW,
                   "parallelism": "cpu (reference arm: the oracle port, all host threads)"},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--decode", default=os.environ.get("TRIT_DECODE", "persistent"))
    ap.add_argument("--kv", default="f16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    from trit_b200 import CausalLm, presets

    config, fmt, _ = presets.CONFIGS[CONFIG_NAME]
    if rank == 0 or world == 1:
        model_dir = presets.model_path(CONFIG_NAME)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        model_dir = presets.model_path(CONFIG_NAME)
    lm = CausalLm.load(model_dir, device=local, kv=args.kv, decode=args.decode, max_context=PROMPT + MAX_NEW + 8)
    vocab = lm.vocab()
    ps = prompts(vocab, args.warmup + args.steps, 77 + rank)
    for i in range(args.warmup):
        lm.generate(ps[i], max_new=MAX_NEW)
    decode_ms, decode_steps, made, launches, prefill_ms = 0.0, 0, 0, 0, 0.0
    with Clocks(local) as clocks:
        barrier_sync(world)
        t0 = time.perf_counter()
        for i in range(args.steps):
            toks = lm.generate(ps[args.warmup + i], max_new=MAX_NEW)
            t = lm.last_timing()
            decode_ms += t["decode_ms"]
            prefill_ms += t["prefill_ms"]
            decode_steps += t["decode_steps"]
            launches += t["launches"]
            made += len(toks)
        barrier_sync(world)
        wall = time.perf_counter() - t0
    wall_max = max_over_ranks(wall, world)
    decode_max = max_over_ranks(decode_ms, world)
    value = world * decode_steps / (decode_max / 1e3)
    e2e = world * made / wall_max
    positions = [PROMPT + i for i in range(MAX_NEW - 1)]
    alg = algorithmic_bytes(config, fmt, positions, 2 if args.kv == "f16" else 4)
    hbm, peak_kind = peaks()
    per_step_s = decode_ms / 1e3 / max(1, decode_steps)
    achieved = alg["total"] / per_step_s / 1e9
    line = {
        "metric": "decode tok/s (batch 1 per GPU)", "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall_max * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> i32, f32",
        "data": "synthetic (seeded weights N(0,0.02) -> Q8_0, uniform random prompt ids)",
        "config": {"workload": "C1: Qwen3-0.6B-shaped Q8_0, batch 1 per GPU, 64-token prompt, 128 greedy tokens",
                   "model": CONFIG_NAME, "global_batch": world, "seq_len": PROMPT + MAX_NEW,
                   "parallelism": f"dp{world} (independent streams, no collective)", "decode": args.decode,
                   "kv_cache": args.kv, "l2": "weights 633 MB > 126 MB L2; no flush"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": MAX_NEW * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_token": alg["total"],
                     "kernel": "decode step (persistent kernel)" if args.decode == "persistent" else "layered step"},
        "prefill_ms_per_step": prefill_ms / args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(model_dir, None, 8, 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    lm.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
