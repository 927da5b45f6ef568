"""Decode throughput of the B200 decoder (Trit's CausalLm token loop).

Default workload (the configuration the north
star's target is quoted on): C1, a Qwen3-0.6B-shaped decoder with seeded
synthetic Q8_0 weights, batch 1 per GPU, a 64-token prompt of uniform
random ids, 128 greedy tokens. One step = one generation.

  --config c1   (default) batch 1, Q8_0 0.6B, persistent decode kernel
  --config c2   16 streams per GPU, per-row int8 0.6B, 256-token prompts,
                256 greedy steps (trit_lm_generate_batch)
  --config c3   batch 1, ternary 1.7B, 375 audio-prefix rows + 16 ids,
                200 greedy steps (trit_lm_answer)
  --config c5   64 streams per GPU, Q8_0 Ministral-3B shape, 1024-token
                prompts, 256 greedy steps (trit_lm_generate_batch)
  --config c4   op sweep: Q8_0 products of five shapes at 1, 4, 16, 64 rows

With --gpus N (torchrun, one process per GPU) every rank runs its own
streams: data parallel over independent streams, no collective on the
data path (weak scaling). Timing: a barrier + device synchronize on both
sides of the K timed steps, the maximum over ranks.

  value : decode tokens/s of the whole job, from CUDA events around the
          greedy steps inside the library (weights and prompts resident).
  e2e   : tokens/s through the public C ABI call (trit_lm_generate /
          _generate_batch / _answer) with the prompt in host memory and
          the tokens copied back, prefill included, wall clock between
          barriers.
The weights (0.6-3.8 GB) are larger than the 126 MB L2, so no L2 flush is
done between steps; the op sweep rotates copies of each matrix so that
every repetition reads it from HBM.

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

from trit_b200 import dp  # noqa: E402

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
SEED = 20261201

WORKLOADS = {
    "c1": {"model": "c1_qwen3_0.6b_q8_0", "streams": 1, "prompt": 64, "new": 128, "kind": "generate",
           "metric": "decode tok/s (batch 1 per GPU)",
           "workload": "C1: Qwen3-0.6B-shaped Q8_0, batch 1 per GPU, 64-token prompt, 128 greedy tokens"},
    "c2": {"model": "c2_qwen3_0.6b_int8", "streams": 16, "prompt": 256, "new": 256, "kind": "batch",
           "metric": "decode tok/s (16 streams per GPU)",
           "workload": "C2: Qwen3-0.6B-shaped per-row int8, 16 streams per GPU, 256-token prompts, 256 greedy steps"},
    "c3": {"model": "c3_qwen3_1.7b_ternary", "streams": 1, "rows": 375, "prompt": 16, "new": 200, "kind": "answer",
           "metric": "decode tok/s (batch 1, 391-row prefix)",
           "workload": "C3: Qwen3-1.7B-shaped ternary, batch 1, 375 audio rows + 16 ids, 200 greedy steps"},
    "c5": {"model": "c5_ministral_3b_q8_0", "streams": 64, "prompt": 1024, "new": 256, "kind": "batch",
           # The CPU legs time decode tokens after a 64-id prompt: the oracle's
           # 1024-id prefill alone takes ~9 minutes on 8 host cores.
           "sample_prompt": 64,
           "metric": "decode tok/s (64 streams per GPU)",
           "workload": "C5: Ministral-3B-shaped Q8_0, 64 streams per GPU, 1024-token prompts, 256 greedy steps"},
}
SWEEP_SHAPES = [(1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (151936, 1024)]
SWEEP_ROWS = [1, 4, 16, 64]


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(info: dict, streams: int, positions: list[int], kv_bytes: int) -> dict:
    """Bytes one greedy step must move: every weight once (products, norms,
    the output table), each stream's KV cache up to its position, and one
    new KV row per stream. `positions` are the positions the steps feed."""
    d, L, hd = info["hidden_size"], info["num_hidden_layers"], info["head_dim"]
    kvd = info["num_key_value_heads"] * hd
    norms = L * 4 * (2 * d + (2 * hd if info["qk_norm"] else 0)) + 4 * d
    weights = info["product_bytes"] + info["output_table_bytes"] + norms
    kv_row = L * 2 * kvd * kv_bytes
    kv = streams * (sum(kv_row * (p + 1) for p in positions) / max(1, len(positions)) + kv_row)
    return {"weights": weights, "kv": kv, "total": weights + kv}


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


def audio_rows(width: int, count: int, stream: int) -> np.ndarray:
    """The seeded N(0, 1) prefix rows of C3 (audio frames in the reference)."""
    return np.random.default_rng([SEED, 3, stream]).normal(0, 1, (count, width)).astype(np.float32)


# ------------------------------------------------------------ CPU legs ----
def cpu_sample(w: dict, model_dir: str, tokens: int, reps: int, threads: int | None = None) -> dict:
    """The oracle (a C++ restatement of the reference CPU decoder) on the
    host cores: the per-token time of `reps` generations of `tokens` greedy
    tokens after the workload's prompt. Streams are decoded one after
    another, as calls on one reference engine take turns."""
    from oracle import oracle as O

    if threads:
        O.lib().oracle_set_threads(threads)
    orc = O.Oracle(model_dir, kv_f16=False)
    if w["kind"] == "answer":
        # answer() reports no per-token times: the difference of a call with
        # `tokens` + 1 tokens and one with 1 token, per token.
        def call(r, n):
            tail = dp.stream_prompt(SEED, 20_000 + r, w["prompt"], orc.vocab)
            t0 = time.perf_counter()
            orc.answer([], audio_rows(orc.width, w["rows"], 20_000 + r), tail, n)
            return time.perf_counter() - t0

        short = [call(r, 1) for r in range(reps)]
        full = [call(r, tokens + 1) for r in range(reps)]
        per = (sum(full) - sum(short)) / (reps * tokens)
        pre = statistics.median(short)
    else:
        per_token, prefill = [], []
        prompt = w.get("sample_prompt", w["prompt"])
        for r in range(reps):
            p = dp.stream_prompt(SEED, 10_000 + r, prompt, orc.vocab)
            res = orc.generate(p, tokens + 1, timing=True)
            per_token.extend(res["seconds"][1:].tolist())
            prefill.append(res["prefill_seconds"])
        per = statistics.median(per_token)
        pre = statistics.median(prefill)
    orc.close()
    return {"value": 1.0 / per, "unit": "tok/s", "cores": int(O.lib().oracle_threads()), "kind": "port",
            "isa": O.lib().oracle_isa().decode(),
            "sample": (f"{reps} x (the workload's prompt + {tokens} greedy tokens)" if "sample_prompt" not in w else
                       f"{reps} x ({w['sample_prompt']}-id prompt instead of the workload's {w['prompt']} + {tokens} "
                       f"greedy tokens)") + f", one stream at a time, per-token time; prefill {pre * 1e3:.0f} ms"}


def cpu_sweep(reps: int) -> dict:
    """C4 on the host cores: the oracle's W8A8 product (the reference's
    VNNI tile) for each shape and row count, `reps` repetitions."""
    from oracle import oracle as O

    rng = np.random.default_rng(SEED + 4)
    hbm_bytes, seconds, cases = 0.0, 0.0, []
    for (n, k) in SWEEP_SHAPES:
        codes = rng.integers(-127, 128, (n, k)).astype(np.int8)
        scales = rng.uniform(1e-4, 1e-3, (n, k // 32)).astype(np.float32)
        layer = O.IntLayer(codes, scales, 32, 32, True)
        for m in SWEEP_ROWS:
            x = rng.normal(0, 1, (m, k)).astype(np.float32)
            layer.forward(x)
            t0 = time.perf_counter()
            for _ in range(reps):
                layer.forward(x)
            s = (time.perf_counter() - t0) / reps
            b = n * k * 34 / 32 + 4 * m * (k + n)
            cases.append({"n": n, "k": k, "m": m, "us": s * 1e6, "gbs": b / s / 1e9})
            hbm_bytes += b
            seconds += s
        del layer
    return {"value": hbm_bytes / seconds / 1e9, "unit": "GB/s", "cores": int(O.lib().oracle_threads()),
            "kind": "port", "isa": O.lib().oracle_isa().decode(),
            "sample": f"{reps} repetitions of each of {len(cases)} cases (seeded random codes)", "cases": cases}


def run_reference(args, r: dp.Rank) -> None:
    if r.rank != 0:
        return
    from oracle import oracle as O
    from tests.synth import presets

    # Every host thread this process may use: torchrun sets OMP_NUM_THREADS=1
    # for multi-rank runs, which would leave the reference arm one core.
    O.lib().oracle_set_threads(len(os.sched_getaffinity(0)))
    if args.config == "c4":
        t0 = time.perf_counter()
        base = cpu_sweep(max(1, args.steps))
        wall = time.perf_counter() - t0
        w = {"metric": "GEMV HBM GB/s (Q8_0 op sweep)", "model": None,
             "workload": "C4: Q8_0 products of five shapes at 1, 4, 16, 64 rows"}
    else:
        w = WORKLOADS[args.config]
        model_dir = presets.model_path(w["model"])
        # No separate warm-up: loading the oracle reads every weight, and the
        # per-token times start after the prompt.
        t0 = time.perf_counter()
        base = cpu_sample(w, model_dir, 8, max(1, args.steps))
        wall = time.perf_counter() - t0
    line = {
        "impl": "reference", "metric": w["metric"], "value": base["value"], "unit": base["unit"],
        "n_gpus": r.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3 / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> i32, f32",
        "data": "synthetic (seeded N(0,0.02) weights, uniform random prompt ids)",
        "config": {"workload": w["workload"], "model": w["model"],
                   "parallelism": "cpu (reference arm: the oracle port of the reference decoder, all host threads)"},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": base["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU legs ----
def tp_group_id(r: dp.Rank, tp: int) -> str:
    """The NCCL group id of this rank's tensor-parallel group: made by the
    group's first rank (trit_cuda_tp_id) and handed to the others."""
    import torch.distributed as dist

    from trit_b200 import lm as lmmod

    ids = [None] * r.world
    dist.all_gather_object(ids, lmmod.tp_id() if r.rank % tp == 0 else "")
    return ids[(r.rank // tp) * tp]


def allreduce_us(r: dp.Rank, tp: int, nbytes: int, reps: int = 200) -> float:
    """Device time of one f32 sum all-reduce of `nbytes` within a
    tensor-parallel group (torch's NCCL, the size the library reduces after
    o_proj and down_proj), max over ranks."""
    import torch
    import torch.distributed as dist

    groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(r.world // tp)]
    mine = groups[r.rank // tp]
    x = torch.zeros(max(1, nbytes // 4), dtype=torch.float32, device="cuda")
    for _ in range(10):
        dist.all_reduce(x, group=mine)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        dist.all_reduce(x, group=mine)
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1e3 / reps
    for g in groups:
        dist.destroy_process_group(g)
    return dp.reduce(us, r, "max")


def measure(w: dict, args, r: dp.Rank, steps: int, warmup: int, decode: str, exact: bool) -> tuple[dict, str]:
    """One workload on this rank's GPU: `warmup` untimed generations, then
    `steps` timed ones between barriers. Returns the JSON fields of its line
    (whole-job values: the max of the ranks' times) and the model folder."""
    from trit_b200 import CausalLm, lm as lmmod
    from tests.synth import presets

    if r.rank == 0:
        model_dir = presets.model_path(w["model"])
    dp.barrier(r)
    model_dir = presets.model_path(w["model"])
    info = lmmod.inspect(model_dir)
    S = w["streams"]
    prompt_len = w["prompt"] + w.get("rows", 0)
    tc_attention = bool(getattr(args, "tc_attention", False))
    exact = exact and not tc_attention
    opts = {"device": r.local, "kv": args.kv, "max_context": prompt_len + w["new"] + 8, "exact": exact}
    tp = max(1, getattr(args, "tp", 1) or 1)
    group = r.rank // tp  # ranks of one tensor-parallel group serve the same streams
    if tp > 1:
        opts.update(tp_size=tp, tp_rank=r.rank % tp, tp_id=tp_group_id(r, tp))
    if w["kind"] == "batch":
        # Prompt passes of 4096 rows: 15 % more end to end on C5 than 512
        # (fuller tensor-core and attention grids).
        opts.update(max_streams=S, prefill_rows=max(4096, S))
    if args.tc_rows is not None:
        opts.update(tc_rows=args.tc_rows)
    if getattr(args, "tc_f16", False):
        opts.update(tc_f16=True)
    if tc_attention:
        opts.update(tc_attention=True)
    if args.prefill_rows is not None:
        opts.update(prefill_rows=args.prefill_rows)
    else:
        opts.update(decode=decode)
    lm = CausalLm.load(model_dir, **opts)
    vocab, width = lm.vocab(), lm.width()

    def inputs(step: int):
        base = (group * 1_000_003 + step) * S
        prompts = [dp.stream_prompt(SEED, base + s, w["prompt"], vocab) for s in range(S)]
        rows = audio_rows(width, w["rows"], base) if w["kind"] == "answer" else None
        return prompts, rows

    def one(step: int):
        prompts, rows = inputs(step)
        if w["kind"] == "generate":
            return len(lm.generate(prompts[0], max_new=w["new"]))
        if w["kind"] == "answer":
            return len(lm.answer([], rows, prompts[0], max_new=w["new"]))
        return sum(len(t) for t in lm.generate_batch(prompts, max_new=w["new"]))

    for i in range(warmup):
        one(i)
    decode_ms = prefill_ms = 0.0
    decode_steps = made = launches = 0
    with Clocks(r.local) as clocks:
        dp.barrier(r)
        t0 = time.perf_counter()
        for i in range(steps):
            made += one(warmup + i)
            t = lm.last_timing()
            decode_ms += t["decode_ms"]
            prefill_ms += t["prefill_ms"]
            decode_steps += t["decode_steps"]
            launches += t["launches"]
        dp.barrier(r)
        wall = time.perf_counter() - t0
    lm.close()
    wall_max = dp.reduce(wall, r, "max")
    decode_max = dp.reduce(decode_ms, r, "max")
    # Every rank of a tensor-parallel group reports its group's tokens.
    steps_all = dp.reduce(float(decode_steps), r, "sum") / tp
    made_all = dp.reduce(float(made), r, "sum") / tp
    value = steps_all / (decode_max / 1e3)
    e2e = made_all / wall_max
    positions = [prompt_len + i for i in range(w["new"] - 1)]
    alg = algorithmic_bytes(info, S, positions, 2 if args.kv == "f16" else 4)
    hbm, peak_kind = peaks()
    greedy_steps = decode_steps / S  # forwards of the whole batch
    per_step_s = decode_ms / 1e3 / max(1.0, greedy_steps)
    achieved = alg["total"] / per_step_s / 1e9 / tp  # per GPU: a group's ranks share the step's bytes
    path = "tree-order sums" if not exact else "exact reference order"
    kernel = {"generate": f"decode step (persistent kernel, {path})" if decode == "persistent" else "layered step",
              "answer": f"decode step (persistent kernel, {path})" if decode == "persistent" else "layered step",
              "batch": "batched decode step (layered kernels, one CUDA graph)"}[w["kind"]]
    h2d = S * w["prompt"] * 4 + w.get("rows", 0) * width * 4
    fields = {
        "metric": w["metric"], "value": value, "unit": "tok/s", "n_gpus": r.world,
        "steps": steps, "warmup": warmup, "ms_per_step": wall_max * 1e3 / steps,
        "config": {"workload": w["workload"], "model": w["model"], "global_batch": S * r.world // tp,
                   "seq_len": prompt_len + w["new"], "parallelism": (f"dp{r.world} (independent streams, no collective)" if tp == 1 else
                                   f"tp{tp} x dp{r.world // tp} (NCCL all-reduce of o/down partials, argmax keys)"),
                   "decode": decode if w["kind"] != "batch" else "batched", "exact": exact,
                   "prompt_attention": "tensor cores (f16)" if tc_attention else "exact", "kv_cache": args.kv,
                   "l2": f"weights {alg['weights'] / 1e6:.0f} MB > 126 MB L2; no flush"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": S * w["new"] * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": TRAFFIC.get(w["key"]) if not exact else TRAFFIC_EXACT.get(w["key"]),
                     "algorithmic_bytes_per_step": alg["total"], "kv_bytes_per_step": alg["kv"], "kernel": kernel},
        "prefill_ms_per_step": prefill_ms / steps,
        "clocks": clocks.summary(),
    }
    if tp > 1:
        # The collective's share of a decode step: two f32 all-reduces a layer
        # of [streams x width] (o_proj and down_proj partials) plus one of
        # the argmax keys, timed alone at the same size.
        nbytes = S * info["hidden_size"] * 4
        us = allreduce_us(r, tp, nbytes)
        per_step = 2 * info["num_hidden_layers"]
        fields["tp"] = {"size": tp, "allreduce_bytes": nbytes, "allreduce_us": us, "allreduces_per_step": per_step + 1,
                        "decode_step_us": per_step_s * 1e6,
                        "collective_share": per_step * us / (per_step_s * 1e6)}
    return fields, model_dir


def workload(args) -> dict:
    w = dict(WORKLOADS[args.config], key=args.config)
    for key in ("streams", "prompt", "new"):
        if getattr(args, key) is not None:
            w[key] = getattr(args, key)
            w["workload"] += f" ({key} set to {getattr(args, key)})"
    return w


def run_decode(args, r: dp.Rank) -> None:
    w = workload(args)
    fields, model_dir = measure(w, args, r, args.steps, args.warmup, args.decode, not args.tree)
    line = {**fields, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 x int8 -> i32, f32",
            "data": "synthetic (seeded N(0,0.02) weights, uniform random prompt ids"
                    + (", N(0,1) prefix rows)" if w["kind"] == "answer" else ")")}
    if args.config == "c1" and not args.no_batch64 and args.tp == 1:
        # The batch-64 half of the metric in the same run (and so in the
        # driver's 1/2/4/8-GPU scaling run): C5, 64 streams per GPU.
        b, _ = measure(dict(WORKLOADS["c5"], key="c5"), args, r, BATCH64_STEPS, BATCH64_WARMUP, "persistent",
                       not args.tree)
        b["note"] = (f"C5 workload measured in the same run as the headline line: {BATCH64_WARMUP} warm-up and "
                     f"{BATCH64_STEPS} timed generations (fewer than the headline's, to bound the run)")
        line["batch64"] = b
    if r.rank == 0 and r.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(w, model_dir, 8, 1)
    if r.rank == 0:
        print(json.dumps(line), flush=True)


# Per-step DRAM bytes (read + write) of the dominant kernel from ncu
# captures, where one was taken for the workload (see profiles/).
TRAFFIC: dict = {}
# C1: a 15-step capture (read + write per step) plus the KV bytes of the
# bench's 56 more positions on average (profiles/k_decode_c1.md).
TRAFFIC_EXACT: dict = {"c1": (9.629856e9 + 8.017664e6) / 15 + 56 * 114688}
# The batch-64 object of the default line: generations timed (C5 takes
# ~8 s a generation on one B200).
BATCH64_STEPS = 2
BATCH64_WARMUP = 1


def q8_0_blocks(values: np.ndarray) -> np.ndarray:
    """ggml Q8_0 bytes of a row-major f32 matrix (Blocks::quantize,
    src/cpu/gemm.rs:53-76): per 32 values d = max|x|/127, codes
    round-half-away(x * (1/d)), d stored as f16 before the codes."""
    v = values.astype(np.float32).reshape(-1, 32)
    d = (np.abs(v).max(axis=1) / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    prod = (v * inv[:, None]).astype(np.float32)
    codes = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -128, 127).astype(np.int8)
    out = np.empty((v.shape[0], 34), np.uint8)
    out[:, :2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = codes.view(np.uint8)
    return out.reshape(-1)


def dense_kernel(n: int, m: int) -> str:
    """The product kernel trit_dense_forward_device runs for n rows and m
    frames (the library's rule: the tensor cores from 16 frames, from 4 on
    matrices of 6144 rows or more, always from 32768 rows)."""
    return "k_gemm_tc" if (m >= 16 or (m >= 4 and n >= 6144) or n >= 32768) else "k_gemv_slots"


def sweep_shapes(args) -> list:
    if not getattr(args, "shapes", None):
        return SWEEP_SHAPES
    return [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]


def sweep_rows(args) -> list:
    if not getattr(args, "rows", None):
        return SWEEP_ROWS
    return [int(v) for v in args.rows.split(",")]


def run_sweep(args, r: dp.Rank) -> None:
    """C4: each Q8_0 product (W8A8, Int8::from_q8_0) at 1, 4, 16, 64 rows,
    `reps` repetitions through trit_dense_forward_device; copies of the
    matrix rotate so every repetition reads it from HBM."""
    import torch

    from trit_b200 import Dense

    torch.cuda.set_device(r.local)
    timing_stream = torch.cuda.Stream()
    hbm, peak_kind = peaks()
    rng = np.random.default_rng(SEED + 4)
    cases, total_bytes, total_s = [], 0.0, 0.0
    launches = 0
    with Clocks(r.local) as clocks:
        for (n, k) in sweep_shapes(args):
            blocks = q8_0_blocks(rng.normal(0, 0.02, (n, k)).astype(np.float32))
            wbytes = n * k * 34 // 32
            copies = max(1, -(-256 * 2 ** 20 // wbytes))
            layers = [Dense.q8_0(blocks, n, k, device=r.local) for _ in range(copies)]
            for m in sweep_rows(args):
                x = torch.from_numpy(rng.normal(0, 1, (m, k)).astype(np.float32)).cuda()
                y = torch.empty((m, n), dtype=torch.float32, device="cuda")
                # A stream of our own: its handle is never 0, which the C ABI
                # reads as "the layer's own stream", so the events below see
                # the products they bracket.
                stream = timing_stream.cuda_stream
                torch.cuda.synchronize()
                # Every copy once first: a copy's first call at a new row
                # count sizes its buffers (a device allocation).
                for i in range(copies + 2):
                    layers[i % copies].forward_device(x.data_ptr(), m, y.data_ptr(), stream)
                reps = args.reps
                dp.barrier(r)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(timing_stream)
                for i in range(reps):
                    layers[i % copies].forward_device(x.data_ptr(), m, y.data_ptr(), stream)
                end.record(timing_stream)
                torch.cuda.synchronize()
                s = start.elapsed_time(end) / 1e3 / reps
                s = dp.reduce(s, r, "max")
                b = wbytes + 4 * m * (k + n)
                cases.append({"n": n, "k": k, "m": m, "us": s * 1e6, "gbs": b / s / 1e9, "frac": b / s / 1e9 / hbm,
                              "tops": 2 * m * n * k / s / 1e12})
                total_bytes += b * reps
                total_s += s * reps
                launches += reps * 2 * r.world
            del layers
    value = total_bytes / total_s / 1e9 * r.world
    best = max(cases, key=lambda c: c["gbs"])
    # e2e: the largest product at 1 row through host buffers (trit_dense_forward).
    n, k = SWEEP_SHAPES[-1]
    layer = Dense.q8_0(q8_0_blocks(rng.normal(0, 0.02, (n, k)).astype(np.float32)), n, k, device=r.local)
    xh = rng.normal(0, 1, (1, k)).astype(np.float32)
    layer.forward(xh)
    t0 = time.perf_counter()
    for _ in range(20):
        layer.forward(xh)
    e2e_s = (time.perf_counter() - t0) / 20
    layer.close()
    line = {
        "metric": "GEMV HBM GB/s (Q8_0 op sweep)", "value": value, "unit": "GB/s", "n_gpus": r.world,
        "steps": args.reps, "warmup": 3, "ms_per_step": total_s * 1e3 / max(1, len(cases) * args.reps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> i32, f32",
        "data": "synthetic (seeded N(0,0.02) weights -> Q8_0, x ~ N(0,1))",
        "config": {"workload": "C4: Q8_0 products [1024x3072], [3072x1024], [2048x6144], [6144x2048], "
                               "[151936x1024] (n x k) at 1, 4, 16, 64 rows",
                   "parallelism": f"dp{r.world}", "l2": "matrix copies rotate past 256 MB per case"},
        "e2e": {"value": (n * k * 34 / 32 + 4 * (k + n)) / e2e_s / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": 4 * k, "d2h_bytes_per_step": 4 * n},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": best["gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": best["gbs"] / hbm, "peak_kind": peak_kind, "traffic": None,
                     "kernel": f"{dense_kernel(best['n'], best['m'])}, best case n={best['n']} k={best['k']} m={best['m']}"},
        "cases": cases,
        "clocks": clocks.summary(),
    }
    if r.rank == 0 and r.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sweep(1)
    if r.rank == 0:
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--decode", default=os.environ.get("TRIT_DECODE", "persistent"))
    ap.add_argument("--tree", action="store_true",
                    help="the tree-order persistent decode (\"exact\": false) instead of the default exact one")
    ap.add_argument("--no-batch64", action="store_true", help="leave the C5 batch-64 object out of the C1 line")
    ap.add_argument("--tc-rows", type=int, help="rows from which products use the tensor cores (engine option)")
    ap.add_argument("--tc-f16", action="store_true", help="f16-operand tensor-core products for Q8_0 layers (engine option)")
    ap.add_argument("--tc-attention", action="store_true",
                    help="prompt attention on the tensor cores (f16 flash attention; not bit-exact)")
    ap.add_argument("--prefill-rows", type=int, help="rows a prompt pass (engine option)")
    ap.add_argument("--kv", default="f16")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel group size (ranks of a group split each layer; --gpus a multiple of it)")
    ap.add_argument("--reps", type=int, default=1000, help="repetitions per case of the op sweep")
    ap.add_argument("--shapes", help="op sweep shapes instead of the workload's, e.g. 16384x3072,3072x8192")
    ap.add_argument("--rows", help="op sweep row counts instead of the workload's, e.g. 64,128,512")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--streams", type=int, help="streams per GPU instead of the workload's (profiling runs)")
    ap.add_argument("--prompt", type=int, help="prompt ids instead of the workload's")
    ap.add_argument("--new", type=int, help="greedy tokens instead of the workload's")
    args = ap.parse_args()
    backend = "nccl"
    if args.impl == "reference":
        backend = "gloo"
    r = dp.init(backend, timeout_s=900)
    if args.impl != "reference" and (args.tp < 1 or r.world % args.tp):
        raise SystemExit(f"--tp {args.tp} does not divide the {r.world} ranks")
    try:
        if args.impl == "reference":
            run_reference(args, r)
        elif args.config == "c4":
            run_sweep(args, r)
        else:
            run_decode(args, r)
    finally:
        dp.finish(r)


if __name__ == "__main__":
    main()
