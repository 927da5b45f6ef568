"""Data parallelism over independent streams: one process per GPU, each with
its own model replica, and no collective on the data path (the streams of
a batch never exchange data). torch.distributed is only the plumbing of a
multi-GPU run: it starts the ranks, lines them up before and after a timed
region, and takes the maximum of their device times.

The reference decodes one stream per CausalLm call on one CPU team
(src/models/parts/causal_lm.rs:217-249); a run over many streams is its
callers' loop, which this module splits across GPUs."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import numpy as np


@dataclass
class Rank:
    rank: int = 0
    world: int = 1
    local: int = 0
    backend: str = ""


def environment() -> Rank:
    """RANK / WORLD_SIZE / LOCAL_RANK as torchrun sets them (1 rank without)."""
    return Rank(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str = "nccl", timeout_s: float = 600.0) -> Rank:
    """Joins the process group of a multi-rank run (no-op for one rank).
    With "nccl" each rank takes the GPU of its local rank."""
    r = environment()
    if r.world > 1:
        import torch
        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            torch.cuda.set_device(r.local)
            kwargs["device_id"] = torch.device("cuda", r.local)
        dist.init_process_group(backend, **kwargs)
        r.backend = backend
    return r


def finish(r: Rank) -> None:
    if r.world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def split(total: int, r: Rank) -> range:
    """The streams [begin, end) of rank r: contiguous, sizes differing by at
    most one, every stream on exactly one rank."""
    base, extra = divmod(total, r.world)
    begin = r.rank * base + min(r.rank, extra)
    return range(begin, begin + base + (1 if r.rank < extra else 0))


def barrier(r: Rank) -> None:
    """Device synchronize, then (for several ranks) a barrier, then device
    synchronize: the two sides of a timed region."""
    import torch

    gpu = torch.cuda.is_available() and r.backend != "gloo"
    if gpu:
        torch.cuda.synchronize()
    if r.world > 1:
        import torch.distributed as dist

        dist.barrier()
    if gpu:
        torch.cuda.synchronize()


def reduce(value: float, r: Rank, op: str = "max") -> float:
    """The maximum (or sum) of a per-rank number over all ranks."""
    if r.world == 1:
        return value
    import torch
    import torch.distributed as dist

    device = "cuda" if r.backend == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def stream_prompt(seed: int, stream: int, length: int, vocab: int) -> list[int]:
    """The prompt of global stream `stream`: uniform random ids from a
    generator seeded by (seed, stream), so it does not depend on how the
    streams are split over ranks."""
    rng = np.random.default_rng([seed, stream])
    return rng.integers(0, vocab, size=length).tolist()
