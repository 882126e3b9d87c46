"""Data-parallel replicas: one process per GPU, batch sharded across ranks,
one collective per step (all-gather of the logits).

The SNN forward has no cross-image dependency, so ranks never exchange
activations; the only exchange is gathering every rank's logits (the
reference has no multi-GPU inference path at all -- its DDP lives in the
training engine, ``tengine/dist.py:13-49``).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0, device_id=None):
    """Initialise the default process group from RANK/WORLD_SIZE/MASTER_* with
    a short timeout so a dead rank surfaces as an error, not a hang.  Returns
    ``(rank, world)``; a single process without WORLD_SIZE gets ``(0, 1)``."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if device_id is not None:
            kw["device_id"] = device_id
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous ``(start, count)`` slice of ``total`` images for ``rank``;
    the first ``total % world`` ranks take one extra image."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_logits(local: torch.Tensor, out: torch.Tensor | None = None, group=None):
    """All-gather equal-sized ``[b, classes]`` logits from every rank into
    ``[world*b, classes]`` in rank order (NCCL: one all_gather_into_tensor;
    gloo: all_gather of a list)."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]),
                          dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:
        parts = list(out.chunk(world, dim=0))
        dist.all_gather(parts, local.contiguous(), group=group)
        if parts[0].data_ptr() != out.data_ptr():
            out.copy_(torch.cat(parts, 0))
    return out


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Max of a host scalar over ranks (timings are reported as the slowest rank)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class OverlappedGather:
    """Logits all-gather pipelined behind the forward.

    ``submit(local, slot)`` gathers ``local`` (the logits a forward just
    wrote, in buffer ``slot``) on a side stream once the current stream has
    reached that point, so the collective of step i runs under the forward of
    step i+1 instead of after it.  ``reuse(slot)`` makes the current stream
    wait until the gather that read buffer ``slot`` has finished, before a
    forward overwrites it; ``drain()`` joins the side stream.  Every rank
    issues the same gathers in the same order (one per step)."""

    def __init__(self, shape, world, device, group=None, dtype=torch.float32):
        self.stream = torch.cuda.Stream(device)
        self.out = torch.empty((world * shape[0],) + tuple(shape[1:]), dtype=dtype, device=device)
        self.group = group
        self._done = {}

    def submit(self, local: torch.Tensor, slot: int) -> None:
        cur = torch.cuda.current_stream(local.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        self.stream.wait_event(ready)
        with torch.cuda.stream(self.stream):
            gather_logits(local, self.out, self.group)
            done = torch.cuda.Event()
            done.record(self.stream)
        self._done[slot] = done

    def reuse(self, slot: int) -> None:
        ev = self._done.get(slot)
        if ev is not None:
            torch.cuda.current_stream(self.out.device).wait_event(ev)

    def drain(self) -> torch.Tensor:
        torch.cuda.current_stream(self.out.device).wait_stream(self.stream)
        return self.out
