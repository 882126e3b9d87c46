"""Multi-rank host logic on CPU (gloo, world size 2): sharding, the logits
gather, max-over-ranks timing, and a dead rank surfacing as an error."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist
    from sparsesnn_b200 import dist as sd
    try:
        sd.init_from_env("gloo", timeout_s=5.0)
        if mode == "gather":
            start, n = sd.shard(10, rank, world)
            local = torch.full((3, 4), float(rank)) + torch.arange(4.0)
            g = sd.gather_logits(local)
            m = sd.max_over_ranks(1.0 + rank)
            q.put((rank, start, n, g.tolist(), m))
        elif mode == "dead":
            if rank == 1:
                q.put((rank, "left"))
                q.close()
                q.join_thread()        # flush the message before the abrupt exit
                os._exit(0)            # leaves between steps, before the collective
            try:
                sd.gather_logits(torch.zeros(2, 2))
                q.put((rank, "no error"))
            except Exception as e:     # noqa: BLE001 - any gloo error is the signal
                q.put((rank, "error:" + type(e).__name__))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "exc:" + repr(e)))


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_shard_covers_batch():
    from sparsesnn_b200.dist import shard
    for total in (1, 7, 128):
        for world in (1, 2, 3, 8):
            spans = [shard(total, r, world) for r in range(world)]
            assert spans[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert sum(n for _, n in spans) == total
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def test_gather_and_max_over_ranks_gloo():
    out = _run("gather")
    (r0, s0, n0, g0, m0), (r1, s1, n1, g1, m1) = out
    assert (s0, n0, s1, n1) == (0, 5, 5, 5)
    expect = [[0.0, 1.0, 2.0, 3.0]] * 3 + [[1.0, 2.0, 3.0, 4.0]] * 3
    assert g0 == expect and g1 == expect          # rank order, same on every rank
    assert m0 == m1 == 2.0


def test_dead_rank_is_an_error_not_a_hang():
    out = _run("dead", timeout=90)
    assert out[1] == (1, "left")
    assert out[0][1].startswith("error:")
