"""Run a test body on `world` CPU gloo ranks (spawned processes on 127.0.0.1)."""
from __future__ import annotations

import os
import socket
import sys
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args, q, pg_timeout):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    torch.set_num_threads(1)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout))
        res = fn(rank, world, *args)
        q.put((rank, "ok", res))
    except BaseException as e:  # report to the parent
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run_ranks(fn, world: int, *args, timeout: float = 240.0, pg_timeout: float = 60.0):
    """Run fn(rank, world, *args) on `world` gloo ranks; return the per-rank results.
    Raises AssertionError with the failing rank's traceback."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, pg_timeout)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    errors = []
    import queue as _q
    import time
    deadline = time.time() + timeout
    while len(results) + len(errors) < world and time.time() < deadline:
        try:
            rank, status, payload = q.get(timeout=1.0)
        except _q.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
            continue
        if status == "ok":
            results[rank] = payload
        else:
            errors.append(f"rank {rank}:\n{payload}")
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    if errors:
        raise AssertionError("\n".join(errors))
    if len(results) != world:
        raise AssertionError(f"only {len(results)}/{world} ranks reported (timeout or crash)")
    return [results[r] for r in range(world)]
