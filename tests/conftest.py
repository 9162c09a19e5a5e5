"""Test tiers: CPU/gloo (default, no GPU), `gpu` (one B200), `multigpu` (>= 2 GPUs, subset of gpu)."""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs on one node")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def run_gloo(fn, world: int, *args, timeout: float = 120.0):
    """Run fn(rank, world, *args) in `world` gloo processes on 127.0.0.1; re-raise the first failure."""
    import torch.multiprocessing as mp

    port = free_port()
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_gloo_entry, args=(fn, r, world, port, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    errs = []
    while not q.empty():
        errs.append(q.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append(f"rank process {p.pid} timed out")
    bad = [e for e in errs if e != "ok"]
    if bad:
        raise AssertionError("\n".join(bad))
    assert len(errs) == world, f"only {len(errs)} of {world} ranks reported"


def _gloo_entry(fn, rank, world, port, q, args):
    import traceback

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        fn(rank, world, *args)
        dist.barrier()
        q.put("ok")
    except BaseException:
        q.put(f"rank {rank}:\n{traceback.format_exc()}")
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
