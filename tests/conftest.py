"""Shared fixtures.  Markers: `gpu` = needs a CUDA device (run on the B200 box with -m gpu)."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running case")


def load_pkg():
    """The product package (directory name has dots) under the module name iq4xs_b200."""
    spec = importlib.util.spec_from_file_location("_iq4xs_loader", ROOT / "qwen_3.8_27b_optimizations_b200" / "loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.load()


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def O():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def golden():
    return np.load(ROOT / "tests" / "golden" / "golden_v1.npz")


def free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(target, world: int, args_fn, timeout: float = 600.0):
    """Start `world` spawned processes `target(*args_fn(rank, port, queue))` and collect what they put
    on the queue.  The queue is drained while the ranks run (a child that has queued data does not
    exit before the parent reads it, so joining first can deadlock once the data outgrows the pipe);
    ranks still alive at the deadline are killed by their own handles.  Returns (results, exit codes)."""
    import queue as _queue
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=args_fn(r, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out, deadline = [], time.time() + timeout
    while len(out) < world and time.time() < deadline:
        try:
            out.append(q.get(timeout=1.0))
        except _queue.Empty:
            if all(p.exitcode is not None for p in procs):
                try:
                    out.append(q.get(timeout=2.0))
                except _queue.Empty:
                    break
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return out, [p.exitcode for p in procs]
