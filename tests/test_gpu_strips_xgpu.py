"""Exact strip sharding across GPUs: each of 2 (and, where the box has them,
4) processes drives one GPU and one strip of a 320x256 sensor; after every
layer the strips exchange their band events' next-layer inputs through CUDA
IPC peer memory with bounded device-side waits.  Each rank then drains the
same 200,000 events as one sensor on its own GPU and compares its owned
results -- flags of owned events, hidden rows of every layer, gate counters,
predictions, versions -- bit for bit (ssla_rt_b200.strips.exact_strip_parity).
Skipped with fewer GPUs than ranks: strips that wait on each other never
share a GPU."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, wdir, q):
    import datetime

    import torch.distributed as dist

    from ssla_rt_b200 import events as E
    from ssla_rt_b200 import strips
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        ev = E.config_events(3, n=200_000)
        res = strips.exact_strip_parity(wdir, ev, rank, world, rank, dist.all_gather_object, dist.barrier)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, {"ok": False, "error": repr(e)}))


@pytest.mark.parametrize("world", [2, 4])
def test_exact_strips_across_gpus(stub_dir, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    d = stub_dir(256, 320, 1, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, d, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, res = q.get(timeout=600)
            results[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert results[r]["ok"], str(results)
        assert results[r]["owned"] > 0 and results[r]["exchange_status"] == 0
    assert sum(results[r]["owned"] for r in range(world)) == 200_000
    assert all(p.exitcode == 0 for p in procs)
