"""Strip sharding of the 320x256 sensor (host logic, CPU):

* strip bounds lie on 8-row units, cover the sensor, and are balanced;
* every event is owned by exactly one strip and routed to it, with the halo;
* two gloo ranks, each sharding the same seeded stream, own a disjoint
  cover of it (the multi-GPU routing without a GPU);
* with the C oracle as the per-strip engine: drop decisions of owned events
  equal the full-frame run exactly (drop drift 0), and the stage-3 features
  of owned head events stay within the reference's max|d| s3_feat <= 5.0.
"""
import os

import numpy as np
import pytest

from ssla_rt_b200 import events as E
from ssla_rt_b200 import strips


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_strip_bounds(n):
    b = strips.strip_bounds(256, n)
    assert b[0][0] == 0 and b[-1][1] == 256
    assert all(lo % 8 == 0 and hi % 8 == 0 and lo < hi for lo, hi in b)
    assert all(b[i][1] == b[i + 1][0] for i in range(n - 1))
    sizes = [hi - lo for lo, hi in b]
    assert max(sizes) - min(sizes) <= 8


def test_routing_owns_each_event_once():
    ev = E.make_events(40_000, 256, 320, rate_mev=20.0, seed=5, n_blobs=16, blob_frac=0.7, sigma=4.0)
    sh = strips.shard(ev, 256, 4)
    owned_total = 0
    for (lo, hi), sev, own in sh:
        owned_total += int(own.sum())
        y = sev[:, 2]
        assert ((y >= max(0, lo - 8)) & (y < min(256, hi + 8))).all()
        assert (np.diff(sev[:, 0]) >= 0).all()                  # stream order kept
        assert int(own.sum()) == int(((ev[:, 2] >= lo) & (ev[:, 2] < hi)).sum())
        x0, x1, y0, y1 = strips.owned_s2(lo, hi, 320)
        assert (x0, x1, y0, y1) == (0, 80, lo // 4, hi // 4)
    assert owned_total == len(ev)


def _gloo_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ev = E.make_events(30_000, 256, 320, rate_mev=20.0, seed=9, n_blobs=16, blob_frac=0.7, sigma=4.0)
    (lo, hi), sev, own = strips.shard(ev, 256, world)[rank]
    owned_t = torch.from_numpy(sev[own][:, 0].astype(np.float64))
    n = torch.tensor([owned_t.numel()])
    ns = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(ns, n)
    mx = int(max(int(x) for x in ns))
    pad = torch.full((mx,), -1.0, dtype=torch.float64)
    pad[: owned_t.numel()] = owned_t
    got = [torch.zeros(mx, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(got, pad)
    if rank == 0:
        allt = np.concatenate([g.numpy()[: int(k)] for g, k in zip(got, ns)])
        out.put((len(ev), np.sort(allt).tolist() == np.sort(ev[:, 0].astype(np.float64)).tolist()))
    dist.destroy_process_group()


def test_two_gloo_ranks_own_a_disjoint_cover():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    ps = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    n, same = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert n == 30_000 and same


def test_oracle_strips_exact_drops_bounded_drift(oracle_mod, stub_dir):
    O = oracle_mod
    H, W = 256, 320
    d = stub_dir(H, W, 1, 4)
    tensors = O.load_npz(d)
    ev = E.make_events(60_000, H, W, rate_mev=20.0, seed=3, n_blobs=16, blob_frac=0.7, sigma=4.0)
    full = O.Oracle(tensors, H, W, 4, O.LAYOUT_HYBRID)
    fflags, fso = full.run_events(ev)
    idx = np.arange(len(ev))
    worst = 0.0
    heads = 0
    for lo, hi in strips.strip_bounds(H, 4):
        m = strips.route_mask(ev, lo, hi, H)
        sev = ev[m]
        orc = O.Oracle(tensors, H, W, 4, O.LAYOUT_HYBRID)
        sflags, sso = orc.run_events(sev)
        own = strips.owned_mask(sev, lo, hi)
        gi = idx[m][own]
        np.testing.assert_array_equal(sflags[own], fflags[gi])      # drop drift 0
        hd = (sflags[own] & 16) != 0
        if hd.any():
            worst = max(worst, float(np.abs(sso[3][own][hd] - fso[3][gi][hd]).max()))
            heads += int(hd.sum())
    assert heads > 0
    assert worst <= 5.0, worst
