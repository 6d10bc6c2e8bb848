"""The paced replay producer (ssla_replay_*) on host memory, no GPU: every
event reaches its ring in order across wrap-arounds, full rings hold the
producer back until the consumer releases slots, no event is published
before it is due, and bad rings are refused."""
import threading
import time

import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200.engine import SslaError
from ssla_rt_b200.rings import Replay, RingSet


def _consume(rings, streams, seen_ns, stop):
    """Host consumer: copies each published slot, then releases it (tail)."""
    got = [[] for _ in streams]
    while not stop.is_set():
        idle = True
        for r in range(rings.n):
            h, t = rings.head(r), rings.tail(r)
            for i in range(t, h):
                got[r].append(rings.events[r, i % rings.capacity].copy())
                if seen_ns is not None:
                    seen_ns[r].append(time.monotonic_ns())
            if h > t:
                rings.words[r, 1] = h
                idle = False
        if idle and all(len(g) == len(s) for g, s in zip(got, streams)):
            break
    return got


def _stream(n, seed, span_us):
    rng = np.random.default_rng(seed)
    ev = np.zeros((n, 4), np.float32)
    ev[:, 0] = np.sort(rng.uniform(0, span_us, n)).astype(np.float32)
    ev[:, 1] = rng.integers(0, 80, n)
    ev[:, 2] = rng.integers(0, 64, n)
    ev[:, 3] = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    return ev


def test_replay_order_wrap_and_backpressure():
    streams = [_stream(50, 1, 100.0), _stream(0, 2, 1.0), _stream(17, 3, 100.0)]
    rings = RingSet(3, 8, pinned=False)
    rp = Replay(rings, streams, time_scale=0.0)
    got = _consume(rings, streams, None, threading.Event())
    st = rp.join()
    assert st["published"] == 67
    assert st["full_waits"] > 0                     # 50 events through 8 slots
    for g, s in zip(got, streams):
        np.testing.assert_array_equal(np.array(g).reshape(-1, 4), s)
    assert [rings.head(r) for r in range(3)] == [50, 0, 17]


def test_replay_paces_by_timestamp():
    streams = [_stream(200, 4, 30_000.0), _stream(100, 5, 30_000.0)]     # 30 ms of events
    rings = RingSet(2, 1024, pinned=False)
    seen = [[], []]
    rp = Replay(rings, streams, time_scale=1.0)
    got = _consume(rings, streams, seen, threading.Event())
    st = rp.join()
    assert st["published"] == 300
    for r, s in enumerate(streams):
        assert len(got[r]) == len(s)
        due = st["start_ns"] + s[:, 0].astype(np.float64) * 1000.0
        assert (np.array(seen[r], np.float64) >= due - 1e3).all()     # never before its time
    assert max(seen[0][-1], seen[1][-1]) - st["start_ns"] < 30e6 + 2e9
    assert st["max_lag_ns"] < 1e9


def test_replay_stop_and_bad_rings():
    rings = RingSet(1, 4, pinned=False)
    rp = Replay(rings, [_stream(100, 6, 10.0)], time_scale=0.0)
    time.sleep(0.05)                                # ring full, nobody consumes
    rp.stop()
    st = rp.join()
    assert st["published"] == 4
    bad = RingSet(1, 4, pinned=False)
    bad.descs[0].capacity = 6
    with pytest.raises(SslaError) as ei:
        Replay(bad, [_stream(3, 7, 1.0)])
    assert ei.value.code == abi.SSLA_ERR_ARG
