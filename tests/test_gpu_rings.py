"""Ring drains (ssla_engine_rings_attach / drain_rings / serve_rings): many
streams, each through its own pinned ring, drained together.  Fed by the
replay producer, every stream's events come out with the oracle's flags,
head events with the oracle's decoded prediction rows in the ring's output
slots, and the final state of every partition is the oracle's -- across ring
wrap-arounds, uneven and empty streams and drains of any size.  The ring
words follow the protocol: tail released once copied, events_done after the
outputs; a head beyond the ring's capacity is refused."""
import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _oracle_tail_preds(O, d, ev, n_tail):
    """Oracle over the stream; decoded row of every head event among the
    last n_tail events (index -> row), plus the oracle object."""
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, abi.LAYOUT_HYBRID)
    k = max(0, len(ev) - n_tail)
    flags = list(orc.run_events(ev[:k], want_stage_out=False)[0]) if k else []
    rows = {}
    for i in range(k, len(ev)):
        f, _ = orc.run_events(ev[i:i + 1], want_stage_out=False)
        flags.append(f[0])
        if f[0] & abi.F_R4:
            cell = (int(ev[i, 2]) >> 3) * 10 + (int(ev[i, 1]) >> 3)
            rows[i] = orc.preds_dec()[cell].copy()
    return orc, np.array(flags, np.uint8), rows


def test_serve_rings_replay_matches_oracle(oracle_mod, stub_dir):
    from ssla_rt_b200.engine import SslaEngine
    from ssla_rt_b200.rings import Replay, RingSet
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    streams = [E.config_events(4, n=n, stream=s) if n else np.zeros((0, 4), np.float32)
               for s, n in enumerate((3000, 1700, 0, 2600))]
    P, cap = len(streams), 1024
    eng = SslaEngine(d, n_partitions=P, max_events=P * 400, layout=abi.LAYOUT_HYBRID,
                     max_events_per_partition=400)
    rings = RingSet(P, cap, cols=5 + eng.ncls)
    eng.rings_attach(rings)
    hist = [np.full(3001, 255, np.uint8) for s in streams]
    rp = Replay(rings, streams, time_scale=0.0)
    try:
        out = eng.serve_rings(300, sum(len(s) for s in streams), idle_timeout_ms=5000, log_cap=1000,
                              flags_hist=hist)
    finally:
        rp.stop()
        st = rp.join()
    torch.cuda.synchronize()
    assert out["served"] == st["published"] == sum(len(s) for s in streams)
    assert out["drains"] == len(out["done_ns"]) >= 8
    assert (out["taken"] <= 300).all()
    np.testing.assert_array_equal(out["taken"].sum(axis=0), [len(s) for s in streams])
    for r, ev in enumerate(streams):
        assert rings.head(r) == rings.tail(r) == rings.done(r) == len(ev)
        orc, flags, rows = _oracle_tail_preds(O, d, ev, cap)
        np.testing.assert_array_equal(hist[r][:len(ev)], flags, err_msg=f"flags of stream {r}")
        for i, row in rows.items():
            np.testing.assert_array_equal(rings.preds[r, i % cap], row, err_msg=f"pred row {i} of stream {r}")
        for l in range(8):
            np.testing.assert_array_equal(eng.hidden(l, r), orc.hidden(l), err_msg=f"hidden {l} stream {r}")
        for g in range(4):
            np.testing.assert_array_equal(eng.counters(g, r), orc.counters(g))
        np.testing.assert_array_equal(eng.last_t(r), orc.last_t())
        np.testing.assert_array_equal(eng.preds_dec(r), orc.preds_dec())
        np.testing.assert_array_equal(eng.version(r), orc.version())
    eng.close()


def test_drain_rings_protocol(oracle_mod, stub_dir):
    """Host-published slots: per-ring budget, total budget, tail and
    events_done words, flags in the ring's slots, and a refused head."""
    from ssla_rt_b200.engine import SslaEngine, SslaError
    from ssla_rt_b200.rings import RingSet
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    ev = [E.config_events(4, n=900, stream=10 + s) for s in range(3)]
    eng = SslaEngine(d, n_partitions=3, max_events=3 * 512, layout=abi.LAYOUT_HYBRID,
                     max_events_per_partition=512)
    rings = RingSet(3, 256, cols=5 + eng.ncls)
    eng.rings_attach(rings)
    assert eng.drain_rings(64).sum() == 0                    # nothing published: no work
    pub = [0, 0, 0]

    def publish(r, k):
        for i in range(pub[r], pub[r] + k):
            rings.events[r, i % 256] = ev[r][i]
        pub[r] += k
        rings.words[r, 0] = pub[r]

    publish(0, 200); publish(1, 10)
    taken = eng.drain_rings(64)
    np.testing.assert_array_equal(taken, [64, 10, 0])
    taken = eng.drain_rings(64, max_total=70)
    np.testing.assert_array_equal(taken, [64, 0, 0])
    torch.cuda.synchronize()
    assert [rings.tail(r) for r in range(3)] == [128, 10, 0]
    assert [rings.done(r) for r in range(3)] == [128, 10, 0]
    publish(2, 256)
    publish(0, 184)                                           # ring 0: 256 outstanding
    rings.words[1, 0] = 267                                   # 257 outstanding on ring 1
    with pytest.raises(SslaError):
        eng.drain_rings(512)
    rings.words[1, 0] = 10                                    # ring 1 stalls at 10 events
    while True:
        taken = eng.drain_rings(100)
        if taken.sum() == 0:
            break
        torch.cuda.synchronize()
        for r in (0, 2):
            if pub[r] < len(ev[r]) and rings.tail(r) == pub[r]:
                publish(r, min(256, len(ev[r]) - pub[r]))
    torch.cuda.synchronize()
    assert [rings.done(r) for r in range(3)] == [900, 10, 900]
    for r in range(3):
        n = pub[r]
        orc = O.Oracle(O.load_npz(d), 64, 80, 4, abi.LAYOUT_HYBRID)
        flags, _ = orc.run_events(ev[r][:n], want_stage_out=False)
        last = np.arange(max(0, n - 256), n)
        np.testing.assert_array_equal(rings.flags[r, last % 256], flags[last])
        np.testing.assert_array_equal(eng.hidden(7, r), orc.hidden(7))
        np.testing.assert_array_equal(eng.preds_dec(r), orc.preds_dec())
    eng.close()


def test_serve_rings_paced_latency_log(stub_dir):
    """Real-time replay (2 Mev/s per stream): every drain is logged after
    the due time of the events it holds, and each ring's events_done ends
    at its stream length."""
    from ssla_rt_b200.engine import SslaEngine
    from ssla_rt_b200.rings import Replay, RingSet
    d = stub_dir(64, 80, 1, 4)
    streams = [E.config_events(4, n=20_000, stream=s) for s in range(4)]
    eng = SslaEngine(d, n_partitions=4, max_events=4 * 8192, layout=abi.LAYOUT_HYBRID,
                     max_events_per_partition=8192)
    rings = RingSet(4, 1 << 14, cols=5 + eng.ncls)
    eng.rings_attach(rings)
    rp = Replay(rings, streams, time_scale=1.0)
    try:
        out = eng.serve_rings(8192, 80_000, idle_timeout_ms=5000, log_cap=100_000)
    finally:
        rp.stop()
        st = rp.join()
    assert out["served"] == 80_000
    cum = np.cumsum(out["taken"], axis=0)
    for r, ev in enumerate(streams):
        due = st["start_ns"] + ev[:, 0].astype(np.float64) * 1000.0
        k = np.searchsorted(cum[:, r], np.arange(len(ev)), side="right")   # drain holding event i
        lat = out["done_ns"][k].astype(np.float64) - due
        assert (lat > 0).all()
        assert rings.done(r) == len(ev)
    eng.close()
