"""The live loop (ssla_engine_live_*: a resident cluster fed by a pinned host
ring of raw events) against the oracle: every event's flags, the decoded
prediction row of every head event, and the final state (hidden layers,
counters, last timestamps, predictions, versions) are the oracle's, for
events published one at a time and for a backlog published at once; the
loop ends on its stop flag or by itself when idle; the live loop, drains
and single-event steps advance one shared state."""
import time

import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _assert_state(eng, orc, layout, p=0):
    for l in range(8):
        np.testing.assert_array_equal(eng.hidden(l, p), orc.hidden(l), err_msg=f"hidden {l}")
    for g in range(4 if layout == abi.LAYOUT_HYBRID else 3):
        np.testing.assert_array_equal(eng.counters(g, p), orc.counters(g), err_msg=f"counter {g}")
    np.testing.assert_array_equal(eng.last_t(p), orc.last_t())
    np.testing.assert_array_equal(eng.preds_dec(p), orc.preds_dec())
    np.testing.assert_array_equal(eng.preds_raw(p), orc.preds_raw())
    np.testing.assert_array_equal(eng.version(p), orc.version())


def _check_events(orc, ev, flags, preds, W=80):
    heads = 0
    for i in range(len(ev)):
        f, _ = orc.run_events(ev[i:i + 1], want_stage_out=False)
        assert flags[i] == f[0], f"flags of event {i}"
        if f[0] & abi.F_R4:
            cell = (int(ev[i, 2]) >> 3) * (W >> 3) + (int(ev[i, 1]) >> 3)
            np.testing.assert_array_equal(preds[i], orc.preds_dec()[cell], err_msg=f"pred of event {i}")
            heads += 1
    return heads


@pytest.mark.parametrize("layout,window,n", [(abi.LAYOUT_HYBRID, 4, 3000), (abi.LAYOUT_DECOMP, 2, 1500)])
def test_live_one_at_a_time_matches_oracle(oracle_mod, stub_dir, layout, window, n):
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    d = stub_dir(64, 80, 1, window)
    ev = E.config_events(0, n=n).copy()
    ev[5] = [ev[4, 0], -2.0, 7.0, 1.0]            # out of bounds: flags 0, no state change
    ev[9] = [ev[8, 0], 12.0, 64.0, -1.0]
    eng = SslaEngine(d, n_partitions=2, max_events=16, layout=layout)
    lat, flags, preds = eng.live_latency(ev, partition=1)
    orc = O.Oracle(O.load_npz(d), 64, 80, window, layout)
    assert _check_events(orc, ev, flags, preds) > 0
    _assert_state(eng, orc, layout, p=1)
    assert eng.version(0).sum() == 0              # the other partition is untouched
    assert (lat > 0).all()
    eng.close()


def test_live_backlog_ring_and_stop(oracle_mod, stub_dir):
    """A Python-owned pinned ring: the whole stream published at once, the
    loop drains it in ring order, then ends on the stop flag."""
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    n, cap = 2500, 4096
    ev = E.config_events(0, n=n)
    eng = SslaEngine(d, n_partitions=1, max_events=16, layout=abi.LAYOUT_HYBRID)
    cols = 5 + eng.ncls
    events = torch.zeros((cap, 4), dtype=torch.float32).pin_memory()
    words = torch.zeros(8, dtype=torch.int64).pin_memory()     # head, tail, done, stop
    flags = torch.zeros(cap, dtype=torch.uint8).pin_memory()
    preds = torch.zeros((cap, cols), dtype=torch.float32).pin_memory()
    base = words.data_ptr()
    ring = abi.SslaLiveRing(events.data_ptr(), cap, base, base + 8, base + 16, flags.data_ptr(),
                            preds.data_ptr(), base + 24)
    events[:n] = torch.from_numpy(ev)
    words[0] = n                                     # publish everything (slots written first)
    eng.live_start(ring, idle_timeout_ms=5000)
    t0 = time.time()
    while int(words[2]) < n and time.time() - t0 < 60:
        time.sleep(0.01)
    words[3] = 1
    status = eng.live_join()
    assert status & abi.LIVE_EXIT_STOP and not status & 0xFF
    assert int(words[1]) == n and int(words[2]) == n
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    assert _check_events(orc, ev, flags.numpy()[:n], preds.numpy()[:n]) > 0
    _assert_state(eng, orc, abi.LAYOUT_HYBRID)
    eng.close()


def test_live_idle_exit_and_shared_state(oracle_mod, stub_dir):
    """Without events the loop leaves by itself; drain -> live -> steps
    advance one state exactly as the oracle's single stream."""
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    eng = SslaEngine(d, n_partitions=1, max_events=5000, layout=abi.LAYOUT_HYBRID)
    words = torch.zeros(8, dtype=torch.int64).pin_memory()
    events = torch.zeros((16, 4), dtype=torch.float32).pin_memory()
    base = words.data_ptr()
    ring = abi.SslaLiveRing(events.data_ptr(), 16, base, base + 8, base + 16, None, None, base + 24)
    eng.live_start(ring, idle_timeout_ms=50)
    status = eng.live_join()
    assert status & abi.LIVE_EXIT_IDLE and not status & 0xFF
    ev = E.config_events(0, n=7000)
    eng.drain(torch.from_numpy(np.ascontiguousarray(ev[:5000])).cuda(), [0, 5000])
    eng.live_latency(ev[5000:6500])
    for i in range(6500, 7000):
        eng.step(ev[i])
    torch.cuda.synchronize()
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    orc.run_events(ev, want_stage_out=False)
    _assert_state(eng, orc, abi.LAYOUT_HYBRID)
    eng.close()


def test_live_rejects_pageable_ring(stub_dir):
    from ssla_rt_b200.engine import SslaEngine, SslaError
    d = stub_dir(64, 80, 1, 4)
    eng = SslaEngine(d, n_partitions=1, max_events=16, layout=abi.LAYOUT_HYBRID)
    words = np.zeros(8, dtype=np.int64)              # pageable: the device must never touch it
    events = np.zeros((16, 4), dtype=np.float32)
    ring = abi.SslaLiveRing(events.ctypes.data, 16, words.ctypes.data, words.ctypes.data + 8,
                            words.ctypes.data + 16, None, None, words.ctypes.data + 24)
    with pytest.raises(SslaError):
        eng.live_start(ring)
    eng.close()


def test_live_timeout_path_ends_cleanly(oracle_mod, stub_dir):
    """The loop's error path, made to run on purpose without any fault: the
    test hook withholds the completion message of ring event 3 from the
    head CTA.  Events 0-2 finish; the head CTA's bounded wait for event 3
    runs out, so does the coordinator's wait for the head CTA's
    acknowledgement at event 4, and the workers' wait for the next event
    message.  Every CTA leaves through the exit barrier, the status word
    names the waits that ran out, and the context stays usable: a drain
    afterwards equals the oracle."""
    from ssla_rt_b200.engine import SslaEngine, SslaError
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    eng = SslaEngine(d, n_partitions=1, max_events=4000, layout=abi.LAYOUT_HYBRID)
    cap, n = 16, 8
    ev = E.config_events(0, n=4000)
    events = torch.zeros((cap, 4), dtype=torch.float32).pin_memory()
    words = torch.zeros(8, dtype=torch.int64).pin_memory()     # head, tail, done, stop
    base = words.data_ptr()
    ring = abi.SslaLiveRing(events.data_ptr(), cap, base, base + 8, base + 16, None, None, base + 24)
    events[:n] = torch.from_numpy(ev[:n])
    words[0] = n
    eng.live_withhold_completion(3)
    eng.live_start(ring, idle_timeout_ms=100)
    t0 = time.time()
    status = eng.live_join(check=False)
    assert time.time() - t0 < 30
    assert status & abi.LIVE_ERR_DONE
    assert not status & (abi.LIVE_EXIT_STOP | abi.LIVE_ERR_WEIGHTS)
    assert int(words[2]) == 3                     # events 0-2 finished, event 3 withheld
    taken = int(words[1])                         # the loop took events 0-4
    assert taken == 5
    eng.live_withhold_completion(taken)           # again, on the next loop's first event
    eng.live_start(ring, idle_timeout_ms=100)
    with pytest.raises(SslaError):                # a checked join raises the same status
        eng.live_join()
    eng.reset()
    torch.cuda.synchronize()
    eng.drain(torch.from_numpy(np.ascontiguousarray(ev)).cuda(), [0, len(ev)])
    torch.cuda.synchronize()
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    orc.run_events(ev, want_stage_out=False)
    _assert_state(eng, orc, abi.LAYOUT_HYBRID)
    eng.close()
