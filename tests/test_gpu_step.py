"""The single-event step (ssla_engine_step, one 9-CTA cluster launch per
event) against the oracle: stepping a stream event by event leaves exactly
the oracle's state (all hidden layers, counters, last timestamps,
predictions, versions), the per-event flags are the oracle's, and the
prediction row written for each head event is the oracle's row of that
cell at that moment.  Steps and chunk drains interleave on one state."""
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


@pytest.mark.parametrize("layout,window,n", [(abi.LAYOUT_HYBRID, 4, 2500), (abi.LAYOUT_DECOMP, 2, 1200)])
def test_steps_match_oracle(oracle_mod, stub_dir, layout, window, n):
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    d = stub_dir(64, 80, 1, window)
    ev = E.config_events(0, n=n).copy()
    ev[7] = [ev[6, 0], -3.0, 5.0, 1.0]           # out of bounds: flags 0, no state change
    ev[11] = [ev[10, 0], 5.0, 64.0, -1.0]
    eng = SslaEngine(d, n_partitions=1, max_events=16, layout=layout)
    cols = 5 + eng.ncls
    flags = torch.zeros(n, dtype=torch.uint8, device="cuda")
    preds = torch.zeros((n, cols), dtype=torch.float32, device="cuda")
    for i in range(n):
        eng.step(ev[i], 0, flags[i:i + 1], preds[i])
    torch.cuda.synchronize()
    orc = O.Oracle(O.load_npz(d), 64, 80, window, layout)
    got_f = flags.cpu().numpy()
    got_p = preds.cpu().numpy()
    heads = 0
    for i in range(n):
        f, _ = orc.run_events(ev[i:i + 1], want_stage_out=False)
        assert got_f[i] == f[0], f"flags of event {i}"
        if f[0] & abi.F_R4:
            cell = (int(ev[i, 2]) >> 3) * (80 >> 3) + (int(ev[i, 1]) >> 3)
            np.testing.assert_array_equal(got_p[i], orc.preds_dec()[cell], err_msg=f"pred of event {i}")
            heads += 1
    assert heads > 0
    _assert_state(eng, orc, layout)
    eng.close()


def test_drain_then_steps_share_state(oracle_mod, stub_dir):
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=6000)
    eng = SslaEngine(d, n_partitions=1, max_events=6000, layout=abi.LAYOUT_HYBRID)
    eng.drain(torch.from_numpy(np.ascontiguousarray(ev[:5000])).cuda(), [0, 5000])
    for i in range(5000, 6000):
        eng.step(ev[i])
    torch.cuda.synchronize()
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    orc.run_events(ev, want_stage_out=False)
    _assert_state(eng, orc, abi.LAYOUT_HYBRID)
    eng.close()


def test_step_writes_pinned_host_outputs(stub_dir):
    from ssla_rt_b200.engine import SslaEngine
    d = stub_dir(64, 80, 1, 1)                   # window 1: every event reaches the head
    eng = SslaEngine(d, n_partitions=2, max_events=16, layout=abi.LAYOUT_HYBRID)
    flag = torch.zeros(1, dtype=torch.uint8).pin_memory()
    pred = torch.full((5 + eng.ncls,), -7.0, dtype=torch.float32).pin_memory()
    eng.step(np.array([10.0, 33.0, 20.0, 1.0], np.float32), 1, flag, pred)
    torch.cuda.synchronize()
    assert int(flag[0]) == abi.F_VALID | abi.F_R1 | abi.F_R2 | abi.F_R3 | abi.F_R4
    np.testing.assert_array_equal(pred.numpy(), eng.preds_dec(1)[(20 >> 3) * 10 + (33 >> 3)])
    assert eng.version(1).sum() == 1 and eng.version(0).sum() == 0
    eng.close()
