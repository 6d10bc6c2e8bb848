"""Strip-sharded 320x256 sensor on the GPU engine (one strip per engine, as
one per GPU): each strip's engine, given its owned stage-2 rows, equals the
oracle run on the same routed events bit for bit (hidden state, counters,
and the predictions / versions of owned cells), and the flags of owned
events equal the full-frame run's exactly (drop drift 0)."""
import numpy as np
import pytest

from ssla_rt_b200 import abi, strips
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("n_strips,halo", [(4, 16), (8, 8)])
def test_strip_engines(oracle_mod, stub_dir, n_strips, halo):
    from ssla_rt_b200.engine import SslaEngine
    O = oracle_mod
    H, W = 256, 320
    d = stub_dir(H, W, 1, 4)
    ev = E.make_events(120_000, H, W, rate_mev=20.0, seed=7, n_blobs=16, blob_frac=0.7, sigma=4.0)
    full = SslaEngine(d, n_partitions=1, max_events=len(ev), layout=abi.LAYOUT_HYBRID)
    ff = torch.zeros(len(ev), dtype=torch.uint8, device="cuda")
    full.drain(torch.from_numpy(ev).cuda(), [0, len(ev)], flags=ff)
    fflags = ff.cpu().numpy()
    full.close()
    idx = np.arange(len(ev))
    tensors = O.load_npz(d)
    for lo, hi in strips.strip_bounds(H, n_strips):
        m = strips.route_mask(ev, lo, hi, H, halo)
        sev = np.ascontiguousarray(ev[m])
        eng = SslaEngine(d, n_partitions=1, max_events=len(sev), layout=abi.LAYOUT_HYBRID)
        eng.set_owned(0, *strips.owned_s2(lo, hi, W))
        sf = torch.zeros(len(sev), dtype=torch.uint8, device="cuda")
        eng.drain(torch.from_numpy(sev).cuda(), [0, len(sev)], flags=sf)
        sflags = sf.cpu().numpy()
        own = strips.owned_mask(sev, lo, hi)
        np.testing.assert_array_equal(sflags[own], fflags[idx[m][own]])       # drop drift 0
        orc = O.Oracle(tensors, H, W, 4, O.LAYOUT_HYBRID)
        oflags, _ = orc.run_events(sev, want_stage_out=False)
        np.testing.assert_array_equal(sflags, oflags)
        for l in range(8):
            np.testing.assert_array_equal(eng.hidden(l), orc.hidden(l), err_msg=f"hidden {l}")
        for g in range(4):
            np.testing.assert_array_equal(eng.counters(g), orc.counters(g))
        rows3 = np.arange((H >> 3) * (W >> 3)) // (W >> 3)
        mine = (rows3 >= lo // 8) & (rows3 < hi // 8)
        np.testing.assert_array_equal(eng.preds_dec()[mine], orc.preds_dec()[mine])
        np.testing.assert_array_equal(eng.version()[mine], orc.version()[mine])
        assert (eng.version()[~mine] == 0).all()                               # halo cells commit nothing
        eng.close()
