"""Exact strip sharding (ssla_engine_strip_*): strips exchanging the next-layer
inputs of their boundary-band events after every layer give, for the events
and cells each strip owns, exactly the single-sensor engine's results --
flags, hidden state of every stage, gate counters, predictions and
versions -- across consecutive drains, including drains where some strips
have no events.  The strips share one GPU here and
run in lockstep (ssla_strip_drain_lockstep); across GPUs the same steps
wait for the neighbours' rows on the device."""
import numpy as np
import pytest

from ssla_rt_b200 import abi, strips
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CH = (12, 24, 48, 96)


def _rows(a, cols, s, lo, hi, ch=None):
    """Rows [lo >> s, hi >> s) of a per-cell array on the stage-s grid."""
    H, W = 256 >> s, 320 >> s
    a = a.reshape(H, W, -1) if ch else a.reshape(H, W)
    return a[lo >> s:hi >> s]


@pytest.mark.parametrize("n_strips,window", [(4, 4), (3, 1)])
def test_exact_strips_lockstep(stub_dir, n_strips, window):
    from ssla_rt_b200.engine import SslaEngine, strip_drain_lockstep
    H, W = 256, 320
    d = stub_dir(H, W, 1, window)
    ev = E.make_events(180_000, H, W, rate_mev=20.0, seed=11, n_blobs=16, blob_frac=0.7, sigma=4.0)
    late = ev[160_000:]
    chunks = [ev[:90_000], ev[90_000:160_000], late[late[:, 2] < 40]]    # the last: most strips empty
    full = SslaEngine(d, n_partitions=1, max_events=90_000, layout=abi.LAYOUT_HYBRID)
    bounds = strips.strip_bounds(H, n_strips)
    engs = []
    for r, (lo, hi) in enumerate(bounds):
        e = SslaEngine(d, n_partitions=1, max_events=90_000, layout=abi.LAYOUT_HYBRID)
        # a different exchange capacity per strip, as ranks sized by their own
        # routed events have: senders lay rows out by the receiver's capacity
        e.strip_init(lo, hi, 16, r > 0, r < n_strips - 1, 30_000 + 9_000 * r)
        engs.append(e)
    for r in range(n_strips):
        if r > 0:
            engs[r].strip_connect(0, peer_ptr=engs[r - 1].strip_recv_buffer(1)[0])
        if r < n_strips - 1:
            engs[r].strip_connect(1, peer_ptr=engs[r + 1].strip_recv_buffer(0)[0])
    for ch in chunks:
        ff = torch.zeros(len(ch), dtype=torch.uint8, device="cuda")
        full.drain(torch.from_numpy(np.ascontiguousarray(ch)).cuda(), [0, len(ch)], flags=ff)
        fflags = ff.cpu().numpy()
        sev, sfl, masks = [], [], []
        for lo, hi in bounds:
            m = strips.route_mask(ch, lo, hi, H, 16)
            masks.append(m)
            sev.append(torch.from_numpy(np.ascontiguousarray(ch[m])).cuda())
            sfl.append(torch.zeros(int(m.sum()), dtype=torch.uint8, device="cuda"))
        strip_drain_lockstep(engs, sev, sfl)
        torch.cuda.synchronize()
        idx = np.arange(len(ch))
        for (lo, hi), m, f in zip(bounds, masks, sfl):
            own = strips.owned_mask(ch[m], lo, hi)
            np.testing.assert_array_equal(f.cpu().numpy()[own], fflags[idx[m][own]])
    for e in engs:
        assert e.strip_status() == 0
    for (lo, hi), e in zip(bounds, engs):
        for l in range(8):
            s = l // 2
            np.testing.assert_array_equal(_rows(e.hidden(l), CH[s], s, lo, hi, True),
                                          _rows(full.hidden(l), CH[s], s, lo, hi, True), err_msg=f"hidden {l}")
        for g, s in enumerate((1, 2, 2, 3)):
            np.testing.assert_array_equal(_rows(e.counters(g), 1, s, lo, hi), _rows(full.counters(g), 1, s, lo, hi))
        np.testing.assert_array_equal(_rows(e.preds_dec(), 7, 3, lo, hi, True),
                                      _rows(full.preds_dec(), 7, 3, lo, hi, True))
        np.testing.assert_array_equal(_rows(e.version(), 1, 3, lo, hi), _rows(full.version(), 1, 3, lo, hi))
        e.close()
    full.close()
