"""Stages 0-1 on the GPU behind the libstage01_to_gpu ABI.

* ssla_engine_drain_records: the ring records (t, stage-2 x / y, feat1 =
  stage-1 output) of the events that pass gates 0 and 1, exactly the
  oracle's stage-1 outputs, with the stage-0/1 state and counters exact.
* s01g_*: submitted events come out of the attached rings with the
  reference's protocol (seq_done = slot + 1, routing by stage-2 ranges with
  overlap, push / emit stamps) and statistics.
* s01g rings drained by ssla_s2s3_drain_n_multi reproduce the single-pass
  engine exactly (stage-2/3 state, tdrop_s2 / tdrop_s3 counters, s3_feat
  of records that reach the head).
"""
import numpy as np
import pytest

from ssla_rt_b200 import abi, stub
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

REC = abi.INPUT_DTYPE


def _oracle_run(O, d, ev):
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    flags, so = orc.run_events(ev)
    return orc, flags, so


def test_drain_records_match_oracle(oracle_mod, stub_dir):
    from ssla_rt_b200.engine import SslaEngine
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=20000)
    n = len(ev)
    eng = SslaEngine(d, n_partitions=1, max_events=n, layout=abi.LAYOUT_HYBRID)
    t = torch.from_numpy(np.ascontiguousarray(ev)).cuda()
    rec = torch.zeros(n * REC.itemsize, dtype=torch.uint8, device="cuda")
    flags = torch.zeros(n, dtype=torch.uint8, device="cuda")
    off = eng.drain_records(t, [0, n], rec, n, flags)
    orc, oflags, so = _oracle_run(oracle_mod, d, ev)
    np.testing.assert_array_equal(flags.cpu().numpy(), oflags & (abi.F_VALID | abi.F_R1 | abi.F_R2))
    r2 = (oflags & abi.F_R2) != 0
    assert off[0] == 0 and off[1] == int(r2.sum()) > 0
    recs = rec.cpu().numpy().view(REC)[: off[1]]
    np.testing.assert_array_equal(recs["t"], ev[r2, 0])
    np.testing.assert_array_equal(recs["x"], ev[r2, 1].astype(np.int64) >> 2)
    np.testing.assert_array_equal(recs["y"], ev[r2, 2].astype(np.int64) >> 2)
    np.testing.assert_array_equal(recs["feat1"], so[1][r2])
    assert (recs["seq_done"] == 0).all()
    for l in range(4):
        np.testing.assert_array_equal(eng.hidden(l), orc.hidden(l), err_msg=f"hidden {l}")
    for g in range(2):
        np.testing.assert_array_equal(eng.counters(g), orc.counters(g), err_msg=f"counter {g}")
    for g in range(2, 4):                      # later gates belong to the GPU drain
        assert (eng.counters(g) == 0).all()
    eng.close()


def test_s01g_rings_match_oracle(oracle_mod, stub_dir):
    from ssla_rt_b200.s01g import S01gAPI
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=12000)
    oob = np.array([[1.0, -1.0, 5.0, 1.0], [2.0, 80.0, 5.0, 1.0], [3.0, 5.0, 64.0, 1.0]], np.float32)
    api = S01gAPI()
    api.init(d, n_shards=4, halo=2)
    cap = 1 << 14
    rings = [np.zeros(cap, dtype=REC) for _ in range(2)]
    heads = [np.zeros(1, dtype=np.uint64) for _ in range(2)]
    W2, H2 = 20, 16
    ranges = [(0, 12), (8, 20)]                  # overlapping stage-2 x ranges
    api.attach(rings[0].ctypes.data, heads[0].ctypes.data, rings[1].ctypes.data, heads[1].ctypes.data,
               cap - 1, W2, H2, ranges[0][0], ranges[0][1], ranges[1][0], ranges[1][1])
    accepted = sum(api.submit(c) for c in np.array_split(ev, 7))
    accepted += api.submit(oob)
    assert accepted == len(ev)
    assert api.flush(120.0)
    st = api.snapshot()
    _, oflags, so = _oracle_run(oracle_mod, d, ev)
    r2 = (oflags & abi.F_R2) != 0
    x2 = ev[r2, 1].astype(np.int64) >> 2
    y2 = ev[r2, 2].astype(np.int64) >> 2
    for b, (lo, hi) in enumerate(ranges):
        sel = (x2 >= lo) & (x2 < hi)
        n = int(sel.sum())
        assert int(heads[b][0]) == n
        r = rings[b][:n]
        np.testing.assert_array_equal(r["seq_done"], np.arange(1, n + 1, dtype=np.uint64))
        np.testing.assert_array_equal(r["t"], ev[r2, 0][sel])
        np.testing.assert_array_equal(r["x"], x2[sel])
        np.testing.assert_array_equal(r["y"], y2[sel])
        np.testing.assert_array_equal(r["feat1"], so[1][r2][sel])
        assert (r["t_emit_ns"] > 0).all() and (r["t_push_ns"] >= r["t_emit_ns"]).all()
        assert st[14 + b] == n
    assert st[0] == len(ev) and st[1] == 0 and st[3] == 3
    assert st[2] == int(((oflags & abi.F_R1) != 0).sum())
    assert st[13] == int(r2.sum())
    assert st[12] > 0 and 0 < st[6] <= st[8] <= st[10]
    api.shutdown()


def test_s01g_then_drain_n_equals_single_pass_engine(oracle_mod, stub_dir):
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200.engine import SslaEngine, drain_n_multi
    from ssla_rt_b200.s01g import S01gAPI
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=16000)
    n = len(ev)
    full = SslaEngine(d, n_partitions=1, max_events=n, layout=abi.LAYOUT_HYBRID, record_stage_outputs=True)
    fflags = torch.zeros(n, dtype=torch.uint8, device="cuda")
    full.drain(torch.from_numpy(np.ascontiguousarray(ev)).cuda(), [0, n], flags=fflags)
    torch.cuda.synchronize()
    fl = fflags.cpu().numpy()

    api = S01gAPI()
    api.init(d)
    cap = 1 << 14
    ring = np.zeros(cap, dtype=REC)
    head = np.zeros(1, dtype=np.uint64)
    api.attach_multi([ring.ctypes.data], [head.ctypes.data], cap - 1, 20, 16, [0], [20], [0], [16])
    api.submit(ev)
    assert api.flush(120.0)
    nrec = int(head[0])
    assert nrec == int(((fl & abi.F_R2) != 0).sum())
    api.shutdown()

    rng = np.random.default_rng(0)
    cfg, keep, _, hid, td2, td3 = build_cfg(oracle_mod, stub.stub_tensors(seed=1), 16, 20, 4, 1,
                                            [(0, 20)], rng)
    for h in hid:
        h.zero_()
    rec_dev = torch.from_numpy(ring[:nrec].view(np.uint8).copy()).cuda()
    out = torch.zeros(nrec * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda")
    drain_n_multi(cfg, [rec_dev.data_ptr()], [nrec], [out.data_ptr()])
    torch.cuda.synchronize()
    for li in range(4):
        np.testing.assert_array_equal(hid[li].cpu().numpy(), full.hidden(4 + li), err_msg=f"hidden {4 + li}")
    np.testing.assert_array_equal(td2[0].cpu().numpy(), full.counters(2))
    np.testing.assert_array_equal(td3[0].cpu().numpy(), full.counters(3))
    o = out.cpu().numpy().view(abi.OUTPUT_DTYPE)
    r2 = (fl & abi.F_R2) != 0
    np.testing.assert_array_equal(o["pass2"], ((fl[r2] & abi.F_R3) != 0).astype(np.int32))
    np.testing.assert_array_equal(o["pass3"], ((fl[r2] & abi.F_R4) != 0).astype(np.int32))
    head_rows = full.stage_out(3, n)[(fl & abi.F_R4) != 0]
    np.testing.assert_array_equal(o["s3_feat"][o["pass3"] == 1], head_rows)
    del keep
    full.close()


def test_s01g_synthetic_producer(stub_dir):
    from ssla_rt_b200.s01g import S01gAPI
    import time
    d = stub_dir(64, 80, 1, 4)
    api = S01gAPI()
    api.init(d)
    cap = 1 << 16
    ring = np.zeros(cap, dtype=REC)
    head = np.zeros(1, dtype=np.uint64)
    api.attach_multi([ring.ctypes.data], [head.ctypes.data], cap - 1, 20, 16, [0], [20], [0], [16])
    api.start_synthetic(1.0, -1, 7)
    time.sleep(0.3)
    api.stop_synthetic()
    pushed = api.synthetic_n_pushed()
    assert api.flush(120.0)
    st = api.snapshot()
    assert pushed > 10000
    assert st[0] == pushed and st[3] == 0
    assert st[13] == int(head[0]) == st[14] > 0
    n = min(int(head[0]), cap)
    r = ring[:n]
    assert (r["x"] < 20).all() and (r["y"] < 16).all()
    assert (np.diff(r["t"]) > 0).all()
    api.shutdown()
