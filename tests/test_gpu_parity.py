"""CUDA engine vs the CPU oracle on seeded inputs, through the C ABI.

The engine and the oracle share one arithmetic contract (fmaf chains in the
reference's loop order, sequential fp64 LayerNorm sums, the portable exp), so
every comparison here is exact: gate flags, stage outputs, hidden state of
all eight layers, counters, last timestamps, predictions and versions.
"""
import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _engine(d, **kw):
    from ssla_rt_b200.engine import SslaEngine
    return SslaEngine(d, **kw)


def run_oracle(O, d, h, w, tdrop, layout, parts):
    """Oracle per partition (independent streams): flags, stage outs, state."""
    out = []
    for ev in parts:
        orc = O.Oracle(O.load_npz(d), h, w, tdrop, layout)
        flags, so = orc.run_events(ev)
        out.append((orc, flags, so))
    return out


def assert_engine_equals_oracle(eng, oracles, parts, layout):
    n = sum(len(p) for p in parts)
    flags = eng.flags(n)
    so = [eng.stage_out(s, n) for s in range(4)]
    base = 0
    for p, (orc, oflags, oso) in enumerate(oracles):
        k = len(parts[p])
        sl = slice(base, base + k)
        np.testing.assert_array_equal(flags[sl], oflags, err_msg=f"flags p{p}")
        for s in range(4):
            bit = (abi.F_R1 << s) if s < 3 else abi.F_R4
            m = (oflags & bit) != 0
            np.testing.assert_array_equal(so[s][sl][m], oso[s][m], err_msg=f"stage {s} p{p}")
        for l in range(8):
            np.testing.assert_array_equal(eng.hidden(l, p), orc.hidden(l), err_msg=f"hidden {l} p{p}")
        for g in range(4 if layout == abi.LAYOUT_HYBRID else 3):
            np.testing.assert_array_equal(eng.counters(g, p), orc.counters(g), err_msg=f"cnt {g} p{p}")
        np.testing.assert_array_equal(eng.last_t(p), orc.last_t(), err_msg=f"last_t p{p}")
        np.testing.assert_array_equal(eng.preds_dec(p), orc.preds_dec(), err_msg=f"preds p{p}")
        np.testing.assert_array_equal(eng.preds_raw(p), orc.preds_raw(), err_msg=f"raw p{p}")
        np.testing.assert_array_equal(eng.version(p), orc.version(), err_msg=f"version p{p}")
        base += k


def drain_device(eng, parts, off=None):
    ev = np.concatenate(parts) if parts else np.zeros((0, 4), np.float32)
    off = eng.offsets([len(p) for p in parts]) if off is None else off
    t = torch.from_numpy(np.ascontiguousarray(ev, np.float32)).cuda()
    eng.drain(t, off)
    torch.cuda.synchronize()


@pytest.mark.parametrize("layout", [abi.LAYOUT_DECOMP, abi.LAYOUT_HYBRID])
def test_config0_slice_single_stream(oracle_mod, stub_dir, layout):
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=6000)
    eng = _engine(d, n_partitions=1, max_events=6000, layout=layout, record_stage_outputs=True)
    drain_device(eng, [ev])
    assert_engine_equals_oracle(eng, run_oracle(oracle_mod, d, 64, 80, 4, layout, [ev]), [ev], layout)


@pytest.mark.parametrize("layout", [abi.LAYOUT_DECOMP, abi.LAYOUT_HYBRID])
def test_partitions_ragged_and_empty(oracle_mod, stub_dir, layout):
    """Independent ring partitions of different sizes, one of them empty."""
    d = stub_dir(64, 80, 1, 4)
    full = E.config_events(1, n=9000)
    parts = [full[:4000], full[4000:4000], full[4000:4100], full[4100:]]
    eng = _engine(d, n_partitions=4, max_events=9000, layout=layout, record_stage_outputs=True,
                  max_events_per_partition=5000)
    drain_device(eng, parts)
    assert_engine_equals_oracle(eng, run_oracle(oracle_mod, d, 64, 80, 4, layout, parts), parts, layout)


def test_all_events_pass_small_grid(oracle_mod, stub_dir):
    """Window 1: every event reaches every stage; 16x16 makes most events
    boundary events at s2/s3 (2x2 cells)."""
    d = stub_dir(16, 16, 5, 1)
    ev = E.make_events(1500, 16, 16, rate_mev=1.0, seed=12)
    eng = _engine(d, n_partitions=1, max_events=1500, layout=abi.LAYOUT_HYBRID, record_stage_outputs=True)
    drain_device(eng, [ev])
    assert_engine_equals_oracle(eng, run_oracle(oracle_mod, d, 16, 16, 1, abi.LAYOUT_HYBRID, [ev]),
                                [ev], abi.LAYOUT_HYBRID)


def test_window3_hot_cells_and_invalid_events(oracle_mod, stub_dir):
    """Window 3 (counter wrap mod 256 matters), clustered hot cells, and
    out-of-bounds / NaN coordinates (skipped, as the reference drivers do)."""
    d = stub_dir(16, 24, 6, 3)
    ev = E.make_events(5000, 16, 24, rate_mev=3.0, seed=13, n_blobs=2, blob_frac=0.8, sigma=1.0)
    ev[::53, 1] = -1.0
    ev[7::61, 2] = 16.0
    ev[11::71, 1] = np.nan
    ev[13::79, 1] = -0.5          # truncates to 0: valid, like the reference's (int) cast
    eng = _engine(d, n_partitions=1, max_events=5000, layout=abi.LAYOUT_DECOMP, record_stage_outputs=True)
    drain_device(eng, [ev])
    assert_engine_equals_oracle(eng, run_oracle(oracle_mod, d, 16, 24, 3, abi.LAYOUT_DECOMP, [ev]),
                                [ev], abi.LAYOUT_DECOMP)


def test_hot_tiles_scanned_cell_by_cell(oracle_mod, stub_dir):
    """A near-stationary blob puts most of 40,000 events into one s3 block:
    its stage-0 and stage-1 tile lists exceed the hot-tile bound, so those
    tiles are scanned with one work item per cell; a second partition stays
    uniform.  Everything still equals the oracle."""
    d = stub_dir(64, 80, 1, 4)
    hot = E.make_events(40_000, 64, 80, rate_mev=5.0, seed=21, n_blobs=1, blob_frac=0.97, sigma=2.0,
                        speed_px_per_ms=(0.0, 0.05))
    parts = [hot, E.config_events(0, n=3000, seed=22)]
    eng = _engine(d, n_partitions=2, max_events=43_000, layout=abi.LAYOUT_HYBRID, record_stage_outputs=True,
                  max_events_per_partition=40_000)
    drain_device(eng, parts)
    oracles = run_oracle(oracle_mod, d, 64, 80, 4, abi.LAYOUT_HYBRID, parts)
    assert_engine_equals_oracle(eng, oracles, parts, abi.LAYOUT_HYBRID)


def test_state_carries_across_drains(oracle_mod, stub_dir):
    """Three consecutive drain calls == one sequential run."""
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(2, n=12000)
    eng = _engine(d, n_partitions=1, max_events=5000, layout=abi.LAYOUT_HYBRID)
    for chunk in (ev[:5000], ev[5000:5001], ev[5001:10000], ev[10000:]):
        drain_device(eng, [chunk])
    orc = oracle_mod.Oracle(oracle_mod.load_npz(d), 64, 80, 4, oracle_mod.LAYOUT_HYBRID)
    orc.run_events(ev, want_stage_out=False)
    for l in range(8):
        np.testing.assert_array_equal(eng.hidden(l), orc.hidden(l))
    np.testing.assert_array_equal(eng.preds_dec(), orc.preds_dec())
    np.testing.assert_array_equal(eng.version(), orc.version())


def test_host_path_and_reset(oracle_mod, stub_dir):
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=3000)
    eng = _engine(d, n_partitions=1, max_events=3000)
    flags = np.zeros(3000, np.uint8)
    eng.drain_host(np.ascontiguousarray(ev), eng.offsets([3000]), flags)
    eng.reset()
    torch.cuda.synchronize()
    eng.drain_host(np.ascontiguousarray(ev), eng.offsets([3000]), flags)
    orc = oracle_mod.Oracle(oracle_mod.load_npz(d), 64, 80, 4, oracle_mod.LAYOUT_HYBRID)
    oflags, _ = orc.run_events(ev, want_stage_out=False)
    np.testing.assert_array_equal(flags, oflags)
    np.testing.assert_array_equal(eng.preds_dec(), orc.preds_dec())


def test_capacity_errors_are_reported(stub_dir):
    from ssla_rt_b200.engine import SslaError
    d = stub_dir(64, 80, 1, 4)
    eng = _engine(d, n_partitions=2, max_events=100)
    ev = torch.zeros((150, 4), device="cuda")
    with pytest.raises(SslaError) as ei:
        eng.drain(ev, np.array([0, 50, 150], np.int32))
    assert ei.value.code == abi.SSLA_ERR_CAPACITY
    with pytest.raises(SslaError) as ei:
        eng.drain(ev, np.array([0, 60, 50], np.int32))
    assert ei.value.code == abi.SSLA_ERR_ARG


def test_config1_full_size(oracle_mod, stub_dir):
    """The bench workload itself (config 1: 200,000 uniform events at 80x64 in
    8 partitions of 25,000, HYBRID gates), two consecutive drains (the
    streams continue), compared exactly with the oracle run over the same
    event streams."""
    d = stub_dir(64, 80, 1, 4)
    parts = E.split_partitions(E.config_events(1), 8)
    span = float(max(p[:, 0].max() for p in parts)) + 1.0
    second = [p.copy() for p in parts]
    for p in second:
        p[:, 0] += span
    eng = _engine(d, n_partitions=8, max_events=200_000, layout=abi.LAYOUT_HYBRID,
                  record_stage_outputs=True, max_events_per_partition=max(len(p) for p in parts))
    drain_device(eng, parts)
    drain_device(eng, second)
    oracles = []
    for a, b in zip(parts, second):
        orc = oracle_mod.Oracle(oracle_mod.load_npz(d), 64, 80, 4, abi.LAYOUT_HYBRID)
        orc.run_events(a, want_stage_out=False)
        flags, so = orc.run_events(b)
        oracles.append((orc, flags, so))
    assert_engine_equals_oracle(eng, oracles, second, abi.LAYOUT_HYBRID)


@pytest.mark.parametrize("outputs", ["pinned", "pageable"])
def test_pipelined_host_drains_match_sync(stub_dir, outputs):
    """ssla_engine_drain_host_async (copies on the engine's copy stream,
    two device buffers in turn; results written into pinned outputs by a
    kernel chained to the drain, or copied back into pageable ones) gives,
    drain for drain, the flags, predictions and state of the synchronous
    host path, with several drains in flight."""
    d = stub_dir(64, 80, 1, 4)
    parts = E.split_partitions(E.config_events(1, n=40_000, seed=31), 4)
    base = np.ascontiguousarray(np.concatenate(parts))
    span = float(base[:, 0].max()) + 1.0
    off = np.array([0] + list(np.cumsum([len(p) for p in parts])), np.int32)
    n = len(base)
    sync = _engine(d, n_partitions=4, max_events=n, layout=abi.LAYOUT_HYBRID,
                   max_events_per_partition=max(len(p) for p in parts))
    pipe = _engine(d, n_partitions=4, max_events=n, layout=abi.LAYOUT_HYBRID,
                   max_events_per_partition=max(len(p) for p in parts))
    steps = 4
    ins = [torch.from_numpy(base.copy()).pin_memory() for _ in range(steps)]
    for k in range(steps):
        ins[k][:, 0] += span * k
    pin = (lambda t: t.pin_memory()) if outputs == "pinned" else (lambda t: t)
    flags = [pin(torch.zeros(n, dtype=torch.uint8)) for _ in range(steps)]
    preds = [pin(torch.zeros(tuple(sync.preds_dec_all().shape), dtype=torch.float32)) for _ in range(steps)]
    stream = torch.cuda.current_stream()
    for k in range(steps):
        pipe.drain_host_async(ins[k], off, flags[k], preds[k], stream=stream)
    torch.cuda.synchronize()
    for k in range(steps):
        f = np.zeros(n, np.uint8)
        sync.drain_host(ins[k].numpy(), off, f)
        np.testing.assert_array_equal(flags[k].numpy(), f, err_msg=f"flags of drain {k}")
        np.testing.assert_array_equal(preds[k].numpy(), sync.preds_dec_all(), err_msg=f"preds of drain {k}")
    for p in range(4):
        for l in range(8):
            np.testing.assert_array_equal(pipe.hidden(l, p), sync.hidden(l, p))
        np.testing.assert_array_equal(pipe.version(p), sync.version(p))
    sync.close()
    pipe.close()
