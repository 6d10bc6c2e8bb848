"""Acceptance parity at the BASELINE sizes.

* Config 0 in full (50,000 uniform events at 80x64, seed 0) through the
  engine and through the reference's own C++ pipeline (oracle/_ref, built
  from the reference sources by oracle/Makefile): drop drift 0 (every gate
  flag equal), max|d| s3_feat within the reference's P1 budget of 5.0
  (orin/bench_s2_s3_head_celled.py:285-332) and, stricter, every stage's
  output, the predictions and all hidden layers within the fp32 tolerance
  stated below.  The engine is also exactly the C restatement there.
* Config 2 in full (1,000,000 clustered events, one stream, the hot-cell
  path at full chain length) against the C restatement, exactly.

Stated per-stage fp32 tolerance against the reference build: 1e-3 absolute
on LayerNorm-normalised stage outputs, hidden state and predictions (+1e-4
relative for the decoded boxes).  The differences come from the reference's
std::exp and -ffast-math against the portable exp; measured on config 0
they are at most 2.6e-5 (stage 3) and 5.1e-4 (layer-7 hidden state).
"""
import os

import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL_STAGE = 1e-3
S3_FEAT_BUDGET = 5.0


def _stage_bit(s):
    return (abi.F_R1 << s) if s < 3 else abi.F_R4


def _run_engine(d, ev, h=64, w=80):
    from ssla_rt_b200.engine import SslaEngine
    eng = SslaEngine(d, n_partitions=1, max_events=len(ev), layout=abi.LAYOUT_HYBRID, record_stage_outputs=True)
    eng.drain(torch.from_numpy(np.ascontiguousarray(ev)).cuda(), [0, len(ev)])
    torch.cuda.synchronize()
    return eng


def test_config0_full_against_reference_build(oracle_mod, stub_dir):
    O = oracle_mod
    if not os.path.exists(O.REF_SO):
        pytest.skip("oracle/_ref not built (needs the reference sources: make -C oracle ref)")
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0)
    assert len(ev) == 50_000
    eng = _run_engine(d, ev)
    n = len(ev)
    flags = eng.flags(n)
    so = [eng.stage_out(s, n) for s in range(4)]
    ref = O.RefPipeline(d, O.LAYOUT_HYBRID)
    rflags, rso = ref.run_events(ev)
    assert int((flags != rflags).sum()) == 0, "drop drift"
    for s in range(4):
        m = (rflags & _stage_bit(s)) != 0
        assert m.any()
        dmax = float(np.abs(so[s][m] - rso[s][m]).max())
        assert dmax <= TOL_STAGE, f"stage {s}: max|d| {dmax}"
        if s == 3:
            assert dmax <= S3_FEAT_BUDGET
    for l in range(8):
        dmax = float(np.abs(eng.hidden(l) - ref.hidden(l)).max())
        assert dmax <= TOL_STAGE, f"hidden {l}: max|d| {dmax}"
    rp = ref.predictions()
    np.testing.assert_allclose(eng.preds_dec(), rp, rtol=1e-4, atol=TOL_STAGE)
    # and exactly the C restatement
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    of, oso = orc.run_events(ev)
    np.testing.assert_array_equal(flags, of)
    for s in range(4):
        m = (of & _stage_bit(s)) != 0
        np.testing.assert_array_equal(so[s][m], oso[s][m], err_msg=f"stage {s}")
    for l in range(8):
        np.testing.assert_array_equal(eng.hidden(l), orc.hidden(l), err_msg=f"hidden {l}")
    np.testing.assert_array_equal(eng.preds_dec(), orc.preds_dec())
    eng.close()


def test_config2_full_size_exact(oracle_mod, stub_dir):
    """1,000,000 clustered events in one stream: hot s3 blocks and tile lists
    long enough for the per-cell scan items, compared exactly."""
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(2)
    assert len(ev) == 1_000_000
    eng = _run_engine(d, ev)
    n = len(ev)
    flags = eng.flags(n)
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    of, oso = orc.run_events(ev)
    np.testing.assert_array_equal(flags, of)
    for s in range(4):
        m = (of & _stage_bit(s)) != 0
        np.testing.assert_array_equal(eng.stage_out(s, n)[m], oso[s][m], err_msg=f"stage {s}")
    for l in range(8):
        np.testing.assert_array_equal(eng.hidden(l), orc.hidden(l), err_msg=f"hidden {l}")
    for g in range(4):
        np.testing.assert_array_equal(eng.counters(g), orc.counters(g), err_msg=f"counter {g}")
    np.testing.assert_array_equal(eng.last_t(), orc.last_t())
    np.testing.assert_array_equal(eng.preds_dec(), orc.preds_dec())
    np.testing.assert_array_equal(eng.preds_raw(), orc.preds_raw())
    np.testing.assert_array_equal(eng.version(), orc.version())
    eng.close()
