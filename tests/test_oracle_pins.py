"""Pins the C restatement (oracle/ssla_oracle.c) to the reference.

Fixtures in tests/golden/ are outputs of the reference's own code run in the
build container (tests/golden/make_golden.py): its C++ SslaSPipeline compiled
from its sources (DECOMP and HYBRID orders, plus the drain_n stage-2 path)
and its numpy oracle orin/orin/ssla_ref.py.  Gate decisions must match bit
for bit; floating-point results within the stated tolerances (the reference
build uses -ffast-math and libmvec's vector expf, the restatement plain fp32
with explicit fmaf and a portable exp, so values agree to ~1e-5 relative).
"""
import os

import numpy as np
import pytest

from ssla_rt_b200 import events as E
from ssla_rt_b200 import stub

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")

# Same table as tests/golden/make_golden.py
PIPELINE_CASES = {
    "80x64_w4": (64, 80, 1, 4, 4000, 11, 0),
    "16x16_w1": (16, 16, 5, 1, 600, 12, 0),
    "16x24_w3": (16, 24, 6, 3, 3000, 13, 2),
}
FEAT_ATOL = 2e-3        # stage outputs are LayerNorm outputs, O(1)
PRED_RTOL = 1e-4
PRED_ATOL = 2e-3
HID_RTOL = 2e-3
HID_ATOL = 2e-3


def case_events(h, w, n, seed, blobs):
    if blobs:
        return E.make_events(n, h, w, rate_mev=2.0, seed=seed, n_blobs=blobs, blob_frac=0.6, sigma=2.0)
    return E.make_events(n, h, w, rate_mev=2.0, seed=seed)


@pytest.mark.parametrize("name", sorted(PIPELINE_CASES))
@pytest.mark.parametrize("layout", ["decomp", "hybrid"])
def test_oracle_matches_reference_pipeline(oracle_mod, name, layout):
    O = oracle_mod
    h, w, wseed, tdrop, n, eseed, blobs = PIPELINE_CASES[name]
    g = np.load(os.path.join(GOLD, f"ref_pipeline_{name}_{layout}.npz"))
    lay = O.LAYOUT_DECOMP if layout == "decomp" else O.LAYOUT_HYBRID
    orc = O.Oracle(stub.stub_tensors(seed=wseed), h, w, tdrop, lay)
    flags, so = orc.run_events(case_events(h, w, n, eseed, blobs))
    np.testing.assert_array_equal(flags, g["flags"])            # gates: bit-exact
    for s in range(4):
        idx = g[f"so{s}_idx"]
        np.testing.assert_allclose(so[s][idx], g[f"so{s}"], rtol=0, atol=FEAT_ATOL)
    np.testing.assert_allclose(orc.preds_dec(), g["preds"], rtol=PRED_RTOL, atol=PRED_ATOL)
    for l in range(8):
        hl = orc.hidden(l)
        np.testing.assert_allclose(hl[g[f"h{l}_idx"]], g[f"h{l}"], rtol=HID_RTOL, atol=HID_ATOL)
        sums = np.array([hl.astype(np.float64).sum(), np.abs(hl.astype(np.float64)).sum()])
        np.testing.assert_allclose(sums, g[f"h{l}_sum"], rtol=1e-3, atol=1e-2)


def test_oracle_matches_reference_drain_n(oracle_mod):
    O = oracle_mod
    g = np.load(os.path.join(GOLD, "ref_records.npz"))
    rng = np.random.default_rng(21)
    n = 2000
    x2 = rng.integers(0, 20, n).astype(np.int32)
    y2 = rng.integers(0, 16, n).astype(np.int32)
    f1 = rng.normal(scale=0.5, size=(n, 24)).astype(np.float32)
    owner = (x2 < 12).astype(np.int32)
    orc = O.Oracle(stub.stub_tensors(seed=3), 64, 80, 4, O.LAYOUT_HYBRID)
    p2, p3, s3 = orc.run_s2_records(x2, y2, f1, owner)
    np.testing.assert_array_equal(p2, g["pass2"])
    np.testing.assert_array_equal(p3, g["pass3"])
    np.testing.assert_allclose(s3[g["s3_idx"]], g["s3"], rtol=0, atol=FEAT_ATOL)


def test_oracle_matches_numpy_reference_step(oracle_mod):
    """orin/orin/ssla_ref.py step_ref (fp64 layer math, DECOMP gates, no head)."""
    O = oracle_mod
    g = np.load(os.path.join(GOLD, "ssla_ref_step.npz"))
    window = int(g["window"][0])
    orc = O.Oracle(stub.stub_tensors(seed=7), 16, 16, window, O.LAYOUT_DECOMP)
    ev = E.make_events(300, 16, 16, rate_mev=0.01, seed=31)
    flags, so = orc.run_events(ev)
    passed = ((flags & O.F_R3) != 0).astype(np.uint8)          # finished stage 3
    np.testing.assert_array_equal(passed, g["passed"])
    np.testing.assert_allclose(so[3][passed == 1], g["s3"], rtol=0, atol=FEAT_ATOL)


def test_oracle_matches_live_reference_build(oracle_mod, stub_dir):
    """A case not in the fixtures, against oracle/_ref when it is built."""
    O = oracle_mod
    if not os.path.exists(O.REF_SO):
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    d = stub_dir(32, 40, 9, 4)
    ev = E.make_events(5000, 32, 40, rate_mev=4.0, seed=77, n_blobs=3, blob_frac=0.5, sigma=2.0)
    ev[::97, 1] = -3.0          # out-of-bounds events are skipped by both
    ev[5::131, 2] = 32.0
    for lay in (O.LAYOUT_DECOMP, O.LAYOUT_HYBRID):
        ref = O.RefPipeline(d, lay)
        orc = O.Oracle(O.load_npz(d), 32, 40, 4, lay)
        f1, s1 = orc.run_events(ev)
        f2, s2 = ref.run_events(ev)
        np.testing.assert_array_equal(f1, f2)
        m = (f1 & O.F_R4) != 0
        np.testing.assert_allclose(s1[3][m], s2[3][m], rtol=0, atol=FEAT_ATOL)
        np.testing.assert_allclose(orc.preds_dec(), ref.predictions(), rtol=PRED_RTOL, atol=PRED_ATOL)


def test_gate_counter_wraps_mod_256(oracle_mod):
    """uint8 counters (src/ssla_kernels.cpp:916-918): window 3 does not divide
    256, so the pass pattern at one cell shifts after 256 arrivals."""
    O = oracle_mod
    orc = O.Oracle(stub.stub_tensors(seed=2), 16, 16, 3, O.LAYOUT_DECOMP)
    n = 600
    ev = np.zeros((n, 4), np.float32)
    ev[:, 0] = np.arange(n)
    ev[:, 1] = 5.0
    ev[:, 2] = 9.0
    ev[:, 3] = 1.0
    flags, _ = orc.run_events(ev, want_stage_out=False)
    r1 = (flags & O.F_R1) != 0
    pre = np.arange(n) % 256
    np.testing.assert_array_equal(r1, (pre % 3) == 0)
