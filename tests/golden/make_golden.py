"""Regenerates the committed golden fixtures from the reference itself.

Run in a container that has the reference checkout (default: a directory
named `reference` beside this repository, or $SSLA_REFERENCE) and the built
oracle/_ref library
(`make -C oracle ref`):

    python tests/golden/make_golden.py

Fixtures written next to this script:
  stub_digest.json      sha256 digests of the tensors written by the
                        reference's tools/make_ssla_stub.py for two
                        (h, w, seed) settings
  ref_pipeline_*.npz    per-event gate flags, stage outputs of sampled
                        events, final predictions and hidden-state samples
                        from the reference's C++ SslaSPipeline (compiled from
                        its sources into oracle/_ref) driven in the DECOMP and
                        HYBRID orders, on seeded synthetic events
  ref_records.npz       drain_n (stage-2 entry) outputs of the same build
  ssla_ref_step.npz     per-event results of the reference's numpy oracle
                        (orin/orin/ssla_ref.py step_ref) on a small grid
The reference has no stored golden vectors of its own; these are outputs of
its code run here on inputs the tests regenerate from seeds.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("SSLA_REFERENCE", os.path.join(os.path.dirname(REPO), "reference"))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle"))

from ssla_rt_b200 import events as E  # noqa: E402
from ssla_rt_b200 import stub  # noqa: E402
import oracle as O  # noqa: E402

# Cases shared with tests/test_oracle_pins.py.
PIPELINE_CASES = {
    # name: (h, w, weight seed, tdrop, event count, event seed, blobs)
    "80x64_w4": (64, 80, 1, 4, 4000, 11, 0),
    "16x16_w1": (16, 16, 5, 1, 600, 12, 0),
    "16x24_w3": (16, 24, 6, 3, 3000, 13, 2),
}
SAMPLE_HIDDEN = 64


def ref_stub(out_dir: str, h: int, w: int, seed: int, tdrop: int) -> None:
    subprocess.run([sys.executable, os.path.join(REF, "tools", "make_ssla_stub.py"), out_dir,
                    "--h", str(h), "--w", str(w), "--seed", str(seed), "--tdrop", str(tdrop)],
                   check=True, stdout=subprocess.DEVNULL)


def case_events(h, w, n, seed, blobs):
    if blobs:
        return E.make_events(n, h, w, rate_mev=2.0, seed=seed, n_blobs=blobs, blob_frac=0.6, sigma=2.0)
    return E.make_events(n, h, w, rate_mev=2.0, seed=seed)


def hidden_samples(getter, h, w, seed):
    rng = np.random.default_rng(seed)
    idx, vals = [], []
    for l in range(8):
        a = getter(l)
        i = np.sort(rng.choice(a.size, size=min(SAMPLE_HIDDEN, a.size), replace=False))
        idx.append(i)
        vals.append(a[i])
    return idx, vals


def main() -> int:
    out = {}
    digests = {}
    with tempfile.TemporaryDirectory() as tmp:
        for (h, w, seed) in ((64, 80, 1), (16, 16, 5)):
            d = os.path.join(tmp, f"s{h}x{w}_{seed}")
            ref_stub(d, h, w, seed, 4)
            digests[f"{h}x{w}_seed{seed}"] = stub.tensors_digest(O.load_npz(d))
        with open(os.path.join(HERE, "stub_digest.json"), "w") as f:
            json.dump(digests, f, indent=2)

        for name, (h, w, wseed, tdrop, n, eseed, blobs) in PIPELINE_CASES.items():
            d = os.path.join(tmp, name)
            ref_stub(d, h, w, wseed, tdrop)
            ev = case_events(h, w, n, eseed, blobs)
            for layout, lname in ((O.LAYOUT_DECOMP, "decomp"), (O.LAYOUT_HYBRID, "hybrid")):
                ref = O.RefPipeline(d, layout)
                flags, so = ref.run_events(ev)
                rec = {"flags": flags, "preds": ref.predictions()}
                for s in range(4):
                    bit = (O.F_R1 << s) if s < 3 else O.F_R4
                    sel = np.nonzero(flags & bit)[0]
                    sel = sel[:: max(1, sel.size // 40)][:40]
                    rec[f"so{s}_idx"] = sel.astype(np.int32)
                    rec[f"so{s}"] = so[s][sel]
                idx, vals = hidden_samples(ref.hidden, h, w, 99)
                for l in range(8):
                    rec[f"h{l}_idx"] = idx[l].astype(np.int32)
                    rec[f"h{l}"] = vals[l]
                    hl = ref.hidden(l)
                    rec[f"h{l}_sum"] = np.array([hl.astype(np.float64).sum(),
                                                 np.abs(hl.astype(np.float64)).sum()])
                np.savez_compressed(os.path.join(HERE, f"ref_pipeline_{name}_{lname}.npz"), **rec)
                out[f"{name}_{lname}"] = int(flags.size)

        # drain_n records at the stage-2 grid (P1 harness shape, 20x16)
        d = os.path.join(tmp, "records")
        ref_stub(d, 64, 80, 3, 4)
        rng = np.random.default_rng(21)
        n = 2000
        x2 = rng.integers(0, 20, n).astype(np.int32)
        y2 = rng.integers(0, 16, n).astype(np.int32)
        f1 = rng.normal(scale=0.5, size=(n, 24)).astype(np.float32)
        owner = (x2 < 12).astype(np.int32)
        ref = O.RefPipeline(d, O.LAYOUT_HYBRID)
        p2, p3, s3 = ref.run_s2_records(x2, y2, f1, owner)
        sel = np.arange(0, n, 25)
        np.savez_compressed(os.path.join(HERE, "ref_records.npz"), pass2=p2, pass3=p3,
                            s3_idx=sel.astype(np.int32), s3=s3[sel])

    # numpy reference (orin/orin/ssla_ref.py) on a 16x16 grid, DECOMP order
    sys.path.insert(0, os.path.join(REF, "orin"))
    from orin.ssla_ref import LayerRef, StepRefState, step_ref  # noqa: E402
    from orin.weights_ssla import reshape_ssla_layer  # noqa: E402
    t = stub.stub_tensors(seed=7)
    layers = []
    dims = [(2, 12, 1), (12, 12, 3), (12, 24, 3), (24, 24, 3), (24, 48, 3), (48, 48, 3), (48, 96, 3), (96, 96, 3)]
    H0 = W0 = 16
    for li, (i_d, o_d, k) in enumerate(dims):
        p = f"layers/{li}"
        qvg, gow = reshape_ssla_layer(t[f"{p}/W_in_cat"], t[f"{p}/W_out_cat"], t[f"{p}/q_proj/weight"],
                                      t[f"{p}/v_proj/weight"], t[f"{p}/g_proj/weight"],
                                      t[f"{p}/o_proj/weight"], i_d, o_d)
        st = li // 2
        layers.append(LayerRef(qvgIn=qvg, goW=gow, input_proj=t.get(f"{p}/input_proj/weight"),
                               ln_gamma=t[f"{p}/norm/weight"], ln_beta=t[f"{p}/norm/bias"],
                               H=np.zeros(((H0 >> st) * (W0 >> st), o_d), np.float32), K=k))
    window = 2
    state = StepRefState(H0=H0, W0=W0, tdrop_window=window, layers=layers,
                         tdrop=[np.zeros((H0 >> s) * (W0 >> s), np.uint8) for s in (1, 2, 3)])
    ev = E.make_events(300, H0, W0, rate_mev=0.01, seed=31)
    last = np.full(H0 * W0, -1.0)
    passed = np.zeros(len(ev), np.uint8)
    s3 = np.zeros((len(ev), 96), np.float32)
    for i, (tt, x, y, p) in enumerate(ev):
        xi, yi = int(x), int(y)
        prev = last[yi * W0 + xi]
        dt = 1.0 if prev < 0 else float(np.float32(min(max((float(tt) - prev) / 1e5, 0.0), 1.0)))
        last[yi * W0 + xi] = float(tt)
        ok, _, _, _, o3, _, _ = step_ref(state, xi, yi, dt, float(p))
        passed[i] = 1 if ok else 0
        if ok:
            s3[i] = o3
    np.savez_compressed(os.path.join(HERE, "ssla_ref_step.npz"), passed=passed, s3=s3[passed == 1],
                        window=np.array([window]))
    print("golden fixtures written:", out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
