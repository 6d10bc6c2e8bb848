"""ssla_rt_b200.stub reproduces the reference generator's tensors
(tools/make_ssla_stub.py) bit for bit; digests in tests/golden were made by
running the reference script (tests/golden/make_golden.py)."""
import json
import os

from ssla_rt_b200 import stub

HERE = os.path.dirname(os.path.abspath(__file__))


def test_stub_digests_match_reference():
    ref = json.load(open(os.path.join(HERE, "golden", "stub_digest.json")))
    for key, digest in ref.items():
        hw, seed = key.split("_seed")
        h, w = (int(v) for v in hw.split("x"))
        assert stub.tensors_digest(stub.stub_tensors(seed=int(seed))) == digest, key


def test_stub_schema(tmp_path):
    d = stub.write_stub(str(tmp_path), h=16, w=24, seed=3, tdrop=2)
    meta = json.load(open(os.path.join(d, "meta.json")))
    assert meta["model"] == "ssla_s_yolox_det" and meta["height"] == 16 and meta["width"] == 24
    assert meta["ssla_tdrop_window"] == 2
    t = stub.stub_tensors(seed=3)
    assert t["layers/0/W_in_cat"].shape == (2, 12)
    assert t["layers/7/W_in_cat"].shape == (96, 9 * 96)
    assert "layers/1/input_proj/weight" not in t
    assert t["layers/6/input_proj/weight"].shape == (96, 48)
    assert t["head/cls_preds/0/weight"].shape == (2, 96)
