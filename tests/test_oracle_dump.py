"""OracleRecorder dumps (include/oracle.h:10-19): the library's writer
produces the reference's file format, and a dump of the C oracle's
predictions written by it matches the reference's own OracleRecorder dump of
the same stream under the reference's diff_dumps (oracle_diff) tolerance.
The engine's dump (GPU) is checked against the same oracle in
test_gpu_dump.py."""
import ctypes as C
import os

import numpy as np
import pytest

from ssla_rt_b200 import events as E

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "ssla_rt_b200", "libssla_b200.so")
REF = os.path.join(REPO, "oracle", "_ref", "libssla_ref.so")


def oracle_snapshots(O, d, ev, every):
    """The C oracle run in the recorder's rhythm: predictions after events
    0, every, 2*every, ..."""
    orc = O.Oracle(O.load_npz(d), 64, 80, 4, O.LAYOUT_HYBRID)
    idx, snaps, start = [], [], 0
    while start < len(ev):
        cp = 0 if start == 0 else ((start - 1) // every + 1) * every
        end = min(len(ev), cp + 1)
        orc.run_events(ev[start:end], want_stage_out=False)
        if end == cp + 1:
            idx.append(cp)
            snaps.append(orc.preds_dec())
        start = end
    return np.array(idx, np.uint64), np.ascontiguousarray(np.stack(snaps), np.float32)


def write_dump(path, idx, preds):
    lib = C.CDLL(LIB)
    lib.ssla_write_oracle_dump.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    return lib.ssla_write_oracle_dump(os.fsencode(path), preds.shape[1], preds.shape[2], len(idx),
                                      idx.ctypes.data, preds.ctypes.data)


def read_dump(path):
    raw = open(path, "rb").read()
    magic, ver, na, co, nc = np.frombuffer(raw[:20], np.uint32)
    idx, preds, off = [], [], 20
    for _ in range(nc):
        idx.append(int(np.frombuffer(raw[off:off + 8], np.uint64)[0]))
        preds.append(np.frombuffer(raw[off + 8:off + 8 + 4 * na * co], np.float32).reshape(na, co))
        off += 8 + 4 * na * co
    assert off == len(raw)
    return int(magic), int(ver), idx, np.stack(preds) if preds else np.zeros((0, na, co), np.float32)


def test_dump_format_round_trip(oracle_mod, stub_dir, tmp_path):
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=5000)
    idx, preds = oracle_snapshots(oracle_mod, d, ev, 700)
    p = tmp_path / "o.bin"
    assert write_dump(str(p), idx, preds) == 0
    magic, ver, ridx, rpreds = read_dump(str(p))
    assert magic == 0x4F455641 and ver == 1
    assert ridx == [0, 700, 1400, 2100, 2800, 3500, 4200, 4900]
    np.testing.assert_array_equal(rpreds, preds)


@pytest.mark.skipif(not os.path.exists(REF), reason="oracle/_ref not built (make -C oracle ref)")
def test_dump_matches_reference_recorder(oracle_mod, stub_dir, tmp_path):
    d = stub_dir(64, 80, 1, 4)
    ev = np.ascontiguousarray(E.config_events(0, n=20000), np.float32)
    idx, preds = oracle_snapshots(oracle_mod, d, ev, 1000)
    ours, theirs = str(tmp_path / "ours.bin"), str(tmp_path / "ref.bin")
    assert write_dump(ours, idx, preds) == 0
    ref = C.CDLL(REF)
    ref.ref_create.restype = C.c_void_p
    ref.ref_create.argtypes = [C.c_char_p]
    ref.ref_destroy.argtypes = [C.c_void_p]
    ref.ref_oracle_dump.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_char_p]
    ref.ref_diff_dumps.argtypes = [C.c_char_p, C.c_char_p, C.c_double, C.POINTER(C.c_double),
                                   C.POINTER(C.c_int), C.POINTER(C.c_int)]
    h = ref.ref_create(os.fsencode(d))
    assert ref.ref_oracle_dump(h, 1, ev.ctypes.data, len(ev), 1000, os.fsencode(theirs)) == len(idx)
    ref.ref_destroy(h)
    mx, ncp, nmis = C.c_double(), C.c_int(), C.c_int()
    ok = ref.ref_diff_dumps(os.fsencode(theirs), os.fsencode(ours), 1e-4, C.byref(mx), C.byref(ncp), C.byref(nmis))
    assert ok == 1 and ncp.value == len(idx) == 20
    assert nmis.value == 0, mx.value          # within oracle_diff's default tolerance
    assert os.path.getsize(ours) == os.path.getsize(theirs)
