"""drain_n contract (k_ssla_s2s3_celled_drain_n_multi, ssla_s2_s3_head_celled.cuh
:1108-1255) on the reference's own buffer layouts: weights in the reference
GPU layout, caller-owned hidden state (random initial values, as the P1
harness uses) and tdrop counters, per-block rings and output slots.  Compared
exactly with the oracle's stage-2 record path."""
import ctypes as C

import numpy as np
import pytest

from ssla_rt_b200 import abi, stub

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def build_cfg(O, tensors, H2, W2, window, P, strips, rng):
    """Device buffers + HybridS2S3Config exactly as orin/orin/hybrid_common.py
    lays them out (weights transposed to (IN, OUT))."""
    orc = O.Oracle(tensors, H2 * 4, W2 * 4, window, O.LAYOUT_HYBRID)
    keep = []
    cfg = abi.HybridS2S3Config()
    cfg.H2, cfg.W2, cfg.H3, cfg.W3 = H2, W2, H2 // 2, W2 // 2
    cfg.tdrop_window, cfg.head_out_dim, cfg.n_blocks = window, 7, P
    m = orc.lib   # weights as the oracle reshaped them, read back through its structs
    import oracle as OM
    layers = []
    for li, l in enumerate(range(4, 8)):
        L = C.cast(orc.model, C.POINTER(_OrModel)).contents.L[l]
        IN, OUT, A = L.in_dim, L.out_dim, L.A
        qvg = np.ctypeslib.as_array(L.qvg, shape=(A * 3 * OUT * IN,)).reshape(A, 3 * OUT, IN)
        gow = np.ctypeslib.as_array(L.goW, shape=(A * OUT * OUT,)).reshape(A, OUT, OUT)
        qvgT = torch.from_numpy(np.ascontiguousarray(qvg.transpose(0, 2, 1))).cuda()
        goWT = torch.from_numpy(np.ascontiguousarray(gow.transpose(0, 2, 1))).cuda()
        ip = None
        if L.ip:
            ipa = np.ctypeslib.as_array(L.ip, shape=(OUT * IN,)).reshape(OUT, IN)
            ip = torch.from_numpy(np.ascontiguousarray(ipa.T)).cuda()
        gam = torch.from_numpy(np.ctypeslib.as_array(L.gamma, shape=(OUT,)).copy()).cuda()
        bet = torch.from_numpy(np.ctypeslib.as_array(L.beta, shape=(OUT,)).copy()).cuda()
        keep += [qvgT, goWT, gam, bet] + ([ip] if ip is not None else [])
        layers.append((qvgT, goWT, ip, gam, bet))
    hidden_init = []
    for li in range(4):
        grid = (H2 * W2) if li < 2 else (H2 // 2) * (W2 // 2)
        hidden_init.append(rng.normal(scale=0.05, size=(grid * (48 if li < 2 else 96),)).astype(np.float32))
    hid, td2, td3 = [], [], []
    for b in range(P):
        lo, hi = strips[b]
        s = cfg.strip[b]
        s.owned_lo, s.owned_hi, s.s3_owned_lo, s.s3_owned_hi = lo, hi, lo >> 1, hi >> 1
        s.owned_y_lo, s.owned_y_hi, s.s3_owned_y_lo, s.s3_owned_y_hi = 0, H2, 0, H2 // 2
        for li in range(4):
            qvgT, goWT, ip, gam, bet = layers[li]
            lw = cfg.layers[b][li]
            lw.qvgIn, lw.goW = qvgT.data_ptr(), goWT.data_ptr()
            lw.input_proj = ip.data_ptr() if ip is not None else 0
            lw.ln_gamma, lw.ln_beta = gam.data_ptr(), bet.data_ptr()
            h = torch.from_numpy(hidden_init[li].copy()).cuda()
            keep.append(h)
            hid.append(h)
            cfg.hidden[b][li] = h.data_ptr()
        t2 = torch.zeros(H2 * W2, dtype=torch.uint8, device="cuda")
        t3 = torch.zeros((H2 // 2) * (W2 // 2), dtype=torch.uint8, device="cuda")
        keep += [t2, t3]
        td2.append(t2); td3.append(t3)
        cfg.tdrop_s2[b], cfg.tdrop_s3[b] = t2.data_ptr(), t3.data_ptr()
    return cfg, keep, hidden_init, hid, td2, td3


class _OrLayer(C.Structure):
    _fields_ = [("in_dim", C.c_int), ("out_dim", C.c_int), ("A", C.c_int),
                ("qvg", C.POINTER(C.c_float)), ("goW", C.POINTER(C.c_float)),
                ("ip", C.POINTER(C.c_float)), ("gamma", C.POINTER(C.c_float)),
                ("beta", C.POINTER(C.c_float))]


class _OrModel(C.Structure):
    _fields_ = [("H", C.c_int), ("W", C.c_int), ("ncls", C.c_int), ("tdrop_window", C.c_int),
                ("L", _OrLayer * 8)]


@pytest.mark.parametrize("window", [4, 1])
def test_drain_n_multi_matches_oracle(oracle_mod, window):
    from ssla_rt_b200.engine import drain_n_multi
    O = oracle_mod
    rng = np.random.default_rng(5)
    H2, W2, P = 16, 20, 2
    strips = [(0, 10), (10, 20)]
    tensors = stub.stub_tensors(seed=4)
    cfg, keep, hinit, hid, td2, td3 = build_cfg(O, tensors, H2, W2, window, P, strips, rng)
    ns = [3000, 2200]
    recs, outs, clks, inputs = [], [], [], []
    for b in range(P):
        lo, hi = max(0, strips[b][0] - 2), min(W2, strips[b][1] + 2)   # halo 2 (multi_block.py:32)
        r = np.zeros(ns[b], dtype=abi.INPUT_DTYPE)
        r["x"] = rng.integers(lo, hi, ns[b])
        r["y"] = rng.integers(0, H2, ns[b])
        r["feat1"] = rng.normal(scale=0.5, size=(ns[b], 24))
        r["seq_done"] = np.arange(1, ns[b] + 1)
        inputs.append(r)
        rt = torch.from_numpy(r.view(np.uint8).copy()).cuda()
        ot = torch.zeros(ns[b] * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda")
        ct = torch.zeros(2 * ((ns[b] + 7) // 8), dtype=torch.int64, device="cuda")
        recs.append(rt); outs.append(ot); clks.append(ct)
    drain_n_multi(cfg, [r.data_ptr() for r in recs], ns, [o.data_ptr() for o in outs],
                  [c.data_ptr() for c in clks])
    torch.cuda.synchronize()
    for b in range(P):
        orc = O.Oracle(tensors, H2 * 4, W2 * 4, window, O.LAYOUT_HYBRID)
        for li in range(4):
            orc.set_hidden(4 + li, hinit[li])
        r = inputs[b]
        x2 = r["x"].astype(np.int32)
        owner = ((x2 >= strips[b][0]) & (x2 < strips[b][1])).astype(np.int32)
        p2, p3, s3 = orc.run_s2_records(x2, r["y"].astype(np.int32), r["feat1"], owner)
        got = outs[b].cpu().numpy().view(abi.OUTPUT_DTYPE)
        np.testing.assert_array_equal(got["pass2"], p2)
        np.testing.assert_array_equal(got["pass3"], p3)
        np.testing.assert_array_equal(got["s3_feat"], s3)
        for li in range(4):
            np.testing.assert_array_equal(hid[b * 4 + li].cpu().numpy(), orc.hidden(4 + li))
        np.testing.assert_array_equal(td2[b].cpu().numpy(), orc.counters(2))
        np.testing.assert_array_equal(td3[b].cpu().numpy(), orc.counters(3))
        c = clks[b].cpu().numpy()
        assert (c[1::2] >= c[0::2]).all() and c[0] > 0
