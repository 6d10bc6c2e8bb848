"""The B200 stage-2/3 ring consumer module (ssla_rt_b200/kernels/) under the
reference's own launch contract: the four kernels looked up by name, one
288-thread block per ring, the runners' dynamic shared memory, and the
reference's HybridS2S3Config / HybridInputRec / HybridS2S3OutputSlot /
GpuTimingSlot buffers.  Each test runs the module as the runners build it
(NVRTC with --use_fast_math, for compute_87 -- the runners' default -- and
for compute_100a) and as the prebuilt sm_100a cubin, and compares with the
C oracle exactly:

* k_ssla_s2s3_celled_drain_n_multi / _drain_n on pre-filled rings: pass2 /
  pass3 codes, s3_feat slots, hidden state of layers 4-7, tdrop counters;
* k_ssla_s2s3_celled_persistent_multi fed live by s01g (libstage01_to_gpu's
  ABI) through pinned rings with the seq_done protocol: hidden state,
  counters, raw head predictions and versions of the owned cells, timing
  slots, tail / events_done, stop flag."""
import ctypes as C
import time

import numpy as np
import pytest

from ssla_rt_b200 import abi, stub
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

IMAGES = ["nvrtc_compute_87", "nvrtc_compute_100a", "cubin"]


def _module(kind):
    from ssla_rt_b200 import consumer
    if kind == "cubin":
        return consumer.ConsumerModule(None)
    return consumer.ConsumerModule(consumer.nvrtc_compile(kind.split("_", 1)[1]))


def _dev_bytes(obj) -> "torch.Tensor":
    raw = bytes(obj)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()


def _dev_ptrs(ptrs) -> "torch.Tensor":
    return torch.tensor([int(p) for p in ptrs], dtype=torch.int64, device="cuda")


def _records(rng, n, lo, hi, H2):
    r = np.zeros(n, dtype=abi.INPUT_DTYPE)
    r["x"] = rng.integers(lo, hi, n)
    r["y"] = rng.integers(0, H2, n)
    r["feat1"] = rng.normal(scale=0.5, size=(n, 24))
    r["seq_done"] = np.arange(1, n + 1)
    return r


def _oracle_block(O, tensors, H2, W2, window, hinit, r, strip):
    orc = O.Oracle(tensors, H2 * 4, W2 * 4, window, O.LAYOUT_HYBRID)
    if hinit is not None:
        for li in range(4):
            orc.set_hidden(4 + li, hinit[li])
    x2 = r["x"].astype(np.int32)
    y2 = r["y"].astype(np.int32)
    owner = ((x2 >= strip[0]) & (x2 < strip[1]) & (y2 >= strip[2]) & (y2 < strip[3])).astype(np.int32)
    p2, p3, s3 = orc.run_s2_records(x2, y2, r["feat1"], owner)
    return orc, p2, p3, s3


@pytest.mark.parametrize("image", IMAGES)
@pytest.mark.parametrize("window", [4, 3])
def test_drain_n_multi_module_matches_oracle(oracle_mod, image, window):
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200 import consumer as K
    O = oracle_mod
    rng = np.random.default_rng(11)
    H2, W2, P = 16, 20, 3
    strips = [(0, 7), (7, 14), (14, 20)]
    tensors = stub.stub_tensors(seed=4)
    cfg, keep, hinit, hid, td2, td3 = build_cfg(O, tensors, H2, W2, window, P, strips, rng)
    ns = [2000, 1, 1700]
    inputs, recs, outs, clks = [], [], [], []
    for b in range(P):
        r = _records(rng, ns[b], max(0, strips[b][0] - 2), min(W2, strips[b][1] + 2), H2)
        inputs.append(r)
        recs.append(torch.from_numpy(r.view(np.uint8).copy()).cuda())
        outs.append(torch.full((ns[b] * abi.OUTPUT_DTYPE.itemsize,), 0x5A, dtype=torch.uint8, device="cuda"))
        clks.append(torch.zeros(2 * ((ns[b] + 7) // 8), dtype=torch.int64, device="cuda"))
    mod = _module(image)
    cfg_dev = _dev_bytes(cfg)
    rings_dev = _dev_ptrs([t.data_ptr() for t in recs])
    ns_dev = torch.tensor(ns, dtype=torch.int32, device="cuda")
    outs_dev = _dev_ptrs([t.data_ptr() for t in outs])
    clks_dev = _dev_ptrs([t.data_ptr() for t in clks])
    mod.launch("k_ssla_s2s3_celled_drain_n_multi", P,
               [K.ptr(cfg_dev.data_ptr()), K.ptr(rings_dev.data_ptr()), K.ptr(ns_dev.data_ptr()),
                K.ptr(outs_dev.data_ptr()), K.ptr(clks_dev.data_ptr())])
    torch.cuda.synchronize()
    for b in range(P):
        s = strips[b]
        orc, p2, p3, s3 = _oracle_block(O, tensors, H2, W2, window, hinit, inputs[b], (s[0], s[1], 0, H2))
        got = outs[b].cpu().numpy().view(abi.OUTPUT_DTYPE)
        np.testing.assert_array_equal(got["pass2"], p2, err_msg=f"block {b}")
        np.testing.assert_array_equal(got["pass3"], p3, err_msg=f"block {b}")
        np.testing.assert_array_equal(got["s3_feat"], s3, err_msg=f"block {b}")
        for li in range(4):
            np.testing.assert_array_equal(hid[b * 4 + li].cpu().numpy(), orc.hidden(4 + li),
                                          err_msg=f"block {b} hidden {4 + li}")
        np.testing.assert_array_equal(td2[b].cpu().numpy(), orc.counters(2))
        np.testing.assert_array_equal(td3[b].cpu().numpy(), orc.counters(3))
        c = clks[b].cpu().numpy()
        assert (c[1::2] >= c[0::2]).all() and c[0] > 0
    mod.close()
    del keep


def test_drain_n_two_rings_matches_oracle(oracle_mod):
    """k_ssla_s2s3_celled_drain_n: the two-ring form with rings, counts,
    output slots and clocks as scalar arguments; a third block of the grid
    does nothing."""
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200 import consumer as K
    O = oracle_mod
    rng = np.random.default_rng(12)
    H2, W2 = 16, 20
    strips = [(0, 10), (10, 20)]
    tensors = stub.stub_tensors(seed=4)
    cfg, keep, hinit, hid, td2, td3 = build_cfg(O, tensors, H2, W2, 4, 2, strips, rng)
    ns = [1500, 1300]
    inputs = [_records(rng, ns[b], max(0, strips[b][0] - 2), min(W2, strips[b][1] + 2), H2) for b in range(2)]
    recs = [torch.from_numpy(r.view(np.uint8).copy()).cuda() for r in inputs]
    outs = [torch.zeros(n * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda") for n in ns]
    mod = _module("nvrtc_compute_100a")
    cfg_dev = _dev_bytes(cfg)
    mod.launch("k_ssla_s2s3_celled_drain_n", 3,
               [K.ptr(cfg_dev.data_ptr()), K.ptr(recs[0].data_ptr()), K.ptr(recs[1].data_ptr()), K.i32(ns[0]),
                K.i32(ns[1]), K.ptr(outs[0].data_ptr()), K.ptr(outs[1].data_ptr()), K.ptr(0), K.ptr(0)])
    torch.cuda.synchronize()
    for b in range(2):
        s = strips[b]
        orc, p2, p3, s3 = _oracle_block(O, tensors, H2, W2, 4, hinit, inputs[b], (s[0], s[1], 0, H2))
        got = outs[b].cpu().numpy().view(abi.OUTPUT_DTYPE)
        np.testing.assert_array_equal(got["pass2"], p2)
        np.testing.assert_array_equal(got["pass3"], p3)
        np.testing.assert_array_equal(got["s3_feat"], s3)
        for li in range(4):
            np.testing.assert_array_equal(hid[b * 4 + li].cpu().numpy(), orc.hidden(4 + li))
    mod.close()
    del keep


class _OrLayer(C.Structure):
    _fields_ = [("in_dim", C.c_int), ("out_dim", C.c_int), ("A", C.c_int),
                ("qvg", C.POINTER(C.c_float)), ("goW", C.POINTER(C.c_float)),
                ("ip", C.POINTER(C.c_float)), ("gamma", C.POINTER(C.c_float)),
                ("beta", C.POINTER(C.c_float))]


class _OrModelHead(C.Structure):
    _fields_ = [("H", C.c_int), ("W", C.c_int), ("ncls", C.c_int), ("tdrop_window", C.c_int),
                ("L", _OrLayer * 8), ("c_in", C.c_int), ("c_hid", C.c_int), ("stride_h", C.c_int),
                ("stride_w", C.c_int)] + [(n, C.POINTER(C.c_float)) for n in (
                    "cls_conv_W", "cls_conv_b", "reg_conv_W", "reg_conv_b", "cls_pred_W", "cls_pred_b",
                    "reg_pred_W", "reg_pred_b", "obj_pred_W", "obj_pred_b")]


def _head_into_cfg(orc, cfg, keep):
    """The oracle's BN-folded head weights, transposed to the reference's
    (IN, OUT) row-major GPU layout, into cfg's 2-layer head pointers."""
    m = C.cast(orc.model, C.POINTER(_OrModelHead)).contents
    ncls = m.ncls

    def mat(p, out, inn):
        a = np.ctypeslib.as_array(p, shape=(out * inn,)).reshape(out, inn)
        t = torch.from_numpy(np.ascontiguousarray(a.T)).cuda()
        keep.append(t)
        return t.data_ptr()

    def vec(p, n):
        t = torch.from_numpy(np.ctypeslib.as_array(p, shape=(n,)).copy()).cuda()
        keep.append(t)
        return t.data_ptr()
    cfg.head_cls_conv_W, cfg.head_cls_conv_b = mat(m.cls_conv_W, 96, 96), vec(m.cls_conv_b, 96)
    cfg.head_reg_conv_W, cfg.head_reg_conv_b = mat(m.reg_conv_W, 96, 96), vec(m.reg_conv_b, 96)
    cfg.head_cls_pred_W, cfg.head_cls_pred_b = mat(m.cls_pred_W, ncls, 96), vec(m.cls_pred_b, ncls)
    cfg.head_reg_pred_W, cfg.head_reg_pred_b = mat(m.reg_pred_W, 4, 96), vec(m.reg_pred_b, 4)
    cfg.head_obj_pred_W, cfg.head_obj_pred_b = mat(m.obj_pred_W, 1, 96), vec(m.obj_pred_b, 1)


@pytest.mark.parametrize("image", ["nvrtc_compute_87", "cubin"])
def test_persistent_multi_fed_by_s01g(oracle_mod, stub_dir, image):
    """s01g (stages 0-1 on the GPU) publishes records into two pinned rings
    with overlapping stage-2 ranges (halo 2) while the persistent consumer
    polls them: a backlog first, then records arriving as it runs.  Every
    record is consumed in ring order; the result equals the oracle run over
    each ring's records."""
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200 import consumer as K
    from ssla_rt_b200.s01g import S01gAPI
    O = oracle_mod
    d = stub_dir(64, 80, 1, 4)
    tensors = O.load_npz(d)
    H2, W2, P = 16, 20, 2
    owned = [(0, 10), (10, 20)]
    proc = [(0, 12), (8, 20)]
    rng = np.random.default_rng(0)
    cfg, keep, _, hid, td2, td3 = build_cfg(O, tensors, H2, W2, 4, P, owned, rng)
    for h in hid:
        h.zero_()
    orc0 = O.Oracle(tensors, 64, 80, 4, O.LAYOUT_HYBRID)
    _head_into_cfg(orc0, cfg, keep)
    cols = 7
    preds, vers, timing = [], [], []
    tmask = (1 << 13) - 1
    for b in range(P):
        s = cfg.strip[b]
        cells = (s.s3_owned_hi - s.s3_owned_lo) * (s.s3_owned_y_hi - s.s3_owned_y_lo)
        preds.append(torch.zeros(cells * cols, dtype=torch.float32, device="cuda"))
        vers.append(torch.zeros(cells, dtype=torch.int32, device="cuda"))
        timing.append(torch.zeros((tmask + 1) * 40, dtype=torch.uint8, device="cuda"))
        cfg.preds[b], cfg.version[b], cfg.timing[b] = preds[b].data_ptr(), vers[b].data_ptr(), timing[b].data_ptr()
    cfg.timing_mask = tmask
    cap = 1 << 13
    rings = [torch.zeros(cap * abi.INPUT_DTYPE.itemsize, dtype=torch.uint8).pin_memory() for _ in range(P)]
    words = torch.zeros(16, dtype=torch.int64).pin_memory()       # heads [0:2], tails [4:6], done [8:10], stop 12
    base = words.data_ptr()
    api = S01gAPI()
    api.init(d)
    api.attach_multi([r.data_ptr() for r in rings], [base + 8 * b for b in range(P)], cap - 1, W2, H2,
                     [p[0] for p in proc], [p[1] for p in proc], [0] * P, [H2] * P)
    ev = E.config_events(0, n=40000)
    api.submit(ev[:24000])                     # a backlog before the consumer starts
    assert api.flush(120.0)

    mod = _module(image)
    idle_ptr, _ = mod.global_ptr("ssla_consumer_idle_ns")
    status_ptr, _ = mod.global_ptr("ssla_consumer_status")
    drv = K._drv()
    idle = np.array([20_000_000_000], dtype=np.uint64)
    zero = np.zeros(1, dtype=np.uint32)
    K._check(drv.cuMemcpyHtoD(idle_ptr, idle.ctypes.data, 8)[0], "idle bound")
    K._check(drv.cuMemcpyHtoD(status_ptr, zero.ctypes.data, 4)[0], "status")
    cfg_dev = _dev_bytes(cfg)
    rings_dev = _dev_ptrs([r.data_ptr() for r in rings])
    tails_dev = _dev_ptrs([base + 32 + 8 * b for b in range(P)])
    dones_dev = _dev_ptrs([base + 64 + 8 * b for b in range(P)])
    torch.cuda.synchronize()
    err, stream = drv.cuStreamCreate(drv.CUstream_flags.CU_STREAM_NON_BLOCKING.value)
    K._check(err, "cuStreamCreate")
    mod.launch("k_ssla_s2s3_celled_persistent_multi", P,
               [K.ptr(cfg_dev.data_ptr()), K.ptr(rings_dev.data_ptr()), K.u64(cap - 1), K.ptr(tails_dev.data_ptr()),
                K.ptr(base + 96), K.ptr(dones_dev.data_ptr()), K.u32(200)], stream=stream)
    try:
        api.submit(ev[24000:])                 # records arriving while the consumer runs
        assert api.flush(120.0)
        heads = [int(words[b]) for b in range(P)]
        t0 = time.time()
        while any(int(words[8 + b]) < heads[b] for b in range(P)) and time.time() - t0 < 60:
            time.sleep(0.005)
    finally:
        words[12] = 1                          # stop flag
        K._check(drv.cuStreamSynchronize(stream)[0], "persistent kernel")
        drv.cuStreamDestroy(stream)
    api.shutdown()
    status = np.zeros(1, dtype=np.uint32)
    K._check(drv.cuMemcpyDtoH(status.ctypes.data, status_ptr, 4)[0], "status")
    assert status[0] == 0
    for b in range(P):
        n = heads[b]
        assert n > 1000 and int(words[4 + b]) == n and int(words[8 + b]) == n
        r = rings[b].numpy().view(abi.INPUT_DTYPE)[:n]
        np.testing.assert_array_equal(r["seq_done"], np.arange(1, n + 1, dtype=np.uint64))
        orc, p2, p3, s3 = _oracle_block(O, tensors, H2, W2, 4, None, r, (owned[b][0], owned[b][1], 0, H2))
        for li in range(4):
            np.testing.assert_array_equal(hid[b * 4 + li].cpu().numpy(), orc.hidden(4 + li),
                                          err_msg=f"block {b} hidden {4 + li}")
        np.testing.assert_array_equal(td2[b].cpu().numpy(), orc.counters(2))
        np.testing.assert_array_equal(td3[b].cpu().numpy(), orc.counters(3))
        # head: records that own their cell and passed both gates, last writer per cell
        s = cfg.strip[b]
        ow = s.s3_owned_hi - s.s3_owned_lo
        want_p = np.zeros((preds[b].numel() // cols, cols), np.float32)
        want_v = np.zeros(want_p.shape[0], np.int64)
        heads_rec = np.nonzero(p3 == 1)[0]
        assert len(heads_rec) > 0
        for i in heads_rec:
            cx, cy = (int(r["x"][i]) >> 1) - s.s3_owned_lo, (int(r["y"][i]) >> 1) - s.s3_owned_y_lo
            cell = cy * ow + cx
            want_p[cell] = orc.head_raw(s3[i])
            want_v[cell] += 1
        np.testing.assert_array_equal(preds[b].cpu().numpy().reshape(-1, cols), want_p, err_msg=f"preds {b}")
        np.testing.assert_array_equal(vers[b].cpu().numpy(), want_v, err_msg=f"version {b}")
        ts = np.frombuffer(timing[b].cpu().numpy().tobytes(), dtype=np.dtype(
            [("t_pop", "<u8"), ("t_done", "<u8"), ("seq", "<u4"), ("owner", "<u4"), ("t_push", "<u8"),
             ("t_emit", "<u8")]))
        k = min(n, tmask + 1)
        last = ts[np.arange(n - k, n) & tmask]
        np.testing.assert_array_equal(last["seq"], np.arange(n - k, n, dtype=np.uint32))
        np.testing.assert_array_equal(last["owner"], (p3[n - k:] == 1).astype(np.uint32))
        assert (last["t_done"] >= last["t_pop"]).all()
        np.testing.assert_array_equal(last["t_push"], r["t_push_ns"][n - k:])
    mod.close()
    del keep


def test_engine_filled_config_matches_engine_drain_n(stub_dir):
    """ssla_engine_fill_s2s3_config puts the engine's own device weights into
    a HybridS2S3Config; the consumer module's drain_n_multi and the engine's
    ssla_s2s3_drain_n_multi (the chunk engine behind the same contract) then
    give identical slots, hidden state and counters on the same records."""
    from ssla_rt_b200 import consumer as K
    from ssla_rt_b200.engine import SslaEngine, drain_n_multi
    d = stub_dir(64, 80, 1, 4)
    eng = SslaEngine(d, n_partitions=1, max_events=16, layout=abi.LAYOUT_HYBRID)
    rng = np.random.default_rng(21)
    H2, W2, P = 16, 20, 2
    ns = [2500, 1800]
    strips = [(0, 10), (10, 20)]

    def make_cfg():
        cfg = abi.HybridS2S3Config()
        cfg.H2, cfg.W2, cfg.H3, cfg.W3 = H2, W2, H2 // 2, W2 // 2
        cfg.tdrop_window, cfg.n_blocks = 4, P
        bufs = []
        for b in range(P):
            eng.fill_s2s3_config(cfg, b)
            s = cfg.strip[b]
            s.owned_lo, s.owned_hi, s.s3_owned_lo, s.s3_owned_hi = strips[b][0], strips[b][1], strips[b][0] >> 1, strips[b][1] >> 1
            s.owned_y_lo, s.owned_y_hi, s.s3_owned_y_lo, s.s3_owned_y_hi = 0, H2, 0, H2 // 2
            for li, (cells, ch) in enumerate(((H2 * W2, 48), (H2 * W2, 48), (H2 * W2 // 4, 96), (H2 * W2 // 4, 96))):
                t = torch.zeros(cells * ch, dtype=torch.float32, device="cuda")
                bufs.append(t)
                cfg.hidden[b][li] = t.data_ptr()
            t2 = torch.zeros(H2 * W2, dtype=torch.uint8, device="cuda")
            t3 = torch.zeros(H2 * W2 // 4, dtype=torch.uint8, device="cuda")
            bufs += [t2, t3]
            cfg.tdrop_s2[b], cfg.tdrop_s3[b] = t2.data_ptr(), t3.data_ptr()
        return cfg, bufs

    cfg_a, bufs_a = make_cfg()
    cfg_b, bufs_b = make_cfg()
    assert cfg_a.layers[0][0].qvgIn != 0 and cfg_a.head_cls_conv_W != 0
    recs, outs_a, outs_b = [], [], []
    for b in range(P):
        r = _records(rng, ns[b], max(0, strips[b][0] - 2), min(W2, strips[b][1] + 2), H2)
        recs.append(torch.from_numpy(r.view(np.uint8).copy()).cuda())
        outs_a.append(torch.zeros(ns[b] * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda"))
        outs_b.append(torch.zeros(ns[b] * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda"))
    drain_n_multi(cfg_a, [r.data_ptr() for r in recs], ns, [o.data_ptr() for o in outs_a])
    mod = _module("cubin")
    cfg_dev = _dev_bytes(cfg_b)
    rings_dev = _dev_ptrs([r.data_ptr() for r in recs])
    ns_dev = torch.tensor(ns, dtype=torch.int32, device="cuda")
    outs_dev = _dev_ptrs([o.data_ptr() for o in outs_b])
    mod.launch("k_ssla_s2s3_celled_drain_n_multi", P,
               [K.ptr(cfg_dev.data_ptr()), K.ptr(rings_dev.data_ptr()), K.ptr(ns_dev.data_ptr()),
                K.ptr(outs_dev.data_ptr()), K.ptr(0)])
    torch.cuda.synchronize()
    for b in range(P):
        np.testing.assert_array_equal(outs_a[b].cpu().numpy(), outs_b[b].cpu().numpy(), err_msg=f"slots {b}")
    for ta, tb in zip(bufs_a, bufs_b):
        np.testing.assert_array_equal(ta.cpu().numpy(), tb.cpu().numpy())
    mod.close()
    eng.close()
