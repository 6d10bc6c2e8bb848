"""ssla_s2s3_gate_codes_noalloc (the allocation-free gate pass) against the
existing drain entry point ssla_s2s3_drain_n_multi: same configuration, same
rings, separate tdrop counter buffers; the pass2 / pass3 codes of every
output slot and the advanced counters must agree exactly (integer results,
tolerance zero), on two calls in a row that carry the counters forward --
on the 80x64 sensor's stage-2 grid, on the 320x256 one, and with most
records in one hot stage-3 cell (buckets longer than a radix-sort tile).
The entry point exists for callers that must not allocate, so the test
also checks that repeated calls leave the device's free memory unchanged.

Kept in a file collected last so that it also runs after every other GPU
test in the same process, besides passing on its own."""
import numpy as np
import pytest

from ssla_rt_b200 import abi, stub

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _records(rng, n, lo, hi, H2, hot=None):
    r = np.zeros(n, dtype=abi.INPUT_DTYPE)
    r["x"] = rng.integers(lo, hi, n)
    r["y"] = rng.integers(0, H2, n)
    if hot is not None:                      # most records in one stage-3 cell (2x2 stage-2 cells)
        m = rng.random(n) < 0.9
        r["x"][m] = hot[0] + rng.integers(0, 2, int(m.sum()))
        r["y"][m] = hot[1] + rng.integers(0, 2, int(m.sum()))
    r["feat1"] = rng.normal(scale=0.5, size=(n, 24))
    r["seq_done"] = np.arange(1, n + 1)
    return r


CASES = {
    "80x64": (16, 20, [(0, 10), (10, 20)], ([1800, 1300], [700, 2100]), None),
    "320x256": (64, 80, [(0, 40), (40, 80)], ([9000, 6000], [4000, 11000]), None),
    "hot_cell": (16, 20, [(0, 10), (10, 20)], ([30000, 2000], [1000, 32000]), (8, 6)),
}


@pytest.mark.parametrize("case,window", [("80x64", 4), ("80x64", 3), ("320x256", 4), ("hot_cell", 4)])
def test_gate_codes_noalloc_matches_drain(oracle_mod, case, window):
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200.engine import drain_n_multi, gate_codes_noalloc

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    H2, W2, strips, calls, hot = CASES[case]
    P = len(strips)
    rng = np.random.default_rng(17)
    tensors = stub.stub_tensors(seed=4)
    cfg, keep, _, _, td2, td3 = build_cfg(oracle_mod, tensors, H2, W2, window, P, strips, rng)
    # the allocation-free pass gets its own counter buffers (same start)
    td2_b = [torch.zeros_like(t) for t in td2]
    td3_b = [torch.zeros_like(t) for t in td3]
    cfg_b = abi.HybridS2S3Config.from_buffer_copy(cfg)
    for b in range(P):
        cfg_b.tdrop_s2[b], cfg_b.tdrop_s3[b] = td2_b[b].data_ptr(), td3_b[b].data_ptr()
    for call, ns in enumerate(calls):
        rings, outs_a, outs_b = [], [], []
        for b in range(P):
            lo, hi = max(0, strips[b][0] - 2), min(W2, strips[b][1] + 2)
            r = _records(rng, ns[b], lo, hi, H2, hot)
            rings.append(torch.from_numpy(r.view(np.uint8).copy()).cuda())
            nbytes = ns[b] * abi.OUTPUT_DTYPE.itemsize
            outs_a.append(torch.zeros(nbytes, dtype=torch.uint8, device="cuda"))
            outs_b.append(torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda"))
        drain_n_multi(cfg, [r.data_ptr() for r in rings], ns, [o.data_ptr() for o in outs_a])
        gate_codes_noalloc(cfg_b, [r.data_ptr() for r in rings], ns, [o.data_ptr() for o in outs_b])
        torch.cuda.synchronize()
        for b in range(P):
            got = outs_b[b].cpu().numpy().view(abi.OUTPUT_DTYPE)
            want = outs_a[b].cpu().numpy().view(abi.OUTPUT_DTYPE)
            np.testing.assert_array_equal(got["pass2"], want["pass2"], err_msg=f"call {call} block {b}")
            np.testing.assert_array_equal(got["pass3"], want["pass3"], err_msg=f"call {call} block {b}")
            assert (got["pass2"] == -1).any() and (got["pass2"] == 1).any()
            np.testing.assert_array_equal(td2_b[b].cpu().numpy(), td2[b].cpu().numpy())
            np.testing.assert_array_equal(td3_b[b].cpu().numpy(), td3[b].cpu().numpy())
    del keep


def test_gate_codes_noalloc_allocates_nothing(oracle_mod):
    """After one warm-up call (which loads the module and looks the scratch
    array up), further calls leave the device's free memory unchanged."""
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200.engine import gate_codes_noalloc

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rng = np.random.default_rng(5)
    cfg, keep, *_ = build_cfg(oracle_mod, stub.stub_tensors(seed=4), 16, 20, 4, 2, [(0, 10), (10, 20)], rng)
    ns = [5000, 4000]
    rings = [torch.from_numpy(_records(rng, n, 0, 20, 16).view(np.uint8).copy()).cuda() for n in ns]
    outs = [torch.zeros(n * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device="cuda") for n in ns]
    args = ([r.data_ptr() for r in rings], ns, [o.data_ptr() for o in outs])
    gate_codes_noalloc(cfg, *args)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        gate_codes_noalloc(cfg, *args)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    del keep


def test_gate_codes_noalloc_rejects_oversize(oracle_mod):
    from test_gpu_drain_n import build_cfg
    from ssla_rt_b200.engine import SslaError, gate_codes_noalloc

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rng = np.random.default_rng(3)
    cfg, keep, *_ = build_cfg(oracle_mod, stub.stub_tensors(seed=4), 16, 20, 4, 2,
                              [(0, 10), (10, 20)], rng)
    ns = [abi.NOALLOC_MAX_RECORDS, 1]
    with pytest.raises(SslaError) as ei:
        gate_codes_noalloc(cfg, [0, 0], ns, None)   # rejected before any pointer is read
    assert ei.value.code == abi.SSLA_ERR_CAPACITY
    assert "allocation-free limit" in str(ei.value)
    del keep
