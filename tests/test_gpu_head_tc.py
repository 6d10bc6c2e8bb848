"""The tensor-core head (SSLA_HEAD_TENSOR: the head's two 1x1 convolutions
as one tcgen05 GEMM in three TF32 terms) against the exact head on the same
drains: gate flags, hidden state, counters and versions are identical; the
decoded and raw predictions agree within the stated tolerance of the split
TF32 GEMM against the fmaf chain (1e-4 relative + 1e-5 absolute; measured
differences are ~1e-6); the engine reports no timed-out wait.  Covers the
config-1 workload (8 partitions, several 128-row tiles, a partial tile) and
a clustered stream."""
import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

RTOL, ATOL = 1e-4, 1e-5


def _drain(d, parts, mode, n_parts):
    from ssla_rt_b200.engine import SslaEngine
    ev = np.ascontiguousarray(np.concatenate(parts))
    eng = SslaEngine(d, n_partitions=n_parts, max_events=len(ev), layout=abi.LAYOUT_HYBRID,
                     max_events_per_partition=max(len(p) for p in parts))
    eng.set_head_mode(mode)
    flags = torch.zeros(len(ev), dtype=torch.uint8, device="cuda")
    eng.drain(torch.from_numpy(ev).cuda(), eng.offsets([len(p) for p in parts]), flags=flags)
    torch.cuda.synchronize()
    return eng, flags.cpu().numpy()


@pytest.mark.parametrize("workload", ["config1", "clustered"])
def test_tensor_core_head_matches_exact_head(oracle_mod, stub_dir, workload):
    d = stub_dir(64, 80, 1, 4)
    if workload == "config1":
        parts = E.split_partitions(E.config_events(1), 8)
    else:
        parts = [E.config_events(2, n=120_000)]
    P = len(parts)
    exact, f_exact = _drain(d, parts, abi.HEAD_EXACT, P)
    tc, f_tc = _drain(d, parts, abi.HEAD_TENSOR, P)
    assert tc.head_status() == 0
    np.testing.assert_array_equal(f_tc, f_exact)
    assert int(((f_exact & abi.F_R4) != 0).sum()) > 128          # more than one tile of head events
    worst = 0.0
    for p in range(P):
        for l in range(8):
            np.testing.assert_array_equal(tc.hidden(l, p), exact.hidden(l, p))
        np.testing.assert_array_equal(tc.version(p), exact.version(p))
        for a, b in ((tc.preds_dec(p), exact.preds_dec(p)), (tc.preds_raw(p), exact.preds_raw(p))):
            np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL)
            worst = max(worst, float(np.max(np.abs(a - b) / (np.abs(b) + 1e-3))))
    # and the exact head is the oracle's, bit for bit
    orc = oracle_mod.Oracle(oracle_mod.load_npz(d), 64, 80, 4, oracle_mod.LAYOUT_HYBRID)
    orc.run_events(parts[0], want_stage_out=False)
    np.testing.assert_array_equal(exact.preds_dec(0), orc.preds_dec())
    print(f"tensor-core head: max relative difference {worst:.3g}")
    exact.close()
    tc.close()
