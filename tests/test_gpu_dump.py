"""The engine's OracleRecorder dump (ssla_engine_oracle_dump) is byte-for-byte
the dump of the C oracle's predictions at the same checkpoints, for one
partition of a multi-partition engine and for checkpoint intervals larger
than a drain's capacity."""
import numpy as np
import pytest

from ssla_rt_b200 import abi
from ssla_rt_b200 import events as E
from test_oracle_dump import oracle_snapshots, write_dump

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("every,max_events", [(1000, 4096), (3000, 2000)])
def test_engine_dump_equals_oracle(oracle_mod, stub_dir, tmp_path, every, max_events):
    from ssla_rt_b200.engine import SslaEngine
    d = stub_dir(64, 80, 1, 4)
    ev = E.config_events(0, n=12000)
    eng = SslaEngine(d, n_partitions=2, max_events=max_events, layout=abi.LAYOUT_HYBRID)
    ours = str(tmp_path / "engine.bin")
    eng.oracle_dump(ev, every, ours, partition=1)
    eng.close()
    idx, preds = oracle_snapshots(oracle_mod, d, ev, every)
    expect = str(tmp_path / "oracle.bin")
    assert write_dump(expect, idx, preds) == 0
    assert open(ours, "rb").read() == open(expect, "rb").read()
