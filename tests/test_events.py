"""Synthetic workloads (ssla_rt_b200/events.py): the BASELINE configs'
shapes and distributions, seeded and reproducible, with n=0 giving an
empty stream rather than the config's default size."""
import numpy as np

from ssla_rt_b200 import events as E


def test_config_shapes_and_ranges():
    for cfg, (h, w) in ((0, (64, 80)), (1, (64, 80)), (2, (64, 80)), (3, (256, 320)), (4, (64, 80))):
        ev = E.config_events(cfg, n=5000)
        assert ev.shape == (5000, 4) and ev.dtype == np.float32
        assert (np.diff(ev[:, 0]) >= 0).all()                    # monotonic timestamps
        assert ev[:, 1].min() >= 0 and ev[:, 1].max() <= w - 1
        assert ev[:, 2].min() >= 0 and ev[:, 2].max() <= h - 1
        assert set(np.unique(ev[:, 3])) <= {-1.0, 1.0}
        np.testing.assert_array_equal(ev, E.config_events(cfg, n=5000))   # seeded


def test_empty_and_per_stream_seeds():
    assert E.config_events(4, n=0, stream=3).shape == (0, 4)
    assert E.config_events(1, n=0).shape == (0, 4)
    a, b = E.config_events(4, n=1000, stream=0), E.config_events(4, n=1000, stream=1)
    assert not np.array_equal(a, b)


def test_rate_matches_config():
    ev = E.config_events(2, n=200_000)                           # Poisson 5 Mev/s
    rate = len(ev) / float(ev[-1, 0])                            # events per us
    assert abs(rate - 5.0) < 0.1
