"""Seeded synthetic DVS event streams for the BASELINE configurations.

No public dataset is named for this path, so every workload is synthetic with
the shapes, sizes and value distributions the BASELINE configs state:

  uniform:  x ~ U{0..W-1}, y ~ U{0..H-1}
  blobs:    Gaussian blobs (sigma px) whose centres move at a constant random
            velocity of 5-20 px/ms, reflected at the frame borders; an event's
            pixel is the blob centre plus N(0, sigma^2) per axis, rounded and
            clipped into the frame
  polarity: +1 / -1 with probability 0.5
  time:     Poisson process, t_us = cumsum(Exp(1 / rate)) in float32 us from 0

Events are returned as float32 (n, 4) rows ``(t, x, y, p)`` -- the layout of
the reference's ``openeva::Event`` (vendor/openeva/event.h:8-13) and of the
``events_packed`` argument of ``s01g_submit_batch``
(src/lib_stage01_to_gpu.cpp:501-508).
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np


def _reflect(pos: np.ndarray, size: float) -> np.ndarray:
    """Triangle-wave reflection of unbounded positions into [0, size-1]."""
    span = max(size - 1.0, 1e-9)
    m = np.mod(pos, 2.0 * span)
    return np.where(m > span, 2.0 * span - m, m)


def make_events(n: int, h: int, w: int, *, rate_mev: float, seed: int,
                n_blobs: int = 0, blob_frac: float = 0.0, sigma: float = 3.0,
                speed_px_per_ms: Tuple[float, float] = (5.0, 20.0)) -> np.ndarray:
    rng = np.random.default_rng(seed)
    dt = rng.exponential(1.0 / rate_mev, size=n)          # us between events
    t = np.cumsum(dt).astype(np.float32)
    x = rng.integers(0, w, size=n).astype(np.float64)
    y = rng.integers(0, h, size=n).astype(np.float64)
    if n_blobs > 0 and blob_frac > 0.0:
        cx0 = rng.uniform(0, w - 1, size=n_blobs)
        cy0 = rng.uniform(0, h - 1, size=n_blobs)
        ang = rng.uniform(0, 2 * np.pi, size=n_blobs)
        spd = rng.uniform(speed_px_per_ms[0], speed_px_per_ms[1], size=n_blobs)
        vx = spd * np.cos(ang) / 1000.0                    # px per us
        vy = spd * np.sin(ang) / 1000.0
        from_blob = rng.random(n) < blob_frac
        which = rng.integers(0, n_blobs, size=n)
        jx = rng.normal(0.0, sigma, size=n)
        jy = rng.normal(0.0, sigma, size=n)
        tb = t.astype(np.float64)
        bx = _reflect(cx0[which] + vx[which] * tb, w) + jx
        by = _reflect(cy0[which] + vy[which] * tb, h) + jy
        bx = np.clip(np.rint(bx), 0, w - 1)
        by = np.clip(np.rint(by), 0, h - 1)
        x = np.where(from_blob, bx, x)
        y = np.where(from_blob, by, y)
    p = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    ev = np.empty((n, 4), dtype=np.float32)
    ev[:, 0] = t
    ev[:, 1] = x
    ev[:, 2] = y
    ev[:, 3] = p
    return ev


# BASELINE configs (workload name -> generator arguments).
def config_events(cfg: int, *, n: int | None = None, seed: int | None = None,
                  stream: int = 0) -> np.ndarray:
    if cfg == 0:
        return make_events(50_000 if n is None else n, 64, 80, rate_mev=2.0,
                           seed=0 if seed is None else seed)
    if cfg == 1:
        return make_events(200_000 if n is None else n, 64, 80, rate_mev=2.0,
                           seed=1 if seed is None else seed)
    if cfg == 2:
        return make_events(1_000_000 if n is None else n, 64, 80, rate_mev=5.0,
                           seed=2 if seed is None else seed, n_blobs=6,
                           blob_frac=0.9, sigma=3.0)
    if cfg == 3:
        return make_events(10_000_000 if n is None else n, 256, 320, rate_mev=20.0,
                           seed=3 if seed is None else seed, n_blobs=16,
                           blob_frac=0.7, sigma=4.0)
    if cfg == 4:
        base = 4000 if seed is None else seed
        return make_events(1_000_000 if n is None else n, 64, 80, rate_mev=2.0,
                           seed=base + stream, n_blobs=4, blob_frac=0.5,
                           sigma=3.0)
    raise ValueError(f"unknown config {cfg}")


def split_partitions(ev: np.ndarray, n_parts: int) -> List[np.ndarray]:
    """Contiguous, equal slices: the ring partitions of config 1."""
    return [np.ascontiguousarray(a) for a in np.array_split(ev, n_parts)]
