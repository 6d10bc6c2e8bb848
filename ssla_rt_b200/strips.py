"""Horizontal-strip sharding of one sensor across GPUs (the large-sensor
configuration): strip bounds, event routing with a halo, and owned ranges.

Each GPU runs the whole per-event path for the events of its strip plus a
halo of rows on either side, in stream order, with no exchange between GPUs:

* strip boundaries lie on multiples of 8 stage-0 rows (one stage-3 row), so
  a stage-1/2/3 cell and its tdrop counters never straddle two strips, and
  the halo always covers whole stage-3 rows;
* the halo is 2 stage-2 rows (8 stage-0 rows), the reference's HALO
  (orin/orin/multi_block.py:32, :120-123); an event goes to every strip
  whose range extended by the halo contains it -- the routing rule of
  src/lib_stage01_to_gpu.cpp:518-534 along y;
* a strip owns its stage-2 rows [lo/4, hi/4): only events there commit
  predictions (the HybridStrip owned bounds, ssla_s2_s3_head_celled.cuh:
  1663-1670); halo events update the strip's copy of the state only.

Drop decisions are exact on every strip: an event's gates read counters of
its own stage-1/2/3 cells, all inside one stage-3 block, and every event of
a block the strip sees is routed to it.  Features near a strip edge are
approximate (events beyond the halo are missing) -- the drift the reference
accepts within its max|d| s3_feat <= 5.0 budget.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

UNIT_ROWS = 8          # stage-0 rows per stage-3 row
HALO_S2 = 2            # halo in stage-2 rows (orin/orin/multi_block.py:32)
HALO_ROWS = HALO_S2 * 4


def strip_bounds(height: int, n: int) -> List[Tuple[int, int]]:
    """n contiguous strips of stage-0 rows [lo, hi), boundaries on multiples
    of 8, sizes as equal as the 8-row units allow."""
    if height % UNIT_ROWS:
        raise ValueError("sensor height must be a multiple of 8")
    units = height // UNIT_ROWS
    if n < 1 or n > units:
        raise ValueError(f"{n} strips do not fit {units} units of 8 rows")
    cuts = [round(i * units / n) * UNIT_ROWS for i in range(n + 1)]
    return [(cuts[i], cuts[i + 1]) for i in range(n)]


def route_mask(events: np.ndarray, lo: int, hi: int, height: int, halo_rows: int = HALO_ROWS) -> np.ndarray:
    """Events (rows t, x, y, p) that strip [lo, hi) processes: y in
    [lo - halo, hi + halo) clipped to the sensor.  Stream order is kept."""
    y = events[:, 2]
    return (y >= max(0, lo - halo_rows)) & (y < min(height, hi + halo_rows))


def owned_mask(events: np.ndarray, lo: int, hi: int) -> np.ndarray:
    """Events whose pixel lies in the strip's own rows [lo, hi)."""
    y = events[:, 2]
    return (y >= lo) & (y < hi)


def owned_s2(lo: int, hi: int, width: int) -> Tuple[int, int, int, int]:
    """Owned stage-2 range (x0, x1, y0, y1) of strip [lo, hi)."""
    return 0, width >> 2, lo >> 2, hi >> 2


def shard(events: np.ndarray, height: int, n: int, halo_rows: int = HALO_ROWS):
    """Per strip: (bounds, its events in stream order, owned mask over them)."""
    out = []
    for lo, hi in strip_bounds(height, n):
        m = route_mask(events, lo, hi, height, halo_rows)
        ev = np.ascontiguousarray(events[m])
        out.append(((lo, hi), ev, owned_mask(ev, lo, hi)))
    return out
