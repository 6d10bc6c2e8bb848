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


# ---------------------------------------------------------------------------
# Exact strips across GPUs, checked against one sensor
# ---------------------------------------------------------------------------
CHANS = (12, 24, 48, 96)


def connect_exact(eng, rank: int, world: int, all_gather_object) -> None:
    """Connects an engine set up by strip_init to its neighbours' receive
    buffers through CUDA IPC handles, exchanged with `all_gather_object`
    (torch.distributed's, or any callable with its signature)."""
    mine = [eng.strip_recv_buffer(sd)[1] if (sd == 0 and rank > 0) or (sd == 1 and rank < world - 1)
            else None for sd in (0, 1)]
    allh = [None] * world
    all_gather_object(allh, mine)
    if rank > 0:
        eng.strip_connect(0, peer_handle=allh[rank - 1][1])
    if rank < world - 1:
        eng.strip_connect(1, peer_handle=allh[rank + 1][0])


def _rows(a: np.ndarray, height: int, width: int, s: int, lo: int, hi: int) -> np.ndarray:
    """Rows [lo >> s, hi >> s) of a per-cell array on the stage-s grid."""
    hs, ws = height >> s, width >> s
    return a.reshape(hs, ws, -1)[lo >> s:hi >> s]


def exact_strip_parity(weights_dir: str, events: np.ndarray, rank: int, world: int, device: int,
                       all_gather_object, barrier, band: int = 16) -> dict:
    """One aligned chunk of `events` (a prefix of the sensor's stream) drained
    as `world` exact strips, one per rank and GPU, with the per-layer band
    exchange over peer memory; then the same events drained as one sensor on
    this rank's GPU.  Compares this rank's owned results with the
    single-sensor run: the flags of its owned events, the hidden state of its
    rows at every layer, its gate counters, predictions and versions.
    Returns {"ok", "events", "routed", "owned", "exchange_status",
    "mismatch": {name: {"rows": first differing rows (stage-grid rows
    counted from the strip's first), "n": how many}}}; every rank must call
    it together."""
    import torch
    from . import abi
    from .engine import SslaEngine

    full = SslaEngine(weights_dir, n_partitions=1, max_events=max(1, len(events)), layout=abi.LAYOUT_HYBRID,
                      device=device)
    H, W = full.H, full.W
    lo, hi = strip_bounds(H, world)[rank]
    mask = route_mask(events, lo, hi, H, band)
    sev = np.ascontiguousarray(events[mask])
    own = owned_mask(sev, lo, hi)
    n = len(sev)
    eng = SslaEngine(weights_dir, n_partitions=1, max_events=max(1, n), layout=abi.LAYOUT_HYBRID, device=device)
    eng.strip_init(lo, hi, band, rank > 0, rank < world - 1, max(1, n // 2))
    if world > 1:
        connect_exact(eng, rank, world, all_gather_object)
    barrier()
    dev = torch.device("cuda", device)
    sflags = torch.zeros(max(1, n), dtype=torch.uint8, device=dev)
    eng.strip_drain(torch.from_numpy(sev).to(dev), n, flags=sflags)
    torch.cuda.synchronize(dev)
    status = eng.strip_status()
    ff = torch.zeros(max(1, len(events)), dtype=torch.uint8, device=dev)
    full.drain(torch.from_numpy(np.ascontiguousarray(events)).to(dev), [0, len(events)], flags=ff)
    torch.cuda.synchronize(dev)
    bad = {}

    def cmp(name, a, b):
        if not np.array_equal(a, b):
            rows = np.nonzero((a != b).reshape(a.shape[0], -1).any(axis=1))[0]
            bad[name] = {"rows": [int(r) for r in rows[:8]], "n": int(len(rows))}

    idx = np.nonzero(mask)[0]
    cmp("flags", sflags.cpu().numpy()[:n][own], ff.cpu().numpy()[idx[own]])
    for l in range(8):
        s = l // 2
        cmp(f"hidden{l}", _rows(eng.hidden(l), H, W, s, lo, hi), _rows(full.hidden(l), H, W, s, lo, hi))
    for g, s in enumerate((1, 2, 2, 3)):
        cmp(f"counter{g}", _rows(eng.counters(g), H, W, s, lo, hi), _rows(full.counters(g), H, W, s, lo, hi))
    cmp("preds", _rows(eng.preds_dec(), H, W, 3, lo, hi), _rows(full.preds_dec(), H, W, 3, lo, hi))
    cmp("version", _rows(eng.version(), H, W, 3, lo, hi), _rows(full.version(), H, W, 3, lo, hi))
    barrier()                 # no rank closes its buffers while a neighbour may still read them
    eng.close()
    full.close()
    return {"ok": not bad and status == 0, "events": int(len(events)), "routed": int(n),
            "owned": int(own.sum()), "exchange_status": int(status), "mismatch": bad}
