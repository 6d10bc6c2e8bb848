#!/usr/bin/env python
"""Benchmark of the SSLA-S per-event hot path on B200 (one JSON line).

Workload: 200,000 uniform synthetic events at 80x64
(x ~ U{0..79}, y ~ U{0..63}, polarity +-1, Poisson 2 Mev/s timestamps, seed
1), split into 8 ring partitions of 25,000 events -- each an independent
event stream, as the reference's throughput harness splits its events over
independent blocks (orin/perf_celled_multi.py:179-190).  Stub weights
(tools/make_ssla_stub.py schema, seed 1, tdrop 4), production gate layout
(CPU gates at s1/s2 + GPU tdrop_s2/tdrop_s3).  A step drains all 200,000
events through s0..s3 and the head; the streams continue from step to step
(timestamps advance, state persists).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

value  = events drained / device time (CUDA events), max over ranks, L2
         flushed between steps (untimed)
e2e    = same metric through ssla_engine_drain_host_async (pinned host events
         in, flags + all predictions out every step, host<->device copies
         inside the timing; step k+1's copy-in overlaps step k's drain)
N > 1  = one rank per GPU (torchrun), each drains its own 200k-event set
         (weak scaling, no collective on the data path).
parity = BASELINE config 0 in full (50,000 events) through the engine and
         through the reference's own C++ pipeline (oracle/_ref): drop drift,
         max|d| s3_feat, per-stage and per-layer max|d| (rank 0, untimed)
strips = config 3 (10,000,000 events at 320x256) in N exact strips, one per
         GPU (strong scaling), device-timed with clocks and exchange status,
         with its own parity check of every rank's owned results against one
         sensor on the stream's first 200,000 events
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "Mev/s drained (output events) at 1/2/4/8 B200; p50/p99 emit→prediction µs"
N_EVENTS = 200_000
N_PARTS = 8
WL_CFG = 1                       # BASELINE config of the default workload
H, W = 64, 80
CHANS = (12, 24, 48, 96)
LAYER_DIMS = ((2, 12, 1), (12, 12, 9), (12, 24, 9), (24, 24, 9), (24, 48, 9), (48, 48, 9),
              (48, 96, 9), (96, 96, 9))


def workload(rank: int):
    from ssla_rt_b200 import events
    ev = events.config_events(WL_CFG, seed=WL_CFG + 1000 * rank)
    return events.split_partitions(ev, N_PARTS)


def use_config2() -> None:
    """Config 2 in place of config 1: one stream of 1,000,000 clustered
    events at 80x64 per step."""
    global N_EVENTS, N_PARTS, WL_CFG
    N_EVENTS, N_PARTS, WL_CFG = 1_000_000, 1, 2


# ---------------------------------------------------------------------------
# Algorithmic work (exact, from the drain's gate flags and event coordinates)
# ---------------------------------------------------------------------------
def patches(coords_xy: np.ndarray, s: int) -> np.ndarray:
    """In-bounds 3x3 patch positions per event at stage s."""
    x = coords_xy[:, 0].astype(np.int64) >> s
    y = coords_xy[:, 1].astype(np.int64) >> s
    ws, hs = W >> s, H >> s
    nx = 1 + (x > 0) + (x < ws - 1)
    ny = 1 + (y > 0) + (y < hs - 1)
    return nx * ny


def algorithmic_macs(ev: np.ndarray, flags: np.ndarray) -> dict:
    """MACs per layer (the per-layer work model of the path, with exact in-bounds patch counts):
    vg / q = the v,g and q rows of the fused qvg matvec, gather = the goW
    contributions, resid = input_proj; plus the head."""
    from ssla_rt_b200 import abi
    xy = ev[:, 1:3]
    valid = (flags & abi.F_VALID) != 0
    reach = [valid] + [(flags & b) != 0 for b in (abi.F_R1, abi.F_R2, abi.F_R3, abi.F_R4)]
    out = {}
    for l, (IN, OUT, A) in enumerate(LAYER_DIMS):
        s = l // 2
        ent = reach[s]
        np_ = patches(xy[ent], s) if A == 9 else np.ones(int(ent.sum()), np.int64)
        outn = reach[s + 1][ent] if l % 2 == 1 else np.ones(int(ent.sum()), bool)
        out[l] = {"vg": int(np_.sum()) * 2 * OUT * IN,
                  "q": int(np_[outn].sum()) * OUT * IN,
                  "gather": int(np_[outn].sum()) * OUT * OUT,
                  "resid": int(outn.sum()) * IN * OUT if IN != OUT else 0}
    out["head"] = int(reach[4].sum()) * (2 * 96 * 96 + 7 * 96)
    return out


def total_macs(macs: dict) -> int:
    return sum(v["vg"] + v["q"] + v["gather"] + v["resid"] for k, v in macs.items() if k != "head") + macs["head"]


def phase_flops(macs: dict, name: str) -> float:
    """Algorithmic FLOPs of one engine phase (2 per MAC).  Layers 1-3 compute
    their v and g rows inside the scan and their q rows (for events whose
    output is used) in the contribution GEMM, before the goW products;
    layers 4-7 build q, v, g in GEMM phases; k_ln of a stage's second layer
    also computes the next stage's input_proj residual; gates covers layer
    0."""
    parts = name.split("_")
    if name == "head":
        return 2.0 * macs["head"]
    if name == "gates":
        m = macs[0]
        return 2.0 * (m["vg"] + m["q"] + m["gather"] + m["resid"])
    if len(parts) < 2 or not parts[1].startswith("L"):
        return 0.0
    l = int(parts[1][1])
    m = macs[l]
    if parts[0] == "scan":
        return 2.0 * m["vg"] if l <= 3 else 0.0
    if parts[0] == "contrib":
        return 2.0 * (m["gather"] + (m["q"] if l <= 3 else 0))
    if parts[0] == "ln":
        return 2.0 * (macs[l + 1]["resid"] if (l % 2 == 1 and l < 7) else 0)
    if parts[0] == "gemm":
        return 2.0 * {"vg": m["vg"], "q": m["q"], "all": m["vg"] + m["q"]}[parts[2]]
    return 0.0


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_ready(self, timeout_s: float = 10.0) -> None:
        """Returns once nvidia-smi has written its first sample (its start-up
        can take over a second with several GPUs), or after timeout_s."""
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < timeout_s:
            try:
                if os.path.getsize(self.path) > 0:
                    return
            except OSError:
                return
            time.sleep(0.05)

    def stop(self, device_index: int) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) >= 9 and f[0].isdigit():
                rows.append(f)
        os.unlink(self.path)
        mine = [r for r in rows if int(r[0]) == device_index] or rows
        sm = [float(r[1]) for r in mine if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in mine for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(mine)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own SslaSPipeline (oracle/_ref), else the
# C restatement (oracle/), same 8 independent streams, host threads.
# ---------------------------------------------------------------------------
def host_info() -> dict:
    """CPU model and core counts of this host (the CPU baseline's yardstick)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        usable = os.cpu_count()
    return {"cpu_model": model, "host_cores": os.cpu_count(), "usable_cores": usable}


CPU_CLAIM = ("value: one host thread per independent stream (each stream is sequential, so a stream "
             "cannot use more than one thread; threads = min(streams, usable cores)); single_thread: "
             "the reference pipeline's own sequential semantics on one core, the yardstick of the "
             ">=100x target")


def cpu_baseline(parts, weights_dir: str, reps: int = 3, threads: int = 0, sample: str = "") -> dict:
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    threads = min(len(parts), threads or os.cpu_count() or 1)
    n = sum(len(p) for p in parts)
    single = None
    if os.path.exists(O.REF_SO):
        ref = O.RefPipeline(weights_dir, O.LAYOUT_HYBRID)
        best = min(ref.time_streams(parts, threads) for _ in range(reps))
        one_s = min(ref.time_streams(parts[:1], 1) for _ in range(reps))
        single = {"value": len(parts[0]) / one_s / 1e6, "unit": "Mev/s", "cores": 1,
                  "sample": f"stream 0 ({len(parts[0])} events) on one thread, best of {reps} -- the "
                            "reference pipeline's own sequential semantics"}
        kind = "reference"
    else:
        import concurrent.futures as cf
        def one(p):
            orc = O.Oracle(O.load_npz(weights_dir), H, W, 4, O.LAYOUT_HYBRID)
            orc.run_events(p, want_stage_out=False)
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(threads) as ex:
            list(ex.map(one, parts))
        best = time.perf_counter() - t0
        kind = "port"
    return {"value": n / best / 1e6, "unit": "Mev/s", "cores": threads, "kind": kind,
            "sample": (sample or f"the full step workload: {len(parts)} independent streams x "
                                 f"{len(parts[0])} events, one host thread per stream") + f", best of {reps}",
            "single_thread": single, **host_info(), "claim": CPU_CLAIM}


LAT_SAMPLES = 280_000            # ~1,100 head events at tdrop 4 (0.4 % of a uniform stream)


def measure_latency(weights_dir: str, stream_events: np.ndarray, device: int,
                    warmup: int = 500, samples: int = LAT_SAMPLES) -> dict:
    """Batch-of-1 emit -> prediction latency of a live stream, p50 / p99 in
    us, over all events and over the events that produced a prediction.

    Primary: the live loop (ssla_engine_live_latency) -- a resident cluster
    polls a pinned host ring; per event the host writes the slot, publishes
    the ring head and spins until the kernel's events_done passes the event
    (flags and the decoded prediction row are in pinned memory by then).
    Also reported: the one-launch step (ssla_engine_step + stream
    synchronize, ssla_engine_step_latency).  Both timed in the library's
    C++ host loop with steady_clock."""
    from ssla_rt_b200 import abi
    from ssla_rt_b200.engine import SslaEngine

    def pct(v, q):
        v = sorted(v)
        return v[min(len(v) - 1, max(0, int(round(q * len(v))) - 1))] if v else None

    def summary(lat, fl):
        # p50 / p99 over the events that produced a prediction (the
        # reference's latency population, docs/PROFILE.md:56-67); all_* over
        # every event
        lat = lat.tolist()
        head = [x for x, f in zip(lat, fl.tolist()) if f & abi.F_R4]
        return {"p50": pct(head, 0.50), "p99": pct(head, 0.99), "head_events": len(head),
                "all_p50": pct(lat, 0.50), "all_p99": pct(lat, 0.99), "n": len(lat)}

    ev = np.ascontiguousarray(stream_events[: warmup + samples])
    out = {}
    for mode in ("live", "step"):
        eng = SslaEngine(weights_dir, n_partitions=1, max_events=64, layout=abi.LAYOUT_HYBRID, device=device)
        if mode == "live":
            lat, fl, _ = eng.live_latency(ev)
        else:
            lat, fl = eng.step_latency(ev)
        eng.close()
        out[mode] = summary(lat[warmup:], fl[warmup:])
    res = dict(out["live"])
    res["step"] = out["step"]
    res["method"] = ("live: resident 11-CTA cluster (ssla_engine_live_*) polling a pinned raw-event ring; per "
                     "event the host publishes the ring head and spins on events_done (the reference's "
                     "persistent-kernel protocol), host steady_clock from publish to completion seen, in "
                     "the library's C++ loop; step: one 9-CTA cluster launch per event + stream synchronize; "
                     "p50/p99 over events that produced a prediction (the reference's latency population), "
                     "all_* over every event; "
                     f"a {samples:,}-event stream with config 0's distribution (uniform 80x64, Poisson "
                     "2 Mev/s), tdrop 4")
    return res


SWEEP_BLOCKS = (8, 16, 32, 64, 148)
SWEEP_RECORDS = 200_000


def consumer_sweep(weights_dir: str, device: int, reps: int = 3) -> dict:
    """BASELINE config 1's persistent-block sweep through the reference's own
    kernel ABI: 200,000 stage-2 ring records, drawn as the reference's sweep
    harness draws them (uniform stage-2 coordinates, feat1 ~ N(0, 0.5^2),
    orin/perf_celled_multi.py:176-190), split evenly over B rings, one
    288-thread block per ring (k_ssla_s2s3_celled_drain_n_multi of the
    consumer module, prebuilt sm_100a cubin; weights from the engine through
    ssla_engine_fill_s2s3_config), for B from 8 to the SM count.  A
    HybridS2S3Config names at most 16 blocks, so B > 16 runs as concurrent
    launches of <= 16 blocks on their own streams.  Records/s = records /
    device time from the first launch to the last completion (CUDA events),
    best of `reps`, L2 flushed before each rep (untimed)."""
    import ctypes as Cc
    import torch
    from ssla_rt_b200 import abi, consumer
    from ssla_rt_b200.engine import SslaEngine

    dev = torch.device("cuda", device)
    eng = SslaEngine(weights_dir, n_partitions=1, max_events=16, layout=abi.LAYOUT_HYBRID, device=device)
    H2, W2 = H >> 2, W >> 2
    H3, W3 = H2 // 2, W2 // 2
    mod = consumer.ConsumerModule(None)
    rng = np.random.default_rng(1)
    rec = np.zeros(SWEEP_RECORDS, dtype=abi.INPUT_DTYPE)
    rec["x"] = rng.integers(0, W2, SWEEP_RECORDS)
    rec["y"] = rng.integers(0, H2, SWEEP_RECORDS)
    rec["feat1"] = rng.normal(scale=0.5, size=(SWEEP_RECORDS, 24))
    rec["t"] = rng.uniform(0, 1, SWEEP_RECORDS)
    rec["seq_done"] = np.arange(1, SWEEP_RECORDS + 1)
    rec_dev = torch.from_numpy(rec.view(np.uint8).copy()).to(dev)
    out_dev = torch.zeros(SWEEP_RECORDS * abi.OUTPUT_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    cells2, cells3 = H2 * W2, H3 * W3
    points = []
    for B in SWEEP_BLOCKS:
        per = SWEEP_RECORDS // B
        n_launch = (B + 15) // 16
        hidden = torch.zeros(B * (2 * cells2 * 48 + 2 * cells3 * 96), dtype=torch.float32, device=dev)
        td2 = torch.zeros(B * cells2, dtype=torch.uint8, device=dev)
        td3 = torch.zeros(B * cells3, dtype=torch.uint8, device=dev)
        keep, launches = [], []
        for L in range(n_launch):
            b0, b1 = 16 * L, min(B, 16 * L + 16)
            cfg = abi.HybridS2S3Config()
            cfg.H2, cfg.W2, cfg.H3, cfg.W3 = H2, W2, H3, W3
            cfg.tdrop_window, cfg.n_blocks = 4, b1 - b0
            strip_w = max(1, W2 // B)
            rings, ns, outs = [], [], []
            for k, blk in enumerate(range(b0, b1)):
                eng.fill_s2s3_config(cfg, k)
                lo, hi = blk * strip_w, ((blk + 1) * strip_w if blk < B - 1 else W2)
                s = cfg.strip[k]
                s.owned_lo, s.owned_hi, s.s3_owned_lo, s.s3_owned_hi = lo, hi, lo >> 1, hi >> 1
                s.owned_y_lo, s.owned_y_hi, s.s3_owned_y_lo, s.s3_owned_y_hi = 0, H2, 0, H3
                hb = hidden[blk * (2 * cells2 * 48 + 2 * cells3 * 96):]
                offs = (0, cells2 * 48, 2 * cells2 * 48, 2 * cells2 * 48 + cells3 * 96)
                for li in range(4):
                    cfg.hidden[k][li] = hb[offs[li]:].data_ptr()
                cfg.tdrop_s2[k] = td2[blk * cells2:].data_ptr()
                cfg.tdrop_s3[k] = td3[blk * cells3:].data_ptr()
                rings.append(rec_dev[blk * per * 128:].data_ptr())
                outs.append(out_dev[blk * per * abi.OUTPUT_DTYPE.itemsize:].data_ptr())
                ns.append(per)
            cfg_dev = torch.frombuffer(bytearray(bytes(cfg)), dtype=torch.uint8).to(dev)
            rings_dev = torch.tensor(rings, dtype=torch.int64, device=dev)
            ns_dev = torch.tensor(ns, dtype=torch.int32, device=dev)
            outs_dev = torch.tensor(outs, dtype=torch.int64, device=dev)
            keep += [cfg_dev, rings_dev, ns_dev, outs_dev]
            launches.append((b1 - b0, [consumer.ptr(cfg_dev.data_ptr()), consumer.ptr(rings_dev.data_ptr()),
                                       consumer.ptr(ns_dev.data_ptr()), consumer.ptr(outs_dev.data_ptr()),
                                       consumer.ptr(0)]))
        streams = [torch.cuda.Stream(device=dev) for _ in launches]
        main = torch.cuda.current_stream(dev)
        best = None
        for _ in range(reps):
            td2.zero_()
            td3.zero_()
            flush.fill_(1.0)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(main)
            for st, (grid, args) in zip(streams, launches):
                st.wait_event(a)
                mod.launch("k_ssla_s2s3_celled_drain_n_multi", grid, args, stream=st.cuda_stream)
            for st in streams:
                main.wait_stream(st)
            b.record(main)
            b.synchronize()
            ms = a.elapsed_time(b)
            best = ms if best is None else min(best, ms)
        points.append({"blocks": B, "launches": len(launches), "records_per_ring": per, "ms": best,
                       "mrec_s": per * B / (best * 1e-3) / 1e6})
        del hidden, td2, td3, keep
    mod.close()
    eng.close()
    return {"kernel": "k_ssla_s2s3_celled_drain_n_multi (consumer module, prebuilt sm_100a; the reference's "
                      "launch shape: one 288-thread block per ring, 166,128 B dynamic shared memory)",
            "records": SWEEP_RECORDS, "unit": "M ring records/s (post-stage-1 records, the reference's kev/s unit)",
            "points": points,
            "timing": "CUDA events around concurrent launches (<= 16 blocks each), best of "
                      f"{reps}, L2 flushed before each rep"}


def head_modes(weights_dir: str, device: int, parts, reps: int = 5) -> dict:
    """The head on the CUDA cores (exact, the default) against the head's two
    1x1 convolutions on tcgen05 tensor cores (split TF32,
    ssla_engine_set_head_mode): the head phase's mean CUDA-event time over
    `reps` profiled config-1 drains in each mode, and the largest difference
    of the decoded and raw predictions on the same drains (untimed)."""
    import torch
    from ssla_rt_b200 import abi
    from ssla_rt_b200.engine import SslaEngine
    dev = torch.device("cuda", device)
    ev = np.ascontiguousarray(np.concatenate(parts))
    span = float(ev[:, 0].max()) + 1.0
    out = {}
    preds = {}
    for name, mode in (("exact", abi.HEAD_EXACT), ("tensor", abi.HEAD_TENSOR)):
        eng = SslaEngine(weights_dir, n_partitions=len(parts), max_events=len(ev), layout=abi.LAYOUT_HYBRID,
                         device=device, max_events_per_partition=max(len(p) for p in parts))
        eng.set_head_mode(mode)
        t = torch.from_numpy(ev).to(dev)
        off = eng.offsets([len(p) for p in parts])
        eng.drain(t, off)
        eng.set_profiling(True)
        ms = []
        for _ in range(reps):
            t[:, 0] += span
            eng.drain(t, off)
            ms += [m for nm, m, _ in eng.phase_times() if nm == "head"]
        eng.set_profiling(False)
        preds[name] = (eng.preds_dec_all(), np.stack([eng.preds_raw(p) for p in range(len(parts))]))
        out[f"{name}_head_ms"] = sum(ms) / len(ms)
        if mode == abi.HEAD_TENSOR:
            out["tensor_status"] = eng.head_status()
        eng.close()
    d_dec = np.abs(preds["tensor"][0] - preds["exact"][0])
    d_raw = np.abs(preds["tensor"][1] - preds["exact"][1])
    out["max_abs_diff_dec"] = float(d_dec.max())
    out["max_abs_diff_raw"] = float(d_raw.max())
    out["max_rel_diff_raw"] = float((d_raw / (np.abs(preds["exact"][1]) + 1e-3)).max())
    out["method"] = ("config-1 drains, state carried; head phase = CUDA events around k_head / k_head_tc; "
                     "predictions after the same drains in each mode")
    return out


PARITY_TOL_STAGE = 1e-3          # stated per-stage fp32 tolerance against the reference build
PARITY_S3_BUDGET = 5.0           # the reference's own P1 budget on max|d| s3_feat


def acceptance_parity(weights_dir: str, device: int) -> dict:
    """BASELINE config 0 in full -- 50,000 uniform events at 80x64, seed 0 --
    through the engine (one drain on `device`) and through the reference's
    own C++ pipeline (oracle/_ref; the C restatement when that is absent):
    drop drift (events whose gate flags differ), max|d| s3_feat over the
    events that reach the head (the reference's P1 gates,
    orin/bench_s2_s3_head_celled.py:285-332), per-stage and per-layer
    max|d|, and the decoded predictions.  Runs outside any timed region."""
    import torch
    from ssla_rt_b200 import abi, events
    from ssla_rt_b200.engine import SslaEngine
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    ev = events.config_events(0)
    n = len(ev)
    eng = SslaEngine(weights_dir, n_partitions=1, max_events=n, layout=abi.LAYOUT_HYBRID, device=device,
                     record_stage_outputs=True)
    eng.drain(torch.from_numpy(np.ascontiguousarray(ev)).to(torch.device("cuda", device)), [0, n])
    torch.cuda.synchronize(device)
    flags = eng.flags(n)
    so = [eng.stage_out(st, n) for st in range(4)]
    hid = [eng.hidden(l) for l in range(8)]
    preds = eng.preds_dec(0)
    eng.close()
    if os.path.exists(O.REF_SO):
        ref = O.RefPipeline(weights_dir, O.LAYOUT_HYBRID)
        kind = "reference build (the reference's own SslaSPipeline, oracle/_ref)"
        rpreds = lambda: ref.predictions()  # noqa: E731
    else:
        ref = O.Oracle(O.load_npz(weights_dir), H, W, 4, O.LAYOUT_HYBRID)
        kind = "C restatement (oracle/_ref absent)"
        rpreds = lambda: ref.preds_dec()  # noqa: E731
    rflags, rso = ref.run_events(ev)
    bits = [abi.F_R1, abi.F_R2, abi.F_R3, abi.F_R4]
    stage = []
    for st in range(4):
        m = (rflags & bits[st]) != 0
        stage.append(float(np.abs(so[st][m] - rso[st][m]).max()) if m.any() else 0.0)
    hidden = [float(np.abs(hid[l] - ref.hidden(l)).max()) for l in range(8)]
    dpred = float(np.abs(preds - rpreds()).max())
    drift = int((flags != rflags).sum())
    ok = drift == 0 and stage[3] <= PARITY_S3_BUDGET and max(stage + hidden + [dpred]) <= PARITY_TOL_STAGE
    return {"workload": "config0: 50,000 uniform events at 80x64 (seed 0, Poisson 2 Mev/s), one stream, "
                        "full s0..s3 + head",
            "against": kind, "drop_drift": drift, "max_abs_s3_feat": stage[3], "max_abs_stage": stage,
            "max_abs_hidden": hidden, "max_abs_preds": dpred,
            "events_reaching_stage": [int(((rflags & b) != 0).sum()) for b in bits],
            "tolerance": {"drop_drift": 0, "s3_feat": PARITY_S3_BUDGET, "stage_hidden_preds": PARITY_TOL_STAGE},
            "ok": ok}


def measured_traffic(phase: str):
    """DRAM bytes per launch of `phase` from the committed ncu summary
    (profiles/traffic.json: dram__bytes_read.sum + dram__bytes_write.sum of
    the phase's kernel on this workload), or None."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t[phase]["dram_bytes_per_launch"]
    except Exception:
        return None


def run_reference(args, rank: int, world: int) -> None:
    """The reference's own CPU pipeline on the work of all `world` ranks of
    our arm (each rank's 8 streams with that rank's seed), on rank 0, with
    one host thread per stream up to the usable cores."""
    if rank != 0:
        return
    from ssla_rt_b200 import stub
    with tempfile.TemporaryDirectory() as d:
        stub.write_stub(d, h=H, w=W, seed=1, tdrop=4)
        parts = [p for r in range(world) for p in workload(r)]
        n_events = sum(len(p) for p in parts)
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O
        hi = host_info()
        threads = max(1, min(len(parts), hi["usable_cores"] or 1))
        kind = "reference" if os.path.exists(O.REF_SO) else "port"
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            if kind == "reference":
                dt = O.RefPipeline(d, O.LAYOUT_HYBRID).time_streams(parts, threads)
            else:
                dt = cpu_baseline(parts, d, reps=1, threads=threads)["value"]
                dt = n_events / (dt * 1e6)
            if i >= args.warmup:
                times.append(dt)
        total = sum(times)
        value = n_events * args.steps / total / 1e6
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "Mev/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(),
            "cpu_baseline": {"value": value, "unit": "Mev/s", "cores": threads, "kind": kind,
                             "sample": f"the work of all {world} rank(s) of our arm: {len(parts)} independent "
                                       f"streams x {N_EVENTS // N_PARTS} events per step, one host thread per "
                                       f"stream up to the usable cores", **hi, "claim": CPU_CLAIM},
            "e2e": {"value": value, "unit": "Mev/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)


def config_dict() -> dict:
    what = ("config1: 200,000 uniform events at 80x64 in 8 ring partitions of 25,000 (independent streams)"
            if WL_CFG == 1 else
            "config2: 1,000,000 clustered events at 80x64 (6 Gaussian blobs sigma 3 moving at 5-20 px/ms, "
            "10% uniform, Poisson 5 Mev/s) in one stream")
    return {"workload": what + ", full s0..s3 + YOLOX head",
            "model": "SSLA-S stub (tools/make_ssla_stub.py schema, seed 1, tdrop 4)",
            "events_per_step": N_EVENTS, "partitions": N_PARTS, "sensor": "80x64",
            "gate_layout": "hybrid (lib_stage01_to_gpu + celled kernel)",
            "l2": "flushed between steps (256 MiB write, untimed)",
            "parallelism": "per-GPU independent partitions"}


# ---------------------------------------------------------------------------
# Config 3: 320x256 sensor, horizontal strips with a halo, one strip per GPU
# ---------------------------------------------------------------------------
STRIP_EVENTS = 10_000_000
STRIP_H, STRIP_W = 256, 320
STRIP_CHUNK = 1 << 20            # halo mode: events per drain of a rank
STRIP_GLOBAL_CHUNK = 10_000_000  # exact mode: global stream events per aligned chunk (the whole stream)
STRIP_BAND = 16                  # exact mode: band rows (2 stage-3 rows)


STRIP_PARITY_EVENTS = 200_000    # prefix of the stream checked against one sensor


def strips_measure(args, rank: int, world: int, local: int, steps: int, warmup: int,
                   min_timed_s: float = 0.0) -> dict:
    """Strong scaling of config 3: the one 10M-event stream split into `world`
    horizontal strips (ssla_rt_b200/strips.py), one per rank, drained in
    stream order.  value = the stream's events / the slowest rank's device
    time.  Needs the process group when world > 1.  Returns the measurement
    on rank 0 (None elsewhere).

    exact (default): each rank drains its own rows plus a 16-row band of each
    neighbour's rows and, after every layer, exchanges the band events' next-
    layer inputs with its neighbours (ssla_engine_strip_drain, peer memory
    over NVLink through CUDA IPC handles); owned results equal the single-
    sensor run bit for bit, which `parity` checks on the stream's first
    200,000 events (every rank against one sensor drained on its own GPU).
    Chunks are aligned on the global stream (chunk c = global events
    [c*G, (c+1)*G)), so neighbours exchange for the same events.
    halo: the reference's replication -- own rows plus a halo, no exchange,
    approximate near the edges."""
    import torch
    import torch.distributed as dist

    from ssla_rt_b200 import abi, events, strips, stub
    from ssla_rt_b200.engine import SslaEngine

    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    wdir = tempfile.mkdtemp(prefix="ssla_stub_")
    stub.write_stub(wdir, h=STRIP_H, w=STRIP_W, seed=1, tdrop=4)
    ev_all = events.config_events(3)
    span = float(ev_all[:, 0].max()) + 1.0
    exact = args.strip_mode == "exact"
    band = STRIP_BAND if exact else args.halo_rows
    parity = None
    if exact:       # outside the timed region: owned results against one sensor
        parity = strips.exact_strip_parity(wdir, ev_all[:STRIP_PARITY_EVENTS], rank, world, local,
                                           dist.all_gather_object if world > 1 else None, barrier, band)
        if world > 1:
            allp = [None] * world
            dist.all_gather_object(allp, parity)
            parity = allp
        else:
            parity = [parity]
    lo, hi = strips.strip_bounds(STRIP_H, world)[rank]
    mask = strips.route_mask(ev_all, lo, hi, STRIP_H, band)
    gidx = np.nonzero(mask)[0]
    sev = np.ascontiguousarray(ev_all[mask])
    own = strips.owned_mask(sev, lo, hi)
    del ev_all
    n = len(sev)
    G = args.strip_chunk or (STRIP_GLOBAL_CHUNK if exact else STRIP_CHUNK)
    if exact:
        cuts = np.searchsorted(gidx, np.arange(0, STRIP_EVENTS + G, G))
        chunks = [(int(cuts[c]), int(cuts[c + 1])) for c in range(len(cuts) - 1)]
        cap_ev = max(1, max(b - a for a, b in chunks))
    else:
        chunks = [(c, min(c + G, n)) for c in range(0, n, G)]
        cap_ev = G
    eng = SslaEngine(wdir, n_partitions=1, max_events=cap_ev, layout=abi.LAYOUT_HYBRID, device=local)
    if exact:
        eng.strip_init(lo, hi, band, rank > 0, rank < world - 1, max(1, cap_ev // 2))
        if world > 1:
            strips.connect_exact(eng, rank, world, dist.all_gather_object)
            dist.barrier()
    else:
        eng.set_owned(0, *strips.owned_s2(lo, hi, STRIP_W))
    ev = torch.from_numpy(sev).to(dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def one_pass():
        for c0, c1 in chunks:
            if exact:
                eng.strip_drain(ev[c0:], c1 - c0, stream=stream)
            elif c1 > c0:
                eng.drain(ev[c0:c1], [0, c1 - c0], stream=stream)

    for i in range(warmup):
        ev[:, 0] += span
        if i == warmup - 1:
            wa = torch.cuda.Event(enable_timing=True)
            wb = torch.cuda.Event(enable_timing=True)
            wa.record(stream)
        one_pass()
    if warmup > 0:
        wb.record(stream)
    torch.cuda.synchronize(dev)
    if min_timed_s > 0.0 and warmup > 0:
        # enough passes that the clock samples fall inside the timed region
        # (the same count on every rank: each pass has a barrier)
        need = int(math.ceil(min_timed_s * 1e3 / max(wa.elapsed_time(wb), 1e-3)))
        steps = int(max_over_ranks(float(min(max(steps, need), 400))))
    clocks = ClockSampler()
    clocks.start()
    clocks.wait_ready()
    time.sleep(0.2)
    launches = 0
    total_ms = 0.0
    barrier()
    torch.cuda.synchronize(dev)
    for _ in range(steps):
        ev[:, 0] += span
        flush.fill_(1.0)
        barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        one_pass()
        b.record(stream)
        b.synchronize()
        total_ms += a.elapsed_time(b)
        launches += eng.info().launches * len(chunks)
    barrier()
    clk = clocks.stop(local)
    status = eng.strip_status() if exact else 0
    my_ms = total_ms
    total_ms = max_over_ranks(total_ms)
    value = STRIP_EVENTS * steps / (total_ms * 1e-3) / 1e6

    # e2e: pinned host events copied in per chunk (halo: with flags out)
    host = torch.from_numpy(sev).pin_memory()
    host[:, 0] += span * (warmup + steps + 1)
    host_np = host.numpy()
    host_flags = torch.empty(max(1, cap_ev), dtype=torch.uint8).pin_memory().numpy()
    barrier()
    e2e_s = 0.0
    for _ in range(steps):
        host[:, 0] += span
        flush.fill_(2.0)
        torch.cuda.synchronize(dev)
        barrier()
        t0 = time.perf_counter()
        if exact:
            ev.copy_(host, non_blocking=True)
            one_pass()
        else:
            for c0, c1 in chunks:
                eng.drain_host(host_np[c0:c1], [0, c1 - c0], host_flags[: c1 - c0], stream=stream)
        preds = eng.preds_dec(0)
        e2e_s += time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s)
    e2e = STRIP_EVENTS * steps / e2e_s / 1e6
    status = status | (eng.strip_status() if exact else 0)

    routed = torch.tensor([n, int(own.sum()), status], dtype=torch.int64, device=dev)
    per_rank = [routed.clone() for _ in range(world)]
    rank_ms = torch.tensor([my_ms], dtype=torch.float64, device=dev)
    all_ms = [rank_ms.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, routed)
        dist.all_gather(all_ms, rank_ms)
    eng.close()
    del ev, flush
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    how = ("exact: per-layer exchange of band-event inputs between neighbouring strips over peer memory "
           f"(band {band} rows), owned results bit-identical to one sensor" if exact else
           f"halo replication ({band} rows), no exchange")
    out = {
        "value": value, "unit": "Mev/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": total_ms / steps, "scaling": "strong",
        "workload": f"config3: 10,000,000 events at 320x256 (70% from 16 moving Gaussian blobs sigma 4, 30% "
                    f"uniform, Poisson 20 Mev/s) in {world} horizontal strip(s), one per GPU, full s0..s3 + "
                    f"YOLOX head; {how}",
        "chunk_events": G, "chunking": "global stream ranges" if exact else "per-rank",
        "strip_mode": args.strip_mode, "band_rows": band,
        "bounds": strips.strip_bounds(STRIP_H, world),
        "routed_events": [int(x[0]) for x in per_rank],
        "owned_events": [int(x[1]) for x in per_rank],
        "exchange_status": [int(x[2]) for x in per_rank],
        "rank_ms": [float(x.item()) / steps for x in all_ms],
        "clocks": clk,
        "e2e": {"value": e2e, "unit": "Mev/s", "h2d_bytes_per_step": int(sev.nbytes),
                "d2h_bytes_per_step": int(preds.nbytes + (0 if exact else n))},
        "gpu_launches": launches,
        "timing": "device time (CUDA events) of each pass over the whole stream, max over ranks; L2 flushed "
                  "between passes (256 MiB write, untimed); inputs 160 MB > L2",
    }
    if parity is not None:
        out["parity"] = {
            "ok": all(p["ok"] for p in parity),
            "against": "one sensor drained by the same engine on each rank's GPU (itself bit-identical to the "
                       "C oracle); every rank compares its owned flags, hidden rows of every layer, counters, "
                       "predictions and versions",
            "events": STRIP_PARITY_EVENTS, "per_rank": parity}
    return out


def run_strips(args, rank: int, world: int, local: int) -> int:
    """`--workload strips`: config 3 as the line's own metric."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    m = strips_measure(args, rank, world, local, args.steps, args.warmup)
    if rank == 0:
        line = {
            "metric": METRIC, "value": m["value"], "unit": "Mev/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": m["workload"],
                       "model": "SSLA-S stub (320x256, seed 1, tdrop 4)", "events_per_step": STRIP_EVENTS,
                       "chunk_events": m["chunk_events"], "chunking": m["chunking"],
                       "strip_mode": m["strip_mode"], "band_rows": m["band_rows"],
                       "l2": "flushed between steps (256 MiB write, untimed); inputs 160 MB > L2",
                       "parallelism": f"strips{world}"},
            "strips": {k: m[k] for k in ("bounds", "routed_events", "owned_events", "exchange_status",
                                         "rank_ms")},
            "clocks": m["clocks"], "e2e": m["e2e"], "gpu_launches": m["gpu_launches"],
        }
        if "parity" in m:
            line["parity"] = m["parity"]
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# Config 4: 64 independent 80x64 camera streams, each through its own pinned
# ring; stream s on rank s % N
# ---------------------------------------------------------------------------
N_STREAMS = 64
STREAM_EVENTS = 1_000_000
STREAM_RING = 1 << 16            # ring slots per stream
STREAM_DRAIN = 1 << 18           # events per drain of a rank, split evenly over its rings
STREAM_CPU_SAMPLE = 20_000       # events per stream in the CPU baseline
STREAM_LOG = 100_000             # drains logged per serve


def _pct(a: np.ndarray, q: float):
    return float(np.percentile(a, q)) if len(a) else None


def run_streams(args, rank: int, world: int, local: int) -> int:
    """Config 4.  Each rank serves its streams (s = rank, rank + N, ...), one
    ring and one engine partition per stream.

    value   = device-resident drains of STREAM_DRAIN events (STREAM_DRAIN / P
              from each of the rank's P streams, consecutive slices of the
              streams), CUDA-event time, max over ranks, L2 flushed between.
    e2e     = the whole job through the rings: the replay producer publishes
              every stream's 1,000,000 events as fast as ring space allows,
              ssla_engine_serve_rings drains them (ring slots read from
              pinned host memory, flags and head-event rows written back) --
              all streams' events / the slowest rank's wall time.
    latency = the same job replayed in real time (2 Mev/s per stream, every
              event published at its timestamp): emit (the event's due time)
              to the host seeing its drain complete, p50 / p99 over all
              events and over head events."""
    import torch
    import torch.distributed as dist
    import concurrent.futures as cf
    from datetime import timedelta

    from ssla_rt_b200 import abi, stub
    from ssla_rt_b200 import events as ev_gen
    from ssla_rt_b200.engine import SslaEngine, measure_fp32_peak
    from ssla_rt_b200.rings import Replay, RingSet

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    wdir = tempfile.mkdtemp(prefix="ssla_stub_")
    stub.write_stub(wdir, h=H, w=W, seed=1, tdrop=4)
    mine = list(range(rank, N_STREAMS, world))
    P = len(mine)
    per_ring = STREAM_DRAIN // P
    with cf.ThreadPoolExecutor(min(8, os.cpu_count() or 1)) as ex:
        streams = list(ex.map(lambda s: ev_gen.config_events(4, stream=s), mine))
    eng = SslaEngine(wdir, n_partitions=P, max_events=per_ring * P, layout=abi.LAYOUT_HYBRID,
                     device=local, max_events_per_partition=per_ring)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce(vals, op):
        if world == 1:
            return list(vals)
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return [float(x) for x in t.tolist()]

    # ---- (1) device-resident drains ----
    dev_all = torch.from_numpy(np.stack(streams)).to(dev)            # [P, 1M, 4]
    n_slices = STREAM_EVENTS // per_ring
    span = float(max(s[:, 0].max() for s in streams)) + 1.0
    off = eng.offsets([per_ring] * P)

    def batch(b: int):
        i0 = (b % n_slices) * per_ring
        x = dev_all[:, i0:i0 + per_ring].reshape(-1, 4).clone()
        x[:, 0] += span * (b // n_slices)
        return x

    for b in range(args.warmup):
        eng.drain(batch(b), off, stream=stream)
    torch.cuda.synchronize(dev)
    flags_dev = torch.zeros(per_ring * P, dtype=torch.uint8, device=dev)

    def run_steps(b0: int, profile: bool):
        eng.set_profiling(profile)
        ph, fl, ms_l = {}, {}, []
        for k in range(args.steps):
            x = batch(b0 + k)
            flush.fill_(float(k))
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            eng.drain(x, off, flags=flags_dev, stream=stream)
            b.record(stream)
            b.synchronize()
            ms_l.append(a.elapsed_time(b))
            if profile:
                macs = algorithmic_macs(x.cpu().numpy(), flags_dev.cpu().numpy())
                for name, ms, nl in eng.phase_times():
                    acc = ph.setdefault(name, [0.0, 0])
                    acc[0] += ms
                    acc[1] += 1
                    fl[name] = fl.get(name, 0.0) + phase_flops(macs, name)
        eng.set_profiling(False)
        return ph, fl, ms_l

    clocks = ClockSampler()
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    _, _, step_ms = run_steps(args.warmup, False)          # timed: no per-phase events
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop(local)
    launches = eng.info().launches * args.steps
    # the next K slices with an event after every phase: phase times and the
    # dominant kernel's duration for the roofline
    phase_acc, flops_acc, prof_ms = run_steps(args.warmup + args.steps, True)
    my_ms = sum(step_ms)
    total_ms = reduce([my_ms], dist.ReduceOp.MAX if world > 1 else None)[0]
    step_events = reduce([per_ring * P * args.steps], dist.ReduceOp.SUM if world > 1 else None)[0]
    value = step_events / (total_ms * 1e-3) / 1e6
    head_frac = float((flags_dev.cpu().numpy() & abi.F_R4).astype(bool).mean())
    del dev_all
    fp32_peak = measure_fp32_peak(local)
    dom_name, (dom_ms_sum, dom_n) = max(phase_acc.items(), key=lambda kv: kv[1][0])
    achieved = flops_acc[dom_name] / (dom_ms_sum * 1e-3) / 1e12 if flops_acc.get(dom_name) else None
    roofline = {
        "kernel": dom_name, "bound": "fp32", "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s",
        "frac": (achieved / fp32_peak) if (achieved and fp32_peak) else None,
        "traffic": None,
        "peak_source": "measured FFMA peak (ssla_measure_fp32_peak, this run)",
        "avg_ms": dom_ms_sum / dom_n, "algorithmic_flops_per_launch": flops_acc.get(dom_name, 0.0) / dom_n,
        "share_of_step": dom_ms_sum / sum(prof_ms),
        "timing": "phase durations from a profiled pass over the next K slices (CUDA events after every "
                  "phase); the headline value is timed without them",
    }

    # ---- (2) e2e: the whole job through the rings, as fast as they drain ----
    rings = RingSet(P, STREAM_RING, cols=5 + eng.ncls)
    total_events = P * STREAM_EVENTS

    def serve(time_scale: float, hist=None):
        eng.reset(stream)
        torch.cuda.synchronize(dev)
        eng.rings_attach(rings)
        barrier()
        rp = Replay(rings, streams, time_scale=time_scale)
        try:
            out = eng.serve_rings(per_ring, total_events, idle_timeout_ms=10_000, log_cap=STREAM_LOG,
                                  flags_hist=hist)
        finally:
            rp.stop()
            st = rp.join()
        if out["served"] != total_events or st["published"] != total_events or out["drains"] > STREAM_LOG:
            raise RuntimeError(f"rank {rank}: served {out['served']} / published {st['published']} "
                               f"of {total_events} in {out['drains']} drains")
        return out, st

    out, st = serve(0.0)
    wall_s = (int(out["done_ns"][-1]) - st["start_ns"]) * 1e-9
    e2e_s = reduce([wall_s], dist.ReduceOp.MAX if world > 1 else None)[0]
    all_events = reduce([total_events], dist.ReduceOp.SUM if world > 1 else None)[0]
    e2e = all_events / e2e_s / 1e6
    drains = out["drains"]
    per_drain = total_events / drains

    # ---- (3) real-time replay: emit -> prediction latency ----
    hist = [np.zeros(STREAM_EVENTS, np.uint8) for _ in range(P)]
    out, st = serve(1.0, hist)
    cum = np.cumsum(out["taken"], axis=0)
    lat_all, lat_head = [], []
    for r, ev in enumerate(streams):
        k = np.searchsorted(cum[:, r], np.arange(len(ev)), side="right")
        lat = (out["done_ns"][k].astype(np.float64) - (st["start_ns"] + ev[:, 0].astype(np.float64) * 1000.0)) / 1e3
        lat_all.append(lat)
        lat_head.append(lat[(hist[r] & abi.F_R4) != 0])
    lat_all = np.concatenate(lat_all)
    lat_head = np.concatenate(lat_head)
    paced_s = (int(out["done_ns"][-1]) - st["start_ns"]) * 1e-9
    lat_vals = reduce([_pct(lat_all, 50), _pct(lat_all, 99), _pct(lat_head, 50), _pct(lat_head, 99),
                       st["max_lag_ns"] / 1e3, paced_s], dist.ReduceOp.MAX if world > 1 else None)
    latency = {"p50": lat_vals[0], "p99": lat_vals[1], "head_p50": lat_vals[2], "head_p99": lat_vals[3],
               "n": int(len(lat_all)) * world, "head_events": int(len(lat_head)),
               "producer_max_lag_us": lat_vals[4], "paced_wall_s": lat_vals[5],
               "paced_mev_s": all_events / lat_vals[5] / 1e6, "drains": out["drains"],
               "method": "real-time replay (ssla_replay_*: each event published at its timestamp, 2 Mev/s per "
                         "stream) into pinned rings served by ssla_engine_serve_rings; latency = host "
                         "CLOCK_MONOTONIC when the drain holding the event is seen complete (its flags and "
                         "prediction rows written back to the ring) minus the event's due time; max over ranks"}

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            sample = [ev_gen.config_events(4, stream=s, n=STREAM_CPU_SAMPLE) for s in range(N_STREAMS)]
            cpu = cpu_baseline(sample, wdir, reps=1, threads=os.cpu_count() or 1,
                               sample=f"the first {STREAM_CPU_SAMPLE:,} events of each of the {N_STREAMS} "
                                      "streams, independent pipelines over all host threads")
        line = {
            "metric": METRIC, "value": value, "unit": "Mev/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"config4: {N_STREAMS} independent 80x64 streams x {STREAM_EVENTS:,} events "
                                   "(50% uniform / 50% 4 moving blobs sigma 3, Poisson 2 Mev/s each), stream s on "
                                   "GPU s % N, each through its own pinned ring; full s0..s3 + YOLOX head",
                       "model": "SSLA-S stub (tools/make_ssla_stub.py schema, seed 1, tdrop 4)",
                       "streams_per_gpu": P, "events_per_step": per_ring * P,
                       "step": f"one drain of {per_ring} events from each of the GPU's {P} streams",
                       "ring_slots": STREAM_RING,
                       "l2": "flushed between steps (256 MiB write, untimed)",
                       "parallelism": f"streams over {world} GPU(s), no collective on the data path"},
            "clocks": clk,
            "e2e": {"value": e2e, "unit": "Mev/s", "h2d_bytes_per_step": int(16 * per_drain),
                    "d2h_bytes_per_step": int(per_drain * (1 + head_frac * 4 * (5 + eng.ncls))),
                    "events": int(all_events), "wall_s": e2e_s, "drains_per_gpu": drains,
                    "method": "replay producer at full speed into pinned rings, ssla_engine_serve_rings until "
                              "every stream is drained; slowest rank's wall time"},
            "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu,
            "latency_us": latency,
            "phase_ms": {k: round(v[0] / v[1], 4) for k, v in sorted(phase_acc.items(), key=lambda kv: -kv[1][0])},
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-latency", action="store_true", help="skip the batch-of-1 latency samples")
    ap.add_argument("--no-parity", action="store_true", help="skip the config-0 parity check against the reference")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip config 1's persistent-block sweep through the reference kernel ABI")
    ap.add_argument("--no-strips", action="store_true",
                    help="skip the config-3 strips measurement carried by the default line")
    ap.add_argument("--workload", default="config1", choices=["config1", "config2", "strips", "streams"],
                    help="config1: 80x64 partitions per GPU (weak scaling); config2: one clustered "
                         "80x64 stream of 1 M events per GPU (hot cells); strips: config 3, one "
                         "320x256 stream in horizontal strips across the GPUs (strong scaling); "
                         "streams: config 4, 64 camera streams through pinned rings spread over the GPUs")
    ap.add_argument("--strip-mode", default="exact", choices=["exact", "halo"],
                    help="strips: exact per-layer band exchange (default) or halo replication")
    ap.add_argument("--halo-rows", type=int, default=16, help="strips, halo mode: halo in stage-0 rows (multiple of 8)")
    ap.add_argument("--strip-chunk", type=int, default=0,
                    help="strips: events per chunk (exact: global stream events; halo: routed events per rank); "
                         "0 = the mode's default")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "config2":
        use_config2()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return 0
    if args.workload == "strips":
        return run_strips(args, rank, world, local)
    if args.workload == "streams":
        return run_streams(args, rank, world, local)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from ssla_rt_b200 import abi, stub
    from ssla_rt_b200.engine import SslaEngine, measure_fp32_peak

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)
    wdir = tempfile.mkdtemp(prefix="ssla_stub_")
    stub.write_stub(wdir, h=H, w=W, seed=1, tdrop=4)
    parts = workload(rank)
    ev_np = np.ascontiguousarray(np.concatenate(parts))
    counts = [len(p) for p in parts]
    eng = SslaEngine(wdir, n_partitions=N_PARTS, max_events=N_EVENTS, layout=abi.LAYOUT_HYBRID,
                     device=local, max_events_per_partition=max(counts))
    off = eng.offsets(counts)
    ev = torch.from_numpy(ev_np).to(dev)
    span = float(ev_np[:, 0].max()) + 1.0
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)   # 256 MiB
    stream = torch.cuda.current_stream(dev)
    step_no = [0]

    def advance():
        # the streams continue: next batch of events later in time
        step_no[0] += 1
        ev[:, 0] += span

    def flush_l2():
        flush.fill_(float(step_no[0]))

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- warm-up ----
    for _ in range(args.warmup):
        advance()
        eng.drain(ev, off, stream=stream)
    torch.cuda.synchronize(dev)

    # ---- timed: K device-timed drains (no per-phase events: they cost ~5%) ----
    def run_steps(profile: bool):
        eng.set_profiling(profile)
        acc_ph, ms_l = {}, []
        for _ in range(args.steps):
            advance()
            flush_l2()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            eng.drain(ev, off, stream=stream)
            b.record(stream)
            b.synchronize()
            ms_l.append(a.elapsed_time(b))
            for name, ms, nl in (eng.phase_times() if profile else []):
                acc = acc_ph.setdefault(name, [0.0, 0, 0])
                acc[0] += ms
                acc[1] += 1
                acc[2] += nl
        eng.set_profiling(False)
        return acc_ph, ms_l

    clocks = ClockSampler()
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    _, step_ms = run_steps(False)
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop(local)
    launches = eng.info().launches * args.steps
    # the same K drains again with an event after every phase: phase times
    # and the dominant kernel's duration for the roofline
    phase_acc, prof_ms = run_steps(True)
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = world * N_EVENTS * args.steps / (total_ms * 1e-3) / 1e6

    # ---- e2e through the host C-ABI path: pinned host events in, flags and
    # every partition's predictions out, each step; the pipelined host drain
    # copies step k+1's events on the engine's copy stream while step k runs
    base = ev.cpu()                         # continue from the device stream's timestamps
    staged = []
    for i in range(args.warmup + args.steps):
        x = base.clone()
        x[:, 0] += span * (i + 1)
        staged.append(x.pin_memory())
    host_flags = [torch.empty(N_EVENTS, dtype=torch.uint8).pin_memory() for _ in range(2)]
    pshape = tuple(eng.preds_dec_all().shape)
    host_preds = [torch.empty(pshape, dtype=torch.float32).pin_memory() for _ in range(2)]
    for i in range(args.warmup):
        eng.drain_host_async(staged[i], off, host_flags[i % 2], host_preds[i % 2], stream=stream)
    torch.cuda.synchronize(dev)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.warmup, args.warmup + args.steps):
        eng.drain_host_async(staged[i], off, host_flags[i % 2], host_preds[i % 2], stream=stream)
    stream.synchronize()
    e2e_total = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e = world * N_EVENTS * args.steps / e2e_total / 1e6
    d2h = N_EVENTS + host_preds[0].numel() * 4
    del staged

    # ---- batch-of-1 latency: one event in, its predictions out (rank 0) ----
    from ssla_rt_b200 import events as ev_gen
    latency = None if (args.no_latency or rank != 0) else measure_latency(
        wdir, ev_gen.config_events(0, n=LAT_SAMPLES + 500), local)

    # ---- roofline of the dominant phase (live CUDA-event durations) ----
    flags_dev = torch.zeros(N_EVENTS, dtype=torch.uint8, device=dev)
    eng.drain(ev, off, flags=flags_dev, stream=stream)
    flags = flags_dev.cpu().numpy()
    macs = algorithmic_macs(ev_np, flags)
    tot_macs = total_macs(macs)
    dom = max(phase_acc.items(), key=lambda kv: kv[1][0])
    dom_name, (dom_ms_sum, dom_n, _) = dom
    dom_ms = dom_ms_sum / dom_n
    fp32_peak = measure_fp32_peak(local)
    dflops = phase_flops(macs, dom_name)
    achieved = dflops / (dom_ms * 1e-3) / 1e12 if dflops > 0 else None
    roofline = {
        "kernel": dom_name, "bound": "fp32",
        "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s",
        "frac": (achieved / fp32_peak) if (achieved and fp32_peak) else None,
        "traffic": measured_traffic(dom_name),
        "peak_source": "measured FFMA peak (ssla_measure_fp32_peak, this run); the path is FP32 "
                       "CUDA-core work, MEASURED_PEAKS.json holds only HBM and bf16 tensor peaks",
        "avg_ms": dom_ms, "algorithmic_flops_per_launch": dflops,
        "share_of_step": dom_ms_sum / sum(prof_ms),
        "timing": "phase durations from a profiled pass of the same K drains (CUDA events after every "
                  "phase); the headline value is timed without them",
    }
    phases = {k: round(v[0] / v[1], 4) for k, v in sorted(phase_acc.items(), key=lambda kv: -kv[1][0])}
    stage_events = [int(x) for x in eng.info().stage_events]
    eng.close()
    del ev, flush, flags_dev
    torch.cuda.empty_cache()

    # ---- acceptance parity: config 0 against the reference build (rank 0) ----
    parity = None if (args.no_parity or rank != 0) else acceptance_parity(wdir, local)

    # ---- the head on CUDA cores vs tensor cores (rank 0, untimed) ----
    heads = None if (args.no_parity or rank != 0) else head_modes(wdir, local, parts)

    # ---- config 1's persistent-block sweep through the reference kernel ABI (rank 0) ----
    sweep = None if (args.no_sweep or rank != 0) else consumer_sweep(wdir, local)

    # ---- config 3 in N strips (the north star's strong-scaling target) ----
    strips_line = None
    if not args.no_strips:
        strips_line = strips_measure(args, rank, world, local, max(2, min(args.steps, 5)), 3, min_timed_s=0.6)

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline(parts, wdir)
        line = {
            "metric": METRIC, "value": value, "unit": "Mev/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_dict(), "clocks": clk,
            "e2e": {"value": e2e, "unit": "Mev/s", "h2d_bytes_per_step": int(ev_np.nbytes),
                    "d2h_bytes_per_step": int(d2h),
                    "method": "ssla_engine_drain_host_async per step: pinned host events copied in on the "
                              "engine's copy stream (overlapping the previous step), flags and all decoded "
                              "predictions written back into pinned host buffers by a kernel chained to the drain; "
                              "host wall time of the K steps, max over ranks"},
            "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu,
            "latency_us": latency,
            "algorithmic_mac_per_event": tot_macs / N_EVENTS,
            "stage_events": stage_events,
            "phase_ms": phases,
            "parity": parity,
            "head_modes": heads,
            "sweep": sweep,
            "strips": strips_line,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
