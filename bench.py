"""Benchmark of the correlation hot path: corr edges/s on B200.

One step = one pass of the path over one batch of the workload on a resident
keyframe graph (the reference keeps DroidState::fmaps resident and adds one
keyframe per frame, cuda_slam/main.cu:755): the frontend workloads (C1, C2,
C4) receive one new keyframe per step, packed into the store's spare slot
(dc_set_frames) on a side stream beside the step's build + 4-level pyramid +
r=3 lookup of the batch's edges (dc_build_and_lookup, the drop-in for
CudaDroid::batch_build_and_sample_correlation, cuda_slam/main.cu:1555-1613);
the backend workloads (C3, C5) run one pass over all their edges.  Default
workload: C2 (12 keyframes, 48 edges, 48x64x128, the frontend batch the metric
is quoted on), FP16 arithmetic (the reference's own: FP16 fmaps, fp32
accumulate).

  python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

--impl reference times the reference's CPU path (the C/OpenMP restatement in
oracle/, the reference having no CPU implementation of its own) on the host
cores.  Under torchrun (N>1) the keyframe graph is packed once on rank 0 and
replicated by one NCCL broadcast of the packed store (timed and reported
apart); each frontend step's new keyframe is broadcast as one packed slot on
the side stream, beside the kernel (which leaves 4 SMs free for it).  Frontend
workloads give each rank its own seeded batch (weak scaling); the backend
workloads split one edge list into contiguous ranges (strong scaling).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "corr edges/sec (48x64x128, 4-lvl r=3 lookup)"
UNIT = "edges/s"
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="C2")
    ap.add_argument("--precision", default="fp16", choices=["fp32", "tf32", "bf16", "fp16", "fp32x3"])
    ap.add_argument("--tile-order", default=None, choices=["source", "window_row", "auto"],
                    help="how the fused kernel groups source pixels into tiles "
                         "(dc_set_tile_order); default: auto for the backend workloads "
                         "(large flow), source for the frontend")
    ap.add_argument("--edges", type=int, default=0,
                    help="profiling only: keep the first N edges of a backend workload "
                         "(a small case for multi-pass ncu captures); not a bench line")
    ap.add_argument("--encoder", action="store_true",
                    help="time dc_corr_encode (corr encoder first layer) at the workload's sizes instead")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--scatter-mean", action="store_true",
                    help="time dc_scatter_mean (GraphAgg) at the workload's sizes instead")
    ap.add_argument("--project", action="store_true",
                    help="coordinates from poses + inverse depths inside the step "
                         "(dc_project_build_and_lookup: reprojection + fused correlation)")
    ap.add_argument("--materialise", action="store_true",
                    help="store the volume pyramid (dc_build_volume) and look up from it, "
                         "the reference's own data flow, instead of the fused path")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


# ---------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"dc_bench_clocks_gpu{gpu_index}_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------- CPU legs

def cpu_sample(wl, fm_np, ii, jj, coords_np, budget_s=12.0, min_edges=2, threads=0):
    """Time the oracle's fp32 C/OpenMP build+pyramid+lookup on edges of the
    workload until ~budget_s of CPU work; returns (edges/s, edges, threads)."""
    from oracle import oracle as O

    O.lib()
    n = 0
    t0 = time.perf_counter()
    while True:
        e = n % len(ii)
        O.cpu_build_and_sample(fm_np, ii[e:e + 1], jj[e:e + 1], coords_np[e:e + 1], wl.alpha,
                               threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if (el >= budget_s and n >= min_edges) or n >= len(ii) * 4:
            break
    used = threads if threads > 0 else O.max_threads()
    return n / el, n, used


def run_reference_arm(args, wl):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    from slam_hands_b200 import configs

    fm_np = configs.make_fmaps_np(wl)
    ii, jj = configs.make_edges(wl)
    coords = configs.make_coords_np(wl, len(ii))
    from oracle import oracle as O

    O.lib()
    # all host threads (torchrun sets OMP_NUM_THREADS=1 for its workers)
    threads = len(os.sched_getaffinity(0))
    per_step = 2  # edges per step: a bounded sample of the batch
    times = []
    for s in range(args.warmup + args.steps):
        e0 = (s * per_step) % len(ii)
        sl = slice(e0, e0 + per_step)
        t0 = time.perf_counter()
        O.cpu_build_and_sample(fm_np, ii[sl], jj[sl], coords[sl], wl.alpha, threads=threads)
        dt = time.perf_counter() - t0
        if s >= args.warmup:
            times.append(dt)
    tot = sum(times)
    value = per_step * len(times) / tot
    cores = threads
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"{wl.name}: {wl.frames} kf {wl.h}x{wl.w}x{wl.channels}, "
                               f"{wl.edges} edges, {per_step} edges per step on CPU",
                   "alpha": wl.alpha},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{per_step} edges per step x {args.steps} steps of {wl.name}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm

def run_scatter_mean(args, wl):
    """GraphAgg scatter-mean at the workload's sizes (one GPU): E = the batch's
    edges, F = 128 * h * w features per edge, keyframe ids = the batch's ii.
    Prints one JSON line with CUDA-event times (median of `steps`) of the whole
    dc_scatter_mean call and HBM GB/s on its algorithmic bytes."""
    from slam_hands_b200 import DroidCorrelation, configs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ii, _ = configs.make_edges(wl, seed=configs.SEED)
    ii = np.asarray(ii, np.int32)
    E, F = len(ii), 128 * wl.h * wl.w
    K = len(np.unique(ii))
    feats = torch.randn(E, F, device=dev)
    dc = DroidCorrelation(wl.h, wl.w, max_frames=wl.frames, max_edges=E, device=dev)
    agg = torch.empty(K, F, device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, device=dev)
    for _ in range(max(args.warmup, 3)):
        dc.scatter_mean(feats, ii, agg=agg)
    ts = []
    for _ in range(args.steps):
        flush.add_(1.0)  # L2 flush between calls
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dc.scatter_mean(feats, ii, agg=agg)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ms = statistics.median(ts)
    byts = (E + K) * F * 4
    print(json.dumps({"kernel": "dc_scatter_mean", "workload": wl.name, "E": E, "K": K, "F": F,
                      "ms_per_call": ms, "alg_bytes": byts, "GBs": byts / (ms * 1e-3) / 1e9}))
    return 0


def run_encoder(args, wl):
    """The corr encoder's first layer alone (dc_corr_encode) on one batch of the
    workload: M = its edges, 196 fp32 channels in, 128 fp16 channels out,
    seeded features and weights.  Prints one JSON line with the CUDA-event time
    (median of `steps`, L2 flushed between calls) and HBM GB/s on its
    algorithmic bytes (features read once, outputs written once)."""
    from slam_hands_b200 import DroidCorrelation

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M = wl.edges if wl.mode != "alt" else 48
    dc = DroidCorrelation(wl.h, wl.w, max_frames=2, max_edges=M, device=dev)
    g = torch.Generator(device=dev).manual_seed(20261202)
    corr = torch.randn(M, dc.out_channels, wl.h, wl.w, device=dev, generator=g)
    w = torch.randn(128, dc.out_channels, device=dev, generator=g) / 14.0
    b = torch.randn(128, device=dev, generator=g) * 0.1
    dc.set_corr_encoder(w, b)
    out = torch.empty(M, 128, wl.h, wl.w, dtype=torch.float16, device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, device=dev)
    for _ in range(max(args.warmup, 3)):
        dc.corr_encode(corr, out=out)
    ts = []
    for _ in range(args.steps):
        flush.add_(1.0)
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dc.corr_encode(corr, out=out)
        e.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(e))
    ms = statistics.median(ts)
    byts = corr.numel() * 4 + out.numel() * 2
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        peak, src = float(json.load(open(peaks_path))["hbm_gbs"]), "measured"
    gbs = byts / (ms * 1e-3) / 1e9
    print(json.dumps({"kernel": "dc_corr_encode", "workload": wl.name, "M": M,
                      "ms_per_call": ms, "alg_bytes": byts, "GBs": gbs, "frac": gbs / peak,
                      "peak_source": src}))
    return 0


def main():
    args = parse()
    from slam_hands_b200 import configs

    wl = configs.WORKLOADS[args.workload]
    if args.tile_order is None:
        args.tile_order = "auto" if wl.mode == "alt" else "source"
    if args.impl == "reference":
        return run_reference_arm(args, wl)
    if args.scatter_mean:
        return run_scatter_mean(args, wl)
    if args.encoder:
        return run_encoder(args, wl)

    from slam_hands_b200 import DroidCorrelation
    from slam_hands_b200.shard import SlotRing, edge_range, peers_alive, replicate_store

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    store = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
        pg = dist
        store = dist.distributed_c10d._get_default_store()


    # inputs: frames from rank 0 (seeded, replicated by NCCL broadcast).  The
    # frontend workloads (<= 48 edges, C1/C2/C4 up to 96) give every rank its own
    # seeded batch of the same size (weak scaling); the backend workloads
    # (C3, C5) split the edge list into contiguous per-rank ranges.
    fm, ii0, jj0, coords = configs.make_device_inputs(wl, dev, seed=configs.SEED)
    frontend = wl.mode != "alt"
    if not frontend:
        a, b = edge_range(len(ii0), world, rank)
        ii, jj, coords = ii0[a:b], jj0[a:b], coords[a:b].contiguous()
        if args.edges > 0:
            ii, jj, coords = ii[:args.edges], jj[:args.edges], coords[:args.edges].contiguous()
    else:
        ii, jj = configs.make_edges(wl, seed=configs.SEED + 101 * rank) if rank else (ii0, jj0)
    M = len(ii)
    if rank and frontend:
        g = torch.Generator(device=dev)
        g.manual_seed(configs.SEED + 7 * rank)
        base = torch.from_numpy(configs.grid_coords(wl.h, wl.w)).to(dev)[None]
        coords = (base + torch.randn(M, 2, wl.h, wl.w, generator=g, device=dev) * wl.sigma).contiguous()
    # two spare slots: the keyframe of step k + 2 is packed (and replicated)
    # while step k's kernel reads the others, so the transfer between GPUs has
    # a whole step of slack
    SPARES = 2
    dc = DroidCorrelation(wl.h, wl.w, channels=wl.channels, precision=args.precision,
                          alpha=wl.alpha, max_frames=wl.frames + SPARES, max_edges=M, device=dev)
    dc.set_tile_order(args.tile_order)
    out = torch.empty(M, dc.out_channels, wl.h, wl.w, device=dev)
    # L2 flush between steps: READ a buffer twice the L2 size, so the cache is
    # left holding clean lines (a write flush would leave ~126 MB of dirty lines
    # whose write-back the next step would pay for)
    flush = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    flush_sink = torch.empty((), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    s_rep = torch.cuda.Stream(dev)
    BCAST_TIMEOUT_S = 60.0

    # ---- the resident keyframe graph: rank 0 packs every keyframe once and one
    # NCCL broadcast of the packed store reaches the other ranks (timed apart)
    if rank == 0:
        dc.set_frames(fm)
    torch.cuda.synchronize()
    replication = None
    if pg is not None:
        if peers_alive(store, -1, world, rank, timeout_s=60.0):
            raise RuntimeError("a rank did not join")
        # NCCL sets up its communicator on the first collective: not part of the copy
        warm = torch.zeros(1, device=dev)
        pg.all_reduce(warm)
        torch.cuda.synchronize()
        ra, rb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ra.record(stream)
        replicate_store(dc, 0, wl.frames, timeout_s=BCAST_TIMEOUT_S)
        rb.record(stream)
        torch.cuda.synchronize()
        nbytes = dc.store_slots(0, wl.frames).numel()
        rms = ra.elapsed_time(rb)
        replication = {"what": f"NCCL broadcast of the packed store ({wl.frames} keyframes) "
                               "from rank 0, once, before the timed steps",
                       "bytes": nbytes, "ms": rms, "GBs": nbytes / (rms * 1e-3) / 1e9}

    # ---- per-step keyframes on several GPUs: the other ranks pull rank 0's new
    # packed slot through the copy engines over NVLink (CUDA IPC: rank 0's store
    # opened in every process), so no SM is spent on the transfer and it
    # overlaps the fused kernel.  Stream-ordered counters in rank 0's store page
    # order pack -> pull (word 0 = last packed step + 1) and pull -> the next
    # pack (word r = rank r's last pulled step + 1), with no host round trip.
    ipc = False
    if pg is not None and frontend:
        if rank == 0:
            store.set("dc/ipc/store", dc.store_ipc_handle())
        else:
            dc.attach_source(store.get("dc/ipc/store"))
        pg.barrier()
        ipc = True

    # ---- per step (frontend workloads): keyframe f = k % frames arrives; rank 0
    # packs it into the ring's spare slot and broadcasts that slot, while the
    # step's kernel runs on the previous mapping; edges are translated to slots
    n_steps_all = max(args.warmup, 3) + args.steps + 2 * (3 + args.steps) + 2
    step_edges = []
    ring_sim = SlotRing(wl.frames, spares=SPARES)
    for k in range(n_steps_all):
        f = k % wl.frames
        slot = ring_sim.begin(f)
        ring_sim.commit(f)
        step_edges.append((f, slot, np.asarray(ring_sim.slots(ii), np.int32),
                           np.asarray(ring_sim.slots(jj), np.int32)))
    step_ii = [torch.from_numpy(e[2]).to(dev) for e in step_edges]
    step_jj = [torch.from_numpy(e[3]).to(dev) for e in step_edges]
    ii_static = torch.as_tensor(ii, dtype=torch.int32, device=dev)
    jj_static = torch.as_tensor(jj, dtype=torch.int32, device=dev)

    def prep(k, strm, fm_src=None):
        """Keyframe of step k into its slot (rank 0 packs, all ranks receive)."""
        f, slot = step_edges[k][0], step_edges[k][1]
        src = fm[f:f + 1] if fm_src is None else fm_src
        with torch.cuda.stream(strm):
            if rank == 0:
                if ipc and k >= 1:
                    for r in range(1, world):  # every rank has pulled keyframe k - 1
                        dc.sync_wait(r, k, stream=strm)
                dc.set_frames(src, first_slot=slot, stream=strm)
                if ipc:
                    dc.sync_signal(0, k + 1, stream=strm)
            elif ipc:
                dc.sync_wait(0, k + 1, remote=True, stream=strm)
                dc.pull_slots(slot, 1, stream=strm)
                dc.sync_signal(rank, k + 1, remote=True, stream=strm)
            if pg is not None and not ipc:
                replicate_store(dc, slot, 1)  # stream-ordered; NCCL watchdog bounds it

    vols = ([torch.empty(sh, dtype=torch.float32, device=dev) for sh in dc.volume_shapes(M)]
            if args.materialise else None)

    stage_ev = []  # materialised path: (build+pyramid start, lookup start, end) per step
    proj = None
    if args.project:
        # seeded poses near the identity and inverse depths of the step's keyframes
        prng = np.random.default_rng(configs.SEED + 13)
        poses_p = torch.from_numpy(configs.random_poses(wl.frames + 1, prng, trans=0.15, angle=0.08)).to(dev)
        disps_p = torch.from_numpy(prng.uniform(0.15, 1.2, (wl.frames + 1, wl.h, wl.w))
                                   .astype(np.float32)).to(dev)
        intr_p = torch.tensor([0.95 * wl.w, 0.95 * wl.w, wl.w / 2 - 0.5, wl.h / 2 - 0.5],
                              dtype=torch.float32, device=dev)
        proj = (poses_p, disps_p, intr_p, torch.empty_like(coords),
                torch.empty(M, wl.h, wl.w, device=dev))

    def corr(k, coords_=None, record=False, out_=None):
        ii_ = step_ii[k] if frontend else ii_static
        jj_ = step_jj[k] if frontend else jj_static
        coords_ = coords if coords_ is None else coords_
        out_ = out if out_ is None else out_
        if vols is not None:
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
            if evs:
                evs[0].record(stream)
            dc.build_volume(ii_, jj_, vols)
            if evs:
                evs[1].record(stream)
            dc.lookup(vols, coords_, out_)
            if evs:
                evs[2].record(stream)
                stage_ev.append(evs)
        elif proj is not None:
            dc.project_build_and_lookup(proj[0], proj[1], proj[2], ii_, jj_, out=out_,
                                        coords=proj[3], valid=proj[4])
        else:
            dc.build_and_lookup(ii_, jj_, coords_, out_)

    k_glob = 0  # next step index (into step_edges)
    prep_done = {}
    if frontend:
        for k0 in range(SPARES):
            prep(k0, stream)
            prep_done[k0] = torch.cuda.Event()
            prep_done[k0].record(stream)

    def step(record_ev=None):
        """Step k: kernel k on the current slots beside the keyframe of step
        k + 2 (packed and replicated on a side stream); the step ends when the
        kernel and the keyframe of step k + 1 (prepared during step k - 1) are
        both in place."""
        nonlocal k_glob
        k = k_glob
        if record_ev is not None:
            record_ev[0].record(stream)
        if frontend:
            ev_go = torch.cuda.Event()
            ev_go.record(stream)
            s_rep.wait_event(ev_go)
            prep(k + SPARES, s_rep)
            prep_done[k + SPARES] = torch.cuda.Event()
            prep_done[k + SPARES].record(s_rep)
        if record_ev is not None:
            record_ev[2].record(stream)
        corr(k, record=record_ev is not None)
        if record_ev is not None:
            record_ev[3].record(stream)
        if frontend:
            stream.wait_event(prep_done.pop(k + 1))
        if record_ev is not None:
            record_ev[1].record(stream)
        k_glob += 1

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timed region.  Every step is bracketed by CUDA events
    # on the launching stream and preceded by an L2 flush (outside the events).
    # All K steps are enqueued behind a ~20 ms device sleep so that host-side
    # launch overhead never shows up as device time.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    launches0 = dc.launch_count
    torch.cuda._sleep(int(0.02 * 1.9e9))
    if pg is not None:
        # align the GPUs' timelines after the sleep (a one-float all-reduce on the
        # launching stream, outside the step events): the ranks' steps are
        # coupled through the keyframe replication, so a start skew would
        # otherwise be charged to the first steps of the earlier rank
        align = torch.zeros(1, device=dev)
        pg.all_reduce(align)
    for s in range(args.steps):
        torch.sum(flush, dim=0, out=flush_sink)
        step(ev[s])
    torch.cuda.synchronize()
    launches = dc.launch_count - launches0
    if pg is not None:
        pg.barrier()
        if peers_alive(store, -2, world, rank, timeout_s=60.0):
            raise RuntimeError("a rank left during the timed steps")
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b, _, _ in ev) / args.steps
    kern_ms = sum(c.elapsed_time(d) for _, _, c, d in ev) / args.steps
    if pg is not None:
        t = torch.tensor([ms, kern_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, kern_ms = t.tolist()
    value = (M * world if frontend else len(ii0)) / (ms * 1e-3)

    # ---- end to end through the public API with host buffers: per step the
    # new keyframe's feature map (rank 0), the coordinates and the slot-translated
    # edge lists are copied in from pinned memory, the full output copied out
    fm_h = fm.cpu().pin_memory()
    coords_h = coords.cpu().pin_memory()
    ii_h = [torch.from_numpy(e[2]).pin_memory() for e in step_edges]
    jj_h = [torch.from_numpy(e[3]).pin_memory() for e in step_edges]
    ii_sh = torch.as_tensor(ii, dtype=torch.int32).pin_memory()
    jj_sh = torch.as_tensor(jj, dtype=torch.int32).pin_memory()
    out_h = torch.empty(out.shape, dtype=torch.float32).pin_memory()

    # Pipelined: step k's input copies, its correlation in E2E_CHUNKS edge
    # chunks, and each chunk's output copy run on three streams, so the
    # host->device copy of step k+1 and the compute of later chunks overlap the
    # device->host copy of earlier outputs (PCIe is full duplex).  Inputs and
    # outputs are double-buffered by step parity; the keyframe of step k goes
    # into its ring slot on the compute stream, in order behind step k-1's
    # kernels, so no kernel reads a slot while it is rewritten.
    pipelined = vols is None and proj is None
    E2E_CHUNKS = 4
    s_h2d, s_comp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))
    bufs = [dict(fm=torch.empty_like(fm[:1]), coords=torch.empty_like(coords),
                 ii=torch.empty_like(ii_static), jj=torch.empty_like(jj_static),
                 out=torch.empty_like(out),
                 enc=torch.empty(M, 128, wl.h, wl.w, dtype=torch.float16, device=dev))
            for _ in range(2)]
    enc_h = torch.empty(M, 128, wl.h, wl.w, dtype=torch.float16).pin_memory()
    bounds = [(M * c // E2E_CHUNKS, M * (c + 1) // E2E_CHUNKS) for c in range(E2E_CHUNKS)]
    bounds = [(a, b) for a, b in bounds if b > a] if pipelined else [(0, M)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    ev_chunk = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]

    def e2e_pipe_step(j, encode=False):
        nonlocal k_glob
        k = k_glob
        k_glob += 1
        b, B = j % 2, bufs[j % 2]
        f = step_edges[k][0]
        with torch.cuda.stream(s_h2d):
            if j >= 2:
                s_h2d.wait_event(ev_used[b])  # compute of step j-2 is done with them
            if rank == 0 and frontend:
                B["fm"].copy_(fm_h[f:f + 1], non_blocking=True)
            B["coords"].copy_(coords_h, non_blocking=True)
            B["ii"].copy_(ii_h[k] if frontend else ii_sh, non_blocking=True)
            B["jj"].copy_(jj_h[k] if frontend else jj_sh, non_blocking=True)
            ev_in[b].record(s_h2d)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            if j >= 2:
                s_comp.wait_event(ev_free[b])  # the output copy of step j-2 is done
            if frontend:
                prep(k, s_comp, fm_src=B["fm"])
            for c, (a0, a1) in enumerate(bounds):
                if encode:
                    dc.build_lookup_encode(B["ii"][a0:a1], B["jj"][a0:a1], B["coords"][a0:a1],
                                           corr=B["out"][a0:a1], out=B["enc"][a0:a1],
                                           stream=s_comp)
                elif pipelined:
                    dc.build_and_lookup(B["ii"][a0:a1], B["jj"][a0:a1], B["coords"][a0:a1],
                                        out=B["out"][a0:a1], stream=s_comp)
                else:
                    with torch.cuda.stream(s_comp):
                        corr(k, coords_=B["coords"], out_=B["out"])
                ev_chunk[b][c].record(s_comp)
            ev_used[b].record(s_comp)
        with torch.cuda.stream(s_d2h):
            for c, (a0, a1) in enumerate(bounds):
                s_d2h.wait_event(ev_chunk[b][c])
                if encode:
                    enc_h[a0:a1].copy_(B["enc"][a0:a1], non_blocking=True)
                else:
                    out_h[a0:a1].copy_(B["out"][a0:a1], non_blocking=True)
            ev_free[b].record(s_d2h)

    def time_e2e(encode):
        torch.cuda.synchronize()
        for j in range(3):
            e2e_pipe_step(j, encode)
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s_h2d):
            torch.cuda._sleep(int(0.02 * 1.9e9))
        e0.record(s_h2d)
        for j in range(args.steps):
            e2e_pipe_step(3 + j, encode)
        e1.record(s_d2h)
        torch.cuda.synchronize()
        t_ms = e0.elapsed_time(e1) / args.steps
        if pg is not None:
            t = torch.tensor([t_ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            t_ms = t.item()
        return t_ms

    e2e_ms = time_e2e(False)
    h2d = ((fm_h[0].numel() * 4 if frontend else 0) + coords_h.numel() * 4 + 2 * M * 4)
    d2h = out_h.numel() * 4

    # ---- parity spot check of the timed output (cheap, rank 0): the last e2e
    # step's host copy equals a device-resident recomputation of that step
    if rank == 0:
        torch.cuda.synchronize()
        last = bufs[(3 + args.steps - 1) % 2]
        chk = torch.empty_like(out)
        dc.build_and_lookup(last["ii"], last["jj"], last["coords"], chk)
        torch.cuda.synchronize()
        assert torch.isfinite(chk).all().item()
        if pipelined:
            assert torch.equal(out_h, chk.cpu())

    # ---- the same steps with the update operator's first corr-encoder layer
    # fused behind the lookup (dc_build_lookup_encode: corr_enc_0 + ReLU + fp16,
    # cuda_slam/main.cu:603-606, seeded weights): 128 fp16 channels go back
    # to the host instead of 196 fp32 ones
    e2e_enc = None
    if pipelined and frontend and dc.out_channels <= 256:
        wg = torch.Generator(device=dev)
        wg.manual_seed(configs.SEED + 17)
        enc_w = torch.randn(128, dc.out_channels, generator=wg, device=dev) / dc.out_channels ** 0.5
        enc_b = 0.1 * torch.randn(128, generator=wg, device=dev)
        dc.set_corr_encoder(enc_w, enc_b)
        enc_ms = time_e2e(True)
        if rank == 0:
            last = bufs[(3 + args.steps - 1) % 2]
            chk16, _ = dc.build_lookup_encode(last["ii"], last["jj"], last["coords"])
            torch.cuda.synchronize()
            assert torch.equal(enc_h, chk16.cpu())
        e2e_enc = {"value": M * world / (enc_ms * 1e-3), "unit": UNIT,
                   "h2d_bytes_per_step": ((fm_h[0].numel() * 4 if rank == 0 else 0)
                                          + coords_h.numel() * 4 + 2 * M * 4),
                   "d2h_bytes_per_step": enc_h.numel() * 2, "ms_per_step": enc_ms,
                   "what": "each step also encodes the 196 correlation channels to the "
                           "update operator's 128 fp16 channels on the GPU "
                           "(dc_build_lookup_encode) and copies those out"}

    if rank != 0:
        if pg is not None:
            pg.destroy_process_group()
        return 0

    # ---- roofline of the dominant kernel (algorithmic bytes per launch / event time)
    hw = wl.h * wl.w
    D = 2 * dc.radius + 1
    esz = 4 if args.precision in ("fp32", "fp32x3") else 2  # fp32x3: hi + lo fp16 copies
    uniq_frames = len(set(ii) | set(jj))
    pyr_rows = sum((wl.h >> l) * (wl.w >> l) for l in range(dc.levels))
    io_bytes = M * (2 * hw * 4 + dc.out_channels * hw * 4)          # coords in, output out
    frame_bytes = uniq_frames * pyr_rows * wl.channels * esz          # each store row read once
    stages = None
    if vols is None:
        alg_bytes = io_bytes + frame_bytes
        kernel_name = "build_and_lookup"
    else:
        # materialised: V0 written, V0 read back by the pyramid, V1..V3 written,
        # the lookup's (2r+2)^2 taps per pixel and level read once, output written
        taps = (2 * dc.radius + 2) ** 2
        vol_bytes = [M * hw * (wl.h >> l) * (wl.w >> l) * 4 for l in range(dc.levels)]
        build_bytes = vol_bytes[0] * 2 + sum(vol_bytes[1:]) + frame_bytes
        lookup_bytes = io_bytes + M * hw * dc.levels * taps * 4
        alg_bytes = build_bytes + lookup_bytes
        kernel_name = "build_volume (tcgen05 V0 + pyramid) + lookup"
        b_ms = sum(a.elapsed_time(b) for a, b, _ in stage_ev) / len(stage_ev)
        l_ms = sum(b.elapsed_time(c) for _, b, c in stage_ev) / len(stage_ev)
        stages = {"build_volume_ms": b_ms, "build_volume_alg_bytes": build_bytes,
                  "build_volume_gbs": build_bytes / (b_ms * 1e-3) / 1e9,
                  "lookup_ms": l_ms, "lookup_alg_bytes": lookup_bytes,
                  "lookup_gbs": lookup_bytes / (l_ms * 1e-3) / 1e9}
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        peak, peak_src = float(json.load(open(peaks_path))["hbm_gbs"]), "measured"
    if stages is not None:
        stages["build_volume_frac"] = stages["build_volume_gbs"] / peak
        stages["lookup_frac"] = stages["lookup_gbs"] / peak
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "kernel": kernel_name, "peak_source": peak_src,
                "alg_bytes_per_launch": alg_bytes}
    if vols is None and proj is None and args.precision == "fp32":
        # the exact mode runs the alt-corr kernel: FP32 CUDA-core work,
        # (2r+2)^2 taps x 2C flops per pixel and level (windows not clipped at borders)
        flops = M * hw * dc.levels * (2 * dc.radius + 2) ** 2 * 2 * wl.channels
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12  # SMs x FP32 lanes x FMA x max clock
        tfs = flops / (kern_ms * 1e-3) / 1e12
        roofline = {"bound": "fp32", "achieved": tfs, "peak": fp32_peak, "unit": "TFLOP/s",
                    "frac": tfs / fp32_peak, "kernel": "alt_lookup (FFMA gathered dots)",
                    "peak_source": "nominal (148 SMs x 128 FP32 lanes x 2 flop x 1.965 GHz)",
                    "alg_flops_per_launch": flops}
    traffic = None
    tpath = os.path.join(ROOT, "profiles", f"corr_tc_kernel_{wl.name}.md")
    if os.path.exists(tpath) and args.precision == "fp16" and vols is None:
        for ln in open(tpath):
            if ln.startswith("traffic_bytes_per_launch:"):
                traffic = int(ln.split(":")[1])
    roofline["traffic"] = traffic
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if wl.mode == "alt" else "weak",
        "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.frames} kf {wl.h}x{wl.w}x{wl.channels}, "
                               f"{M} edges per GPU ({wl.mode} workload), build+pyramid+r3 "
                               + ("lookup, volumes materialised in HBM" if vols is not None
                                  else "lookup, no volume stored")
                               + (", coords reprojected from poses + inverse depths in the step"
                                  if proj is not None else ""),
                   "alpha": wl.alpha, "l2": "flushed between steps (252 MB read)",
                   "tile_order": args.tile_order,
                   **({"edges_cap": args.edges, "valid": "profiling case, not a bench line"}
                      if args.edges > 0 else {}),
                   "step": ("one keyframe arrives per step: packed into the spare store slot "
                            "(other ranks pull it from rank 0 over NVLink with the copy "
                            "engines) beside the step's kernel over the resident keyframe "
                            "graph" if frontend else
                            "one backend pass over the resident keyframe graph (keyframes "
                            "replicated once before the timed steps, see replication)"),
                   "parallelism": f"edges sharded, dp{world}"},
        "gpu_launches": launches,
        "kernel_ms": kern_ms,
        "roofline": roofline,
        "e2e": {"value": M * world / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "pipelined": (f"{E2E_CHUNKS} edge chunks; input copy, compute and output copy "
                              "on three streams, double-buffered" if pipelined else False)},
        "clocks": clk,
    }
    if stages is not None:
        line["stages"] = stages
    if replication is not None:
        line["replication"] = replication
    if e2e_enc is not None:
        line["e2e_encoded"] = e2e_enc

    # reference kernels on this GPU (cuBLAS FP16 GEMM + pools + lookups), if built
    if not args.no_ref_gpu and world == 1:
        try:
            from oracle import ref as REF

            if REF.available():
                fm_np = fm.cpu().numpy()
                _, _, rms = REF.build_and_sample_fp16(fm_np, np.asarray(ii), np.asarray(jj),
                                                      coords.cpu().numpy(), wl.alpha, iters=10)
                line["reference_gpu"] = {"value": M / (rms * 1e-3), "unit": UNIT,
                                         "ms_per_step": rms,
                                         "what": "reference kernels (main.cu:1077-1217) + "
                                                 "cublasGemmBatchedEx FP16, rebuilt sm_100a, "
                                                 "inputs resident, L2 not flushed"}
        except Exception as ex:  # report, do not fail the bench
            line["reference_gpu"] = {"unavailable": str(ex)[:200]}

    if not args.no_cpu_baseline and world == 1:
        fm_np = fm.cpu().numpy()
        v, n, cores = cpu_sample(wl, fm_np, np.asarray(ii), np.asarray(jj), coords.cpu().numpy(),
                                 threads=len(os.sched_getaffinity(0)))
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": f"{n} edges of {wl.name} (fp32 C/OpenMP oracle)"}
    print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
