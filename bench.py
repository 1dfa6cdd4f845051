"""Benchmark of the nest-splatting render hot path on B200 (benchmark config 2).

One step = one frame of config 2: 1,000,000 surfels whose attributes come from
an RVQ stream decoded on the fly (6 stages x 256 x 59 fp32 codebooks), rendered
at 1297x840 (decode -> activate -> preprocess -> tile binning + onesweep sort
-> blend + 16-level hash grid -> tensor-core MLP -> mask). Synthetic seeded
scene (no dataset exists on this machine).

N GPUs (torchrun, one rank per GPU, NCCL): every rank renders its own camera of
the orbit (weak scaling: one frame per GPU per step). RVQ decode is sharded by
surfel range and followed by an NCCL all-gather of the decoded attributes (the
only collective). value = total megapixels rendered by all ranks / max-over-
ranks step time.

--impl reference: the reference's CPU implementation of the path on the host
cores. The reference CUDA rasterizer cannot be built on this image (its glm
dependency is absent), so the CPU oracle restatement (oracle/, C++ + OpenMP)
stands in for it, timed on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nest-splatting_b200"))
sys.path.insert(0, ROOT)

METRIC = "frames/s & Mpix/s, 1M surfels 1297×840 @1/2/4/8 B200; RVQ decode GB/s vs HBM"
UNIT = "Mpix/s"
WORKLOAD = "config2: 1M RVQ-decoded surfels, 1297x840, 16x2 fp16 hash grid, MLP 32-64-64-3"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with `nvidia-smi -lms` during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 50):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", f"-lms={self.period}"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)  # first sample before the timed work starts
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        rows = [[x.strip() for x in l.split(",")] for l in self.out.splitlines() if l.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        num = lambda v: float(v) if v.replace(".", "", 1).isdigit() else None  # noqa: E731
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        # The decode exchange's all-gather runs on NCCL's stream while the
        # previous frame renders: a high-priority stream lets its CTAs in as
        # the render's CTAs retire (N = 4: 775-776 -> 780 Mpix/s).
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local),
                                pg_options=opts)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def flush_l2(buf):
    buf.add_(1)  # 256 MB read+write evicts the 126 MB L2


def blend_algorithmic_bytes(num_rendered, surfels, width, height, channels, table_bytes):
    """Unique DRAM bytes one blend launch must move: every surfel record once
    (128 B), the sorted point list (4 B per instance), the tile ranges, the
    per-pixel outputs (C features + 14 aux + 3 final T + 2 counts, fp32) and one
    pass over the hash table. Re-gathers of records and table rows are served
    by L2 and are not counted."""
    tiles = ((width + 15) // 16) * ((height + 15) // 16)
    return surfels * 128 + num_rendered * 4 + tiles * 8 + width * height * (channels + 14 + 5) * 4 + table_bytes


def profiled_traffic():
    """dram read+write bytes per blend launch from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "blend_kernel_config2_ncu.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1])
    except OSError:
        pass
    return None


def train_step_timing(sc, cam, dev, steps, warmup=2):
    """benchmark config 4: one training step (forward, MLP, L1 + normal loss,
    backward into the surfels, the hash table and the MLP) on the config-2 scene."""
    import torch

    import diff_surfel_rasterization as dsr
    from nest_b200 import train

    g = sc.grid
    state = train.make_state(sc, device=dev)
    rs = dsr.GaussianRasterizationSettings(
        image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=0, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False, beta=0.0, if_contract=False, record_transmittance=False,
        max_intersections=0)
    hs = dsr.HashGridSettings(L=g.levels, S=g.S, H=g.base_resolution, align_corners=False, interpolation=0,
                              shape_dims=torch.tensor([0, g.channels, g.channels], dtype=torch.int32, device=dev))
    rast = dsr.GaussianRasterizer(rs, hs)

    def one(evs=None):
        for t in state.leaves():
            t.grad = None
        if evs:
            evs[0].record()
        loss, _, _ = train.forward(state, rast, cam)
        if evs:
            evs[1].record()
        loss.backward()
        if evs:
            evs[2].record()
        return loss

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    losses = []
    for i in range(steps):
        losses.append(one(evs[i]))
    torch.cuda.synchronize()
    # Medians over the steps (a step's float-atomic backward occasionally runs
    # far longer than its neighbours; the mean is reported beside).
    fwd = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
    bwd = statistics.median(e[1].elapsed_time(e[2]) for e in evs)
    bwd_mean = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    ms = fwd + bwd
    # The same steps with the fixed-point (bit-reproducible) table gradient, as
    # the drop-in selects it under torch.use_deterministic_algorithms.
    was = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        for _ in range(warmup):
            one()
        torch.cuda.synchronize()
        for i in range(steps):
            one(evs[i])
        torch.cuda.synchronize()
    finally:
        torch.use_deterministic_algorithms(was)
    bwd_det = statistics.median(e[1].elapsed_time(e[2]) for e in evs)
    return {"workload": "config 4: config-2 scene, forward + backward of L1(rgb, target) + 0.05 normal loss; "
                        "leaves means, scales, rotations, opacities, hash table, MLP weights",
            "steps": steps, "ms_per_step": round(ms, 3), "forward_ms": round(fwd, 3),
            "backward_ms": round(bwd, 3), "backward_ms_mean": round(bwd_mean, 3),
            "mpix_per_s": round(cam.width * cam.height / 1e6 * 1000.0 / ms, 3), "statistic": "median over steps",
            "backward_ms_deterministic_table": round(bwd_det, 3),
            "loss_first": round(float(losses[0].detach()), 6)}


def gather_peak(fr, dev, cam, lookups=128, reps=5):
    """The blend's gather roofline: hash-grid lookups per second of a kernel that
    does nothing else (ns_gather_probe: the blend's lookup code at full
    occupancy, four lookups in flight per thread), in corner bytes per second,
    for two point patterns on the same table:
      * "coherent" (the roofline denominator): the blend's pattern and order,
        a warp's 32 lanes as a 16 x 2 pixel strip with 8 samples each on
        stacked surfels, all 16 levels in an outer loop; the strip spacing is
        this camera's pixel footprint at the scene (distance 3) in grid units;
      * "random_hashed": every lane an independent point of the hashed levels
        (5-15), the pattern's worst case, for context."""
    import torch

    from nest_b200 import _lib
    lib = _lib.load()
    g = fr.grid
    T = int(g.offsets[1] - g.offsets[0])
    level0 = next(l for l in range(g.levels)
                  if (int(math.ceil(2 ** (l * g.S) * g.base_resolution - 1)) + 2) ** 3 > T)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 8
    sink = torch.empty(blocks * 256, dtype=torch.float32, device=dev)
    fp16 = int(fr.table.dtype == torch.float16)
    stream = _lib.stream_handle(dev)
    grid_range = float(g.gridrange[1] - g.gridrange[0])
    spacing = 2.0 * cam.tanfovx / cam.width * 3.0 / grid_range  # pixel footprint at distance 3
    out = {}
    for name, l0, nl, sp in (("coherent", 0, g.levels, spacing), ("random_hashed", level0, g.levels - level0, 0.0)):
        def run():
            _lib.check("ns_gather_probe", lib.ns_gather_probe(
                fr.table.data_ptr(), fp16, fr.offsets.data_ptr(), l0, nl, float(g.S), g.base_resolution, lookups,
                float(sp), blocks, sink.data_ptr(), stream))

        for _ in range(2):
            run()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        ms = statistics.median(times)
        nbytes = blocks * 256 * lookups * 8 * fr.table.element_size() * fr.table.shape[1]
        out[name] = {"gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 4), "levels": [l0, l0 + nl - 1],
                     "spacing_grid_units": round(sp, 6)}
    out["lookups"] = blocks * 256 * lookups
    out["gbs"] = out["coherent"]["gbs"]
    return out


def rvq_timing(dev, hbm_peak, sizes=(200_000, 1_000_000, 3_000_000), iters=20, warmup=3):
    """RVQ decode (benchmark config 0 codebooks and indices) on the GPU at the
    sizes the scope names: median device time of `iters` runs after `warmup`,
    L2 flushed before each (the 200k output fits in L2)."""
    import torch

    from nest_b200 import raster, synth
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for n in sizes:
        cb, idx = synth.config0(n)
        cb, idx = cb.to(dev), idx.to(dev)
        dec = torch.empty((n, cb.shape[2]), dtype=torch.float32, device=dev)
        for _ in range(warmup):
            raster.rvq_decode(idx, cb, dec)
        times = []
        for _ in range(iters):
            flush_l2(flush)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            raster.rvq_decode(idx, cb, dec)
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        ms = statistics.median(times)
        nbytes = n * (cb.shape[0] + 4 * cb.shape[2])
        out[str(n)] = {"ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                       "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4)}
        del cb, idx, dec
    return out


def rvq_cpu_timing(n=200_000, iters=20, warmup=3):
    """The reference's PyTorch CPU path of the RVQ decode (benchmark config 0):
    index_select + in-order adds on the host cores, all of them."""
    import torch

    from nest_b200 import synth
    from oracle import oracle
    prev = torch.get_num_threads()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        cb, idx = synth.config0(n)
        for _ in range(warmup):
            oracle.rvq_decode_torch(idx, cb)
        times = []
        for _ in range(iters):
            t0 = time.perf_counter()
            oracle.rvq_decode_torch(idx, cb)
            times.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(prev)
    sec = statistics.median(times)
    nbytes = n * (cb.shape[0] + 4 * cb.shape[2])
    return {"surfels": n, "ms": round(sec * 1e3, 3), "surfels_per_s": round(n / sec, 1),
            "gbs": round(nbytes / sec / 1e9, 3), "cores": cores, "threads": cores,
            "statistic": f"median of {iters} after {warmup} warm-ups",
            "path": "torch CPU: index_select per stage + in-order fp32 adds (oracle.rvq_decode_torch)"}


def config1_timing(dev, steps=20, warmup=3):
    """benchmark config 1: single-view forward render of 200k surfels at 800x800
    (rasterizer forward with its instance-count read-back, then the MLP with the
    alpha mask), device-timed per frame with the L2 flushed before each."""
    import torch

    from nest_b200 import raster, synth
    sc = synth.config1()
    means, scales, rots, opac = synth.activate(sc.base)
    homo = synth.build_homotrans(sc.base)
    cam, g = sc.camera, sc.grid
    t = [x.to(dev).contiguous() for x in (means, scales, rots, opac.reshape(-1), homo,
                                          sc.ap_level.reshape(-1))]
    cfg = raster.RasterConfig(image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx,
                              tanfovy=cam.tanfovy, viewmatrix=cam.world_view_transform.to(dev).contiguous(),
                              projmatrix=cam.full_proj_transform.to(dev).contiguous(), levels=g.levels, S=g.S,
                              base_resolution=g.base_resolution, channels=g.channels, level_dim=g.level_dim)
    table, offs, gr = g.table.to(dev), g.offsets.to(dev), g.gridrange.to(dev)
    weights = raster.pack_mlp(sc.mlp).to(dev)
    scratch = raster.Scratch()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def frame():
        n, color, others, radii, _, _, _ = raster.rasterize_forward(cfg, *t, table, offs, gr, scratch=scratch)
        raster.mlp_forward(color, weights, alpha=others[1])
        return n

    for _ in range(warmup):
        frame()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        n = frame()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    ms = statistics.median(times)
    return {"workload": "config 1: 200k surfels, 800x800, 16x2 fp16 hash grid (U(+-1e-4)), MLP 32-64-64-3",
            "ms_per_frame": round(ms, 4), "frames_per_s": round(1000.0 / ms, 2),
            "mpix_per_s": round(cam.width * cam.height / 1e6 * 1000.0 / ms, 3), "instances": int(n),
            "statistic": f"median of {steps} frames after {warmup} warm-ups, L2 flushed before each",
            "path": "raster.rasterize_forward (ns_rasterize_forward, one count read-back) + ns_mlp_forward"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from nest_b200 import _lib, synth
    from nest_b200.camera import orbit_camera
    from nest_b200.frame import FrameRenderer

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    sc = synth.config2()
    W, H = sc.camera.width, sc.camera.height
    cam = orbit_camera(W, H, 60.0, 4.0, 360.0 * rank / max(world, 1))
    fr = FrameRenderer(sc, device=dev, capacity=10_000_000)
    view = cam.world_view_transform.to(dev).contiguous()
    proj = cam.full_proj_transform.to(dev).contiguous()
    P = sc.P
    from nest_b200 import raster
    from nest_b200.views import DecodeRing, DecodeShard, shard_range
    lo, hi = shard_range(P, world, rank)
    if world > 1:
        # Every rank decodes all 59 columns of its surfel range; the all-gather
        # carries the 10 the rasterizer reads (views.DecodeShard).
        shard = DecodeShard.create(fr.rvq_idx, fr.dims, world, rank, columns=synth.BASE_DIMS)
        # Frame i+1's decode + all-gather runs on a side stream while frame i
        # renders (two attribute buffers); every step still decodes and
        # exchanges its own frame.
        ring = DecodeRing(fr.rvq_idx, fr.dims, world, rank, columns=synth.BASE_DIMS)

    def step(i, events=None, n=None):
        if world > 1:
            if i == 0:
                ring.prefetch(0, fr.codebooks, raster.rvq_decode)
            if n is None or i + 1 < n:
                ring.prefetch(i + 1, fr.codebooks, raster.rvq_decode)
            fr.decoded = ring.acquire(i)
            out = fr.render(cam, view, proj, events=events, skip_decode=True)
            ring.release(i)
            return out
        return fr.render(cam, view, proj, events=events)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    nst = _lib.NS_FRAME_STAGES
    stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * nst)] for _ in range(args.steps)]
    for evs in stage_ev:
        for e in evs:
            e.record()  # creates the underlying cudaEvent
    nw = max(args.warmup, 3)
    for i in range(nw):
        step(i, n=nw)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    flush_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches0 = lib.ns_kernel_launches()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            if world > 1 and i > 0:
                ring.acquire(i)  # frame i's exchange is complete before the flush
            flush_start[i].record()
            flush_l2(flush)
            starts[i].record()
            step(i, stage_ev[i], n=args.steps)
            ends[i].record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = lib.ns_kernel_launches() - launches0
    if world > 1:
        # Frame i+1's exchange overlaps frame i's render, so the steps are timed
        # as one sequence minus the L2 flushes between them; each flush starts
        # only after the next frame's exchange has completed, and frame 0's
        # exchange runs after the first flush, inside the timed interval.
        step_ms = [flush_start[0].elapsed_time(ends[-1]) -
                   sum(f.elapsed_time(s) for f, s in zip(flush_start, starts))]
    else:
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    stage_ms = {name: statistics.mean(ev[2 * k].elapsed_time(ev[2 * k + 1]) for ev in stage_ev)
                for k, name in enumerate(_lib.STAGE_NAMES)}
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    mpix = W * H / 1e6
    value = world * mpix * 1000.0 / ms_per_step

    # End to end through the public API with host buffers: every frame copies its
    # RVQ index stream (this rank's rows when sharded) and camera host -> device
    # and its RGB image device -> host, through FramePipeline (the copies of the
    # neighbouring frames overlap each frame's kernels). Timed over the whole
    # sequence on the device; the L2 flush before every frame (the measurement's
    # cache hygiene, not part of the frame) is timed by its own events and taken
    # out, as for `value`.
    from nest_b200.frame import FramePipeline
    host_idx = sc.rvq_idx.clone().pin_memory()
    host_cam = torch.stack([cam.world_view_transform, cam.full_proj_transform]).contiguous().pin_memory()
    host_rgb = [torch.empty((3, H, W), dtype=torch.float32).pin_memory() for _ in range(2)]
    pipe = FramePipeline(fr, shard if world > 1 else None, graphs=world == 1)
    run_args = (cam, lambda i: host_idx, lambda i: host_cam, lambda i: host_rgb[i % 2])
    pipe.run(2, *run_args)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs = torch.cuda.current_stream(dev)
    fl_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]

    def timed_flush(i):
        fl_ev[i][0].record(cs)
        flush_l2(flush)
        fl_ev[i][1].record(cs)

    e2e_start.record(cs)
    pipe.run(args.steps, *run_args, before_frame=timed_flush)
    cs.wait_stream(pipe.out_stream)
    e2e_end.record(cs)
    torch.cuda.synchronize()
    # At N > 1 the next frame's exchange runs during a flush, so there the
    # flushes stay in the interval.
    e2e_flush_ms = sum(a.elapsed_time(b) for a, b in fl_ev) if world == 1 else 0.0
    e2e_ms = e2e_start.elapsed_time(e2e_end) - e2e_flush_ms
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms_step = float(t.item()) / args.steps
    h2d = host_idx[lo:hi].numel() if world > 1 else host_idx.numel()
    h2d += host_cam.numel() * 4
    d2h = host_rgb[0].numel() * 4

    exchange = exchange_timing(shard, fr.codebooks, dev, P, fr.stages, fr.dims) if world > 1 else None
    identical = frame_identity(fr, shard, cam, view, proj, dev) if world > 1 else None
    graph = graph_timing(fr, cam, view, proj, flush, args.steps) if world == 1 else None

    # Work statistics of the (identical) frames.
    samples = float(fr.others[7].sum().item())
    num_rendered = fr.num_rendered
    hbm_peak, _, peak_kind = peaks()
    table_bytes = fr.table.numel() * fr.table.element_size()
    blend_bytes = blend_algorithmic_bytes(num_rendered, P, W, H, fr.grid.channels, table_bytes)
    blend_ms = stage_ms["blend"]
    achieved = blend_bytes / (blend_ms * 1e-3) / 1e9
    traffic = profiled_traffic()
    rvq_bytes = (hi - lo) * (fr.stages + 4 * fr.dims) if world > 1 else P * (fr.stages + 4 * fr.dims)
    rvq_gbs = rvq_bytes / (stage_ms["decode"] * 1e-3) / 1e9 if world == 1 else None
    gather_tbs = samples * 16 * 8 * 4 / (blend_ms * 1e-3) / 1e12
    gather_gbs = gather_tbs * 1e3
    gpeak = gather_peak(fr, dev, cam)

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16 hash table, fp16 MLP operands)",
        "data": "synthetic (seeded config-2 scene; RVQ stream decoded every frame)",
        "config": {"workload": WORKLOAD, "surfels": P, "width": W, "height": H, "frames_per_step": world,
                   "parallelism": f"camera-sharded x{world}, RVQ decode surfel-sharded + NCCL all-gather"
                   if world > 1 else "single GPU",
                   "l2": "flushed between timed steps (256 MB write)"},
        "frames_per_s": round(world * 1000.0 / ms_per_step, 3),
        "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "work": {"instances": num_rendered, "blended_samples": int(samples)},
        "rvq_decode": {"gbs": round(rvq_gbs, 1) if rvq_gbs else None,
                       "frac_of_hbm": round(rvq_gbs / hbm_peak, 4) if rvq_gbs else None,
                       "bytes_per_surfel": fr.stages + 4 * fr.dims},
        "roofline": {"kernel": "blend_kernel<__half, 0>", "bound": "l1/l2 gather",
                     "achieved": round(gather_gbs, 1), "peak": gpeak["gbs"], "unit": "GB/s",
                     "frac": round(gather_gbs / gpeak["gbs"], 4), "traffic": traffic,
                     "peak_kind": "measured in this run (gather_peak: ns_gather_probe on the same table)",
                     "figure": "hash-table gather bytes (blended samples x 16 levels x 8 corners x 4 B fp16 "
                               "pair) per blend launch time, against the gather rate of a lookup-only kernel "
                               "with the blend's point pattern (gather_peak.coherent); the launch's DRAM "
                               "traffic is far below HBM (dram_figure)",
                     "gather_peak": gpeak,
                     "dram_figure": {"achieved": round(achieved, 1), "algorithmic_bytes": int(blend_bytes),
                                     "peak": hbm_peak, "peak_kind": peak_kind,
                                     "frac": round(achieved / hbm_peak, 4)},
                     "gather_figure_vs_hbm": round(gather_gbs / hbm_peak, 4),
                     "hash_gather_tbs": round(gather_tbs, 3)},
        "e2e": {"value": round(world * mpix * 1000.0 / e2e_ms_step, 3), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms_step, 4),
                "timing": "one device-timed sequence of `steps` frames through FramePipeline "
                          "(one CUDA graph per frame at N=1), L2 flushed before every frame on the compute "
                          "stream; at N=1 the flushes' own event-timed duration is taken out, at N>1 (the "
                          "next frame's exchange runs during a flush) it stays in",
                "flush_ms_per_step": round(e2e_flush_ms / args.steps, 4)},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if world == 1:
        line["rvq_decode"]["gpu_sizes"] = rvq_timing(dev, hbm_peak)
        if not args.no_config1:
            line["config1"] = config1_timing(dev)
    if exchange is not None:
        line["rvq_exchange"] = exchange
    if identical is not None:
        line["frame_bit_identical"] = identical
    if graph is not None:
        line["graph_frame"] = graph
    if not args.no_train:
        line["train_step"] = train_step_timing(sc, cam, dev, steps=min(args.steps, 10))
    if not args.no_multiview:
        del fr
        torch.cuda.empty_cache()
        line["multiview"] = multiview_timing(world, rank, dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(sc, budget_s=args.cpu_budget)
        line["rvq_decode"]["cpu_config0"] = rvq_cpu_timing()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def graph_timing(fr, cam, view, proj, flush, steps):
    """The same frame as one CUDA-graph launch (FrameGraph: device-side instance
    count, no host sync inside the frame), timed like the value line."""
    import torch

    from nest_b200.frame import FrameGraph
    fg = FrameGraph(fr, cam, view, proj)
    for _ in range(3):
        fg.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in ev:
        flush_l2(flush)
        s.record()
        fg.replay()
        e.record()
    torch.cuda.synchronize()
    status = fg.status()
    ms = sum(s.elapsed_time(e) for s, e in ev) / steps
    mpix = cam.width * cam.height / 1e6
    return {"ms_per_step": round(ms, 4), "value": round(mpix * 1000.0 / ms, 3), "unit": UNIT,
            "device_status": int(status),
            "note": "one graph launch per frame (decode, preprocess, binning with the device-side count, "
                    "blend, MLP); L2 flushed between frames"}


def exchange_timing(shard, codebooks, dev, P, stages, dims, iters=20):
    """N > 1: the specified exchange (decode this rank's rows, all-gather the
    decoded attributes) against all-gathering the RVQ indices and decoding every
    row on every rank. Device time per exchange, max over ranks; both leave the
    same rows in the frame's attribute buffer."""
    import torch
    import torch.distributed as dist

    from nest_b200 import raster
    from nest_b200.views import DecodeShard
    out = {}
    world = shard.world
    full = DecodeShard.create(shard.idx_shard.new_zeros((P, shard.idx_shard.shape[1])), dims, world, shard.rank)
    full.idx_shard.copy_(shard.idx_shard)
    for name, fn in (("attributes", lambda: shard.decode_and_gather(codebooks, raster.rvq_decode)),
                     ("attributes_all_columns", lambda: full.decode_and_gather(codebooks, raster.rvq_decode)),
                     ("indices", lambda: shard.gather_indices_and_decode(codebooks, raster.rvq_decode))):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[f"{name}_ms"] = round(float(t.item()), 4)
    out["received_bytes_per_rank"] = {"attributes": int(P * (world - 1) / world) * 4 * shard.columns,
                                      "attributes_all_columns": int(P * (world - 1) / world) * 4 * dims,
                                      "indices": int(P * (world - 1) / world) * stages}
    out["note"] = (f"attributes: decode all {dims} columns of this rank's rows + NCCL all-gather of the "
                   f"{shard.columns} fp32 columns the rasterizer reads (the frame's path); "
                   "attributes_all_columns: the same exchange of every column; "
                   "indices: NCCL all-gather of uint8 indices + decode of all rows on every rank")
    del full
    return out


def frame_identity(fr, shard, cam, view, proj, dev):
    """N > 1 correctness: this rank's frame rendered from the all-gathered
    attribute rows (decode sharded over the ranks) against the same frame from
    a full decode on this rank alone; true when rgb, features and the 14 aux
    channels are bit-identical on every rank."""
    import torch
    import torch.distributed as dist

    from nest_b200 import raster
    shard.decode_and_gather(fr.codebooks, raster.rvq_decode)
    fr.decoded = shard.decoded
    fr.render(cam, view, proj, skip_decode=True)
    sharded = [fr.rgb.clone(), fr.features.clone(), fr.others.clone()]
    fr.decoded = torch.empty((fr.P, fr.dims), dtype=torch.float32, device=dev)
    fr.render(cam, view, proj)  # decodes all rows locally
    local = [fr.rgb, fr.features, fr.others]
    same = all(torch.equal(a, b) for a, b in zip(sharded, local))
    flag = torch.tensor([1 if same else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def oracle_frame(sc, row_stride, threads=None):
    """One frame of the CPU oracle on a bounded sample (tile rows ty % row_stride == 0).
    Returns (seconds, sampled pixels)."""
    import numpy as np
    import torch

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import api_inputs, raw_attributes
    from oracle import oracle

    t0 = time.perf_counter()
    dec = torch.from_numpy(oracle.rvq_decode_c(sc.rvq_idx.numpy(), sc.codebooks.numpy()))
    inp = api_inputs(sc, raw_attributes(sc, dec))
    g, cam = sc.grid, sc.camera
    pre = oracle.preprocess(inp["means3D"].numpy(), inp["scales"].numpy(), inp["rotations"].numpy(),
                            inp["opacities"].numpy(), cam.world_view_transform.numpy(),
                            cam.full_proj_transform.numpy(), cam.width, cam.height)
    keys, vals, ranges = oracle.bin_surfels(pre, cam.width, cam.height)
    out = oracle.render(pre, vals, ranges, inp["homotrans"].numpy(), inp["ap_level"].numpy(), g.table.float().numpy(),
                        g.offsets.numpy(), g.gridrange.numpy(), cam.width, cam.height, g.channels, g.level_dim,
                        g.levels, g.S, g.base_resolution, row_stride=row_stride)
    rows = [ty for ty in range((cam.height + 15) // 16) if ty % row_stride == 0]
    ys = np.concatenate([np.arange(ty * 16, min(cam.height, ty * 16 + 16)) for ty in rows])
    oracle.mlp_oracle(out["out_color"][:, ys, :], sc.mlp, out["out_others"][1][ys, :])
    dt = time.perf_counter() - t0
    return dt, len(ys) * cam.width


def cpu_baseline(sc, budget_s=30.0, row_stride=4):
    from oracle import oracle
    threads = oracle.set_num_threads(os.cpu_count() or 1)
    dt, px = oracle_frame(sc, row_stride)
    return {"value": round(px / dt / 1e6, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one config-2 frame on the CPU oracle (C++/OpenMP restatement): full RVQ decode, "
                      f"preprocess, binning and sort of all 1M surfels, blend + MLP of every "
                      f"{row_stride}th tile row ({px} px); value = sampled px / wall time",
            "seconds": round(dt, 2)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from nest_b200 import synth
    from oracle import oracle
    sc = synth.config2()
    # every host core, whatever the launcher set (torchrun exports OMP_NUM_THREADS=1)
    threads = oracle.set_num_threads(os.cpu_count() or 1)
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    # Bounded sample: choose the tile-row stride so that warmup + steps fit ~3 minutes.
    stride = 4
    dt, px = oracle_frame(sc, stride)
    total = dt * (args.steps + max(args.warmup, 1))
    while total > 180 and stride < 64:
        stride *= 2
        dt, px = oracle_frame(sc, stride)
        total = dt * (args.steps + max(args.warmup, 1))
    for _ in range(max(args.warmup - 1, 0)):
        oracle_frame(sc, stride)
    times = []
    for _ in range(args.steps):
        dt, px = oracle_frame(sc, stride)
        times.append(dt)
    ms = 1000.0 * sum(times) / len(times)
    value = px / (ms * 1e-3) / 1e6
    sample = (f"CPU oracle (C++/OpenMP restatement of the reference path; the reference CUDA rasterizer "
              f"is unbuildable here: glm absent) per step: full RVQ decode + preprocess + sort of 1M "
              f"surfels, blend + MLP of every {stride}th tile row ({px} px)")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded config-2 scene)",
            "config": {"workload": WORKLOAD, "sample_row_stride": stride},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def multiview_timing(world, rank, dev, batches=2):
    """benchmark config 3: a 64-view batch (1920x1080, 3M RVQ surfels, elevation
    20 deg, azimuth 360 i / 64) split over the ranks by camera. Per batch: the
    surfel-sharded RVQ decode and its all-gather once, then this rank's views.
    Time per batch = max over ranks (CUDA events), strong scaling in the ranks."""
    import torch
    import torch.distributed as dist

    from nest_b200 import raster, synth
    from nest_b200.frame import FrameRenderer
    from nest_b200.views import DecodeShard, camera_share

    sc = synth.config3()
    cams = synth.config3_cameras()
    mine = camera_share(len(cams), world, rank)
    fr = FrameRenderer(sc, device=dev, capacity=24_000_000)
    if world > 1:
        shard = DecodeShard.create(fr.rvq_idx, fr.dims, world, rank, columns=synth.BASE_DIMS)
        fr.decoded = shard.decoded
    views = [(cams[i], cams[i].world_view_transform.to(dev).contiguous(),
              cams[i].full_proj_transform.to(dev).contiguous()) for i in mine]

    def batch():
        if world > 1:
            shard.decode_and_gather(fr.codebooks, raster.rvq_decode)
        for k, (cam, v, pr) in enumerate(views):
            fr.render(cam, v, pr, skip_decode=world > 1 or k > 0)

    batch()  # warm-up; sizes the binning capacity
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(batches)]
    for s, e in evs:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        batch()
        e.record()
        torch.cuda.synchronize()
    ms = [s.elapsed_time(e) for s, e in evs]
    t = torch.tensor(ms, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.tolist()
    batch_ms = statistics.median(ms)
    W, H = cams[0].width, cams[0].height
    out = {"workload": "config 3: 3M RVQ surfels, 64 views 1920x1080 per batch, decode + all-gather once "
                       "per batch, views split over the ranks",
           "views": len(cams), "views_per_rank_max": -(-len(cams) // world), "batches": batches,
           "ms_per_batch": round(batch_ms, 3), "views_per_s": round(len(cams) * 1000.0 / batch_ms, 3),
           "mpix_per_s": round(len(cams) * W * H / 1e6 * 1000.0 / batch_ms, 3),
           "instances_last_view": fr.num_rendered}
    del fr
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-train", action="store_true", help="skip the config-4 training-step timing")
    ap.add_argument("--no-multiview", action="store_true", help="skip the config-3 64-view batch timing")
    ap.add_argument("--cpu-budget", type=float, default=30.0)
    ap.add_argument("--no-config1", action="store_true", help="skip the config-1 single-view timing")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
