"""Benchmark of the CubicSplat render/optimise hot path on B200.

Metric: fwd+bwd training iterations/s at 768x512 with 512
closed cubic paths x 4 segments, S=16 (config 2): each step renders, computes
MSE and SSIM (11x11, sigma 1.5), back-propagates and takes an Adam step
(lr 0.5 on points, 0.01 on colours).

  value  -- device-resident throughput of the fused B200 step (one CUDA graph
            per step, inputs already in HBM), timed per step with CUDA events;
  e2e    -- the same step through the drop-in ``manbo`` API a user calls, with
            the target image copied from pinned host memory and the loss read
            back every step, inside the timed region.
L2 is flushed (256 MiB write) before every timed step, outside its events.

Multi-GPU (torchrun, N>1): every rank optimises its own config-2 scene
(different seed), no collective on the data path; value = all ranks'
iterations / max over ranks of the device time ("scaling": "weak").  At every
N the line also carries ``strong_config3``: the config-3 image split across
the N ranks in tile-row bands (below), the strong-scaling curve.

--workload config3: one 2040x1356 image with 4096 closed paths x 6 segments
split across the ranks in tile-row bands balanced by per-row work; every step
sums the ranks' gradients (with the bands' SSIM sums) and takes the Adam step
in one kernel that reads every rank's gradient buffer through NVLink peer
memory, and each band reads the next band's first 10 rows for the SSIM window
the same way (repo_b200/peer.py; --collective nccl uses an NCCL all-reduce and
all-gather instead); value = iterations of the one image / max device time
("scaling": "strong").

--workload config4: stroke mode, 1024x1024, 2048 open one-segment cubics
(width U[1,4] px, S=16) through the drop-in manbo API: forward + MSE + backward
+ Adam per step (the API binds each frame with one host synchronisation).
--workload config5: the batched sweep, one 768x512 scene per rank, paths in
{256, 1024, 4096, 16384} x S in {4, 8, 16, 32}, the fused step (with SSIM)
at every point, plus standalone MSE and SSIM kernel bandwidth; one JSON line
per point.

--impl reference times the reference algorithm's CPU implementation (the C
oracle restating manbo/ops/cubic_splatting.py, all host threads) on the same
workload; the reference has no CPU renderer of its own.

Diagnostics (one GPU): --workload config3 --band K/N runs band K of the
N-way tile-row split alone (no exchange, no SSIM: the per-band compute of an
N-GPU step); --host-profile splits the drop-in API step's host time by phase
and lists its device kernels (torch profiler).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd iters/s at 768x512, 512 paths"
UNIT = "iters/s"
E2E_MIN_WARMUP = 25
KERNEL_TIMING_REPS = 200
WORKLOAD_CONFIG2 = ("config2: 768x512 RGB, 512 closed cubic paths x 4 segs, S=16, "
                    "fwd+MSE+SSIM+bwd+Adam (lr 0.5 pts / 0.01 colours)")
L2_FLUSH_BYTES = 256 << 20
FP32_PEAK_TFLOPS = round(148 * 128 * 2 * 1965e6 / 1e12, 2)  # SIMT FMA peak at the max SM clock


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "config3", "config4", "config5"])
    ap.add_argument("--no-gpu-reference", action="store_true")
    ap.add_argument("--collective", default="peer", choices=["peer", "nccl"],
                    help="band exchange of the config-3 step: peer-memory kernels or NCCL")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the config-3 strong-scaling step of the default workload")
    ap.add_argument("--host-profile", action="store_true",
                    help="config 2 on one GPU: host time per phase of the drop-in API step and "
                         "its device kernels (torch profiler); one JSON line")
    ap.add_argument("--band", default=None, metavar="K/N",
                    help="config3 on one GPU: only band K of the N-way tile-row split, no "
                         "exchange and no SSIM (the per-band compute of an N-GPU step)")
    ap.add_argument("--gpu-reference-child", action="store_true", help=argparse.SUPPRESS)
    return ap.parse_args(argv)


# --------------------------------------------------------------------------
# clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"cs_clocks_{os.getpid()}_{gpu_index}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu_index)], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------
# B200 arm

def time_steps(step_fn, steps, flush, stream):
    import torch
    durs = []
    for _ in range(steps):
        flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step_fn()
        e.record(stream)
        durs.append((s, e))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in durs]


def time_device_calls(fn, reps, flush, stream):
    """Device time of `fn`'s launches alone: all reps (L2 flush, event, fn,
    event) are queued behind a sleep kernel, so host launch overhead does not
    show up between the events."""
    import torch
    torch.cuda.synchronize()
    torch.cuda._sleep(int(4e6))  # a few ms of queue lead for the host
    evs = []
    for _ in range(reps):
        flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        evs.append((s, e))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def graph_kernel_times(tr, reps, flush):
    """Mean CUDA-event durations of the forward and backward raster launches
    over `reps` replays of the captured step (events recorded inside the
    graph around the two launches, read after each replay)."""
    import torch
    fwd, bwd = [], []
    for _ in range(reps):
        flush()
        tr.step()
        f, b = tr.kernel_times()
        fwd.append(f)
        bwd.append(b)
    torch.cuda.synchronize()
    return statistics.mean(fwd), statistics.mean(bwd)


def raster_work(tr):
    """Pixel-edge pairs and pixel-intersect visits of the reference algorithm
    for the current state: every pixel visits the intersects of its tile up to
    its stop (forward: where T fell below 1e-4, else the tile's end; backward:
    final_idx) and evaluates every edge of each visited primitive
    (manbo/ops/cubic_splatting.py:1095-1134, :1451-1501).  Computed on the
    host from tile_bins, per-intersect edge counts and the forward outputs."""
    import numpy as np
    n = int(tr.counters[0].item())
    bins = tr.tile_bins.cpu().numpy()
    pids = tr.prim_sorted[:n].cpu().numpy()
    eoffs = tr.edge_offs.cpu().numpy()
    ne = (eoffs[pids + 1] - eoffs[pids]).astype(np.int64)
    cum = np.concatenate([[0], np.cumsum(ne)])
    fidx = tr.fidx.cpu().numpy().astype(np.int64)
    fts = tr.fts.cpu().numpy()
    h, w = tr.h, tr.w
    ty = np.arange(h)[:, None] // 16
    tx = np.arange(w)[None, :] // 16
    tile = ty * tr.tbx + tx
    start = bins[tile, 0].astype(np.int64)
    end = bins[tile, 1].astype(np.int64)
    has = end > start
    stop = np.where(fts <= 1e-4, fidx, end - 1)
    pe_fwd = np.where(has, cum[np.clip(stop + 1, 0, n)] - cum[start], 0).sum()
    vis_fwd = np.where(has, stop + 1 - start, 0).sum()
    valid_b = has & (fidx >= start)
    pe_bwd = np.where(valid_b, cum[np.clip(fidx + 1, 0, n)] - cum[start], 0).sum()
    vis_bwd = np.where(valid_b, fidx + 1 - start, 0).sum()
    return int(pe_fwd), int(vis_fwd), int(pe_bwd), int(vis_bwd), n


def executed_work(bins, istrips, rowoff, imeta, fidx, fts, h, w, tbx, n, visits=None,
                  winner_codes=False):
    """Pixel-edge pairs and pixel-intersect visits the B200 raster kernels
    evaluate, as opposed to the reference algorithm's (raster_work): a warp
    runs a 4x16-pixel strip, so every staged near-edge record of a walked
    intersect costs 64 pixel-edge pairs and every intersect that can change
    the strip (near records, or a fill row the far-edge offsets put inside)
    costs 64 pixel visits.  The forward walks a strip's intersects until all
    of its pixels have T <= 1e-4 (else to the tile's end), the backward from
    the strip's largest final_idx down -- or, given the forward's visit lists,
    only the listed intersects, and with the fill forward's winner codes only
    each pixel's closest record of a listed intersect (one pair per pixel and
    visit).  Intersects that cannot change the strip are skipped in batches
    and counted as free."""
    import numpy as np
    if n == 0:
        return 0, 0, 0, 0
    rec = istrips[:n, :, 1].astype(np.int64)                      # [n, 4]
    act = rec > 0
    if rowoff is not None:
        ro = rowoff[:n].reshape(n, 4, 4)
        wind = (ro & 0xFFFF).astype(np.int16).astype(np.int32)
        cnt = (ro.view(np.uint32) >> 16).astype(np.int32)
        rule = imeta[:n, 3][:, None, None]
        inside = np.where(rule == 0, (cnt & 1) != 0, wind != 0)
        act |= inside.any(axis=2)
    crec = np.vstack([np.zeros((1, 4), np.int64), np.cumsum(rec, axis=0)])
    cact = np.vstack([np.zeros((1, 4), np.int64), np.cumsum(act, axis=0)])
    tby = (h + 15) // 16
    hp, wp = tby * 16, tbx * 16
    fi = np.full((hp, wp), -1, np.int64)
    fi[:h, :w] = fidx.reshape(h, w)
    done = np.ones((hp, wp), bool)
    done[:h, :w] = fts.reshape(h, w) <= 1e-4
    # [tby, 4 strips, 4 rows, tbx, 16 cols] -> per strip
    fmax = fi.reshape(tby, 4, 4, tbx, 16).max(axis=(2, 4))        # [tby, 4, tbx]
    alld = done.reshape(tby, 4, 4, tbx, 16).all(axis=(2, 4))
    rs = bins[:, 0].astype(np.int64).reshape(tby, 1, tbx)
    re = bins[:, 1].astype(np.int64).reshape(tby, 1, tbx)
    st = np.arange(4).reshape(1, 4, 1)
    has = re > rs
    kf = np.where(alld, np.minimum(fmax, re - 1), re - 1)
    kb = np.minimum(fmax, re - 1)
    okf = has & (kf >= rs)
    okb = has & (kb >= rs)

    def span(c, k, ok):
        hi = np.clip(k + 1, 0, n)
        lo = np.clip(rs, 0, n)
        return np.where(ok, c[hi, st] - c[lo, st], 0).sum()

    pe_f, vis_f = 64 * int(span(crec, kf, okf)), 64 * int(span(cact, kf, okf))
    if visits is None:
        return pe_f, vis_f, 64 * int(span(crec, kb, okb)), 64 * int(span(cact, kb, okb))
    pe_b = vis_b = 0
    for t in np.nonzero(bins[:, 1] > bins[:, 0])[0]:
        t_rs, t_re = int(bins[t, 0]), int(bins[t, 1])
        for s_ in range(4):
            base = 4 * (t_rs + int(t)) + s_ * (t_re - t_rs + 1)
            cnt = int(visits[base])
            ids = visits[base + 1: base + 1 + cnt]
            pe_b += cnt if winner_codes else int(rec[ids, s_].sum())
            vis_b += cnt
    return pe_f, vis_f, 64 * pe_b, 64 * vis_b


def executed_roofline(flop_b, t_b, flop_f, t_f, peak):
    """The raster kernels against the FP32 peak on the work they evaluate
    (executed_work), beside the reference-algorithm figures: above 1.0 on the
    reference work means the culled pairs were never computed, this one
    measures how well the evaluated pairs use the SIMT pipes."""
    a_b = flop_b / (t_b * 1e-3) / 1e12
    a_f = flop_f / (t_f * 1e-3) / 1e12
    return {"flop_per_launch": int(flop_b), "achieved": round(a_b, 3), "frac": round(a_b / peak, 4),
            "forward": {"flop_per_launch": int(flop_f), "achieved": round(a_f, 3),
                        "frac": round(a_f / peak, 4)},
            "model": "same FLOP per pair and per visit, counted over what the kernels evaluate: "
                     "64 pixels x staged near-edge records of walked intersects, 64 pixels x "
                     "intersects that can change the strip (backward: the forward's visit "
                     "lists; for fills one record per pixel and listed visit, the winner "
                     "code's)"}


def ncu_traffic(kernel: str, summary: str = "raster_fill_config2.md"):
    """DRAM bytes (read + write) per launch of `kernel` from a committed ncu
    summary under profiles/ (default: the config-2 raster kernels), or None
    when the summary is absent."""
    path = os.path.join(ROOT, "profiles", summary)
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and parts[0] == "traffic_bytes" and parts[1] == kernel:
                    return int(parts[2])
    except OSError:
        pass
    return None


def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from repo_b200 import scenes
    from repo_b200.train import FillTrainer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    scene = scenes.config2() if rank == 0 else scenes.circles_scene(1 + 7919 * rank, 512, 768,
                                                                     512, 4, 16, 32)
    flush_buf = torch.empty((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    def barrier():
        if world > 1:
            dist.barrier()

    tr = FillTrainer(scene, dev, lr_points=0.5, lr_colors=0.01, with_ssim=True)
    tr.capture(warmup=max(3, args.warmup))
    # a second capture of the same step with timing events around the two
    # raster launches, for the kernel times (the timed graph has none)
    timed = FillTrainer(scene, dev, lr_points=0.5, lr_colors=0.01, with_ssim=True,
                        capacity=(tr.capacity, tr.dcapacity))
    timed.enable_kernel_timing()
    timed.capture(warmup=3)
    for _ in range(args.warmup):
        tr.step()
    torch.cuda.synchronize()
    gpu_index = int(os.environ.get("LOCAL_RANK", "0"))
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        try:
            gpu_index = int(visible.split(",")[local_rank])
        except ValueError:
            pass
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_index) as clk:
        t0 = time.perf_counter()
        durs = time_steps(tr.step, args.steps, flush, stream)
        wall = time.perf_counter() - t0
        # the dominant kernels, timed live with CUDA events on their stream
        # inside graph-replayed steps (one synchronisation per replay)
        t_fwd, t_bwd = graph_kernel_times(timed, KERNEL_TIMING_REPS, flush)
    barrier()
    torch.cuda.synchronize()
    n_isect, status = tr.check_status()
    if status != 0:
        raise RuntimeError(f"device status {status} (intersect capacity {tr.capacity}, needed {n_isect})")
    total_ms = sum(durs)
    t_max = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    total_ms = float(t_max.item())
    value = world * args.steps / (total_ms / 1e3)
    loss_final, ssim_final = tr.loss_value(), tr.ssim_value()

    # work of the kernel-timing trainer's last step (its state tracks the timed one's)
    tk = timed
    pe_fwd, vis_fwd, pe_bwd, vis_bwd, n_now = raster_work(tk)
    xe_fwd, xv_fwd, xe_bwd, xv_bwd = executed_work(
        tk.tile_bins.cpu().numpy(), tk.istrips.cpu().numpy(), tk.rowoff.cpu().numpy(),
        tk.imeta.cpu().numpy(), tk.fidx.cpu().numpy(), tk.fts.cpu().numpy(), tk.h, tk.w, tk.tbx,
        n_now, tk.visits.cpu().numpy(), winner_codes=True)
    timed.release_graphs()

    # e2e through the drop-in API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(scene, dev, args, flush, stream, world)

    result = None
    if rank == 0:
        clocks = clk.summary()
        sm_mhz = clocks.get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12   # TFLOP/s at the sampled clock
        flop_bwd = 24 * pe_bwd + 30 * vis_bwd
        flop_fwd = 20 * pe_fwd + 12 * vis_fwd
        achieved_bwd = flop_bwd / (t_bwd * 1e-3) / 1e12
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD_CONFIG2,
                       "scene": "seed-1 value noise + 32 ellipses target, circles r 5-40 px",
                       "parallelism": f"one scene per rank x{world}" if world > 1 else "single GPU",
                       "l2": "flushed before every step (256 MiB write), outside the step events",
                       "step": "one CUDA graph of the fused B200 step",
                       "intersects": n_now, "intersect_capacity": tr.capacity,
                       "staged_record_capacity": tr.dcapacity},
            "final_loss": loss_final, "final_ssim": ssim_final,
            "gpu_launches": args.steps * tr.launches_per_step,
            "wall_s_timed_region": round(wall, 4),
            "clocks": clocks,
            "roofline": {
                "kernel": "raster_backward (fill)", "bound": "fp32",
                "achieved": round(achieved_bwd, 3), "peak": round(fp32_peak, 2),
                "unit": "TFLOP/s", "frac": round(achieved_bwd / fp32_peak, 4),
                "traffic": ncu_traffic("raster_backward_kernel"),
                "traffic_note": "dram read+write bytes per launch from one ncu capture of "
                                "the same workload (profiles/raster_fill_config2.md)",
                "peak_note": "SIMT FP32 FMA peak 148 SM x 128 lanes x 2 at the sampled median SM "
                             "clock; MEASURED_PEAKS.json holds only HBM and bf16 tensor peaks",
                "flop_per_launch": flop_bwd,
                "flop_model": "reference-algorithm work: 24 FLOP per pixel-edge pair up to "
                              "final_idx + 30 per pixel-intersect visit",
                "launch_ms": round(t_bwd, 4),
                "forward": {"launch_ms": round(t_fwd, 4), "flop_per_launch": flop_fwd,
                            "achieved": round(flop_fwd / (t_fwd * 1e-3) / 1e12, 3)},
                "executed": executed_roofline(24 * xe_bwd + 30 * xv_bwd, t_bwd,
                                              20 * xe_fwd + 12 * xv_fwd, t_fwd, fp32_peak),
            },
        }
        if e2e is not None:
            result["e2e"] = e2e
    return result, tr


def parse_band(spec: str):
    """`--band K/N` -> (K, N): band K (0-based) of an N-way split."""
    try:
        k, n = (int(v) for v in spec.split("/"))
    except ValueError:
        raise ValueError(f"--band {spec}: expected K/N, e.g. 3/8") from None
    if n < 1 or not 0 <= k < n:
        raise ValueError(f"--band {spec}: K must be in [0, N) and N >= 1")
    return k, n


def run_bands(args, rank, world, local_rank):
    """Config 3: one large image across the ranks in tile-row bands."""
    import torch
    import torch.distributed as dist

    from repo_b200 import bands, scenes
    from repo_b200.train import FillTrainer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    scene = scenes.config3()
    nb, bi = world, rank
    if args.band and world == 1 and args.workload == "config3":
        bi, nb = parse_band(args.band)
    split = bands.balanced_bands(bands.tile_row_work(scene, dev), nb)
    band = split[bi]
    collective = "none"
    kw = {}
    if world > 1 and args.collective == "peer":
        # gradient exchange + Adam in one kernel and the SSIM halo read over
        # NVLink peer memory (repo_b200/peer.py)
        kw = dict(peer_group=dist.group.WORLD)
        collective = "peer memory: fused all-reduce + Adam, halo by peer read"
    elif world > 1:
        kw = dict(grad_hook=bands.allreduce_hook(), halo_gather=bands.allgather_halo(rank, world))
        collective = "NCCL all-reduce + all-gather"
    one_band = nb > 1 and world == 1
    tr = FillTrainer(scene, dev, lr_points=0.5, lr_colors=0.01, with_ssim=not one_band,
                     tile_rows=band if nb > 1 else None, **kw)
    flush_buf = torch.empty((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    tr.capture(warmup=max(3, args.warmup))
    for _ in range(args.warmup):
        tr.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    gpu_index = local_rank
    with ClockSampler(gpu_index) as clk:
        durs = time_steps(tr.step, args.steps, flush, stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    _, status = tr.check_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")
    t_max = torch.tensor([sum(durs)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    total_ms = float(t_max.item())
    result = None
    if rank == 0:
        if one_band:
            collective = f"none: band {bi} of {nb} alone (rows {band}), no SSIM"
        result = {
            "metric": "fwd+bwd iters/s at 2040x1356, 4096 paths (tile-row bands)",
            "value": round(args.steps / (total_ms / 1e3), 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config3: 2040x1356 RGB, 4096 closed cubic paths x 6 segs, "
                                   "S=16, fwd+MSE+SSIM+bwd+Adam, one all-reduce of gradients "
                                   "and SSIM sums per step (SSIM halo rows by all-gather)",
                       "bands": split, "parallelism": f"tile-row bands x{world}",
                       "collective": collective,
                       "l2": "flushed before every step (256 MiB write), outside the step events"},
            "final_loss": tr.loss_value(), "final_ssim": tr.ssim_value(),
            "gpu_launches": args.steps * tr.launches_per_step,
            "clocks": clk.summary(),
        }
        if one_band:
            result["metric"] = ("config-3 band step on one GPU: band K of an N-way tile-row split "
                                "alone, no exchange, no SSIM (diagnostic)")
            result["band"] = {"index": bi, "of": nb, "tile_rows": list(band)}
    return result, tr


def binning_work(b, fts, fidx, h, w):
    """Reference-algorithm pixel-edge pairs and pixel-intersect visits of a
    rendered frame (as raster_work), from a Binning and the forward outputs."""
    import numpy as np
    n = int(b.num_intersects)
    bins = b.tile_bins.cpu().numpy()
    pids = b.prim_ids_sorted[:n].cpu().numpy()
    eoffs = b.prim_edge_offsets.cpu().numpy()
    ne = (eoffs[pids + 1] - eoffs[pids]).astype(np.int64)
    cum = np.concatenate([[0], np.cumsum(ne)])
    fidx = fidx.cpu().numpy().astype(np.int64)
    fts = fts.cpu().numpy()
    tbx = b.tile_bounds[0]
    tile = (np.arange(h)[:, None] // 16) * tbx + np.arange(w)[None, :] // 16
    start = bins[tile, 0].astype(np.int64)
    end = bins[tile, 1].astype(np.int64)
    has = end > start
    stop = np.where(fts <= 1e-4, fidx, end - 1)
    pe_fwd = np.where(has, cum[np.clip(stop + 1, 0, n)] - cum[start], 0).sum()
    vis_fwd = np.where(has, stop + 1 - start, 0).sum()
    valid_b = has & (fidx >= start)
    pe_bwd = np.where(valid_b, cum[np.clip(fidx + 1, 0, n)] - cum[start], 0).sum()
    vis_bwd = np.where(valid_b, fidx + 1 - start, 0).sum()
    return int(pe_fwd), int(vis_fwd), int(pe_bwd), int(vis_bwd)


def run_stroke(args, rank, world, local_rank):
    """Config 4: stroke mode through the manbo API (forward, MSE, backward, Adam)."""
    import torch

    import manbo
    from repo_b200 import render, scenes

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sc = scenes.config4(seed=3 + rank)
    h, w, p = sc.height, sc.width, int(sc.cubics_px.shape[0])
    cn = scenes.px_to_norm(sc.cubics_px, w, h).to(dev).requires_grad_(True)
    colors = sc.colors.to(dev).clone().requires_grad_(True)
    widths = sc.stroke_widths.to(dev).clone().requires_grad_(True)
    opac, depths = sc.opacities.to(dev), sc.depths.to(dev)
    aa, bg = sc.aa_widths.to(dev), sc.background.to(dev)
    offs = torch.arange(p + 1, dtype=torch.int32, device=dev)
    target = sc.target.to(dev)
    opt = torch.optim.Adam([{"params": [cn], "lr": 1e-3},
                            {"params": [colors, widths], "lr": 0.01}], fused=True)
    flush_buf = torch.empty((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    def step():
        opt.zero_grad(set_to_none=True)
        out = manbo.ops.render_cubic_polyline_splat_tilelang(
            cn, offs, colors, opac, widths, depths, h, w, 16, 16, bg, aa_widths=aa,
            distance_samples=sc.samples)
        img = torch.clamp(out, 0, 1).permute(2, 0, 1).unsqueeze(0).contiguous()
        loss = manbo.mse_loss_tilelang(img, target)
        loss.backward()
        opt.step()
        return loss

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    with ClockSampler(local_rank) as clk:
        durs = time_steps(step, args.steps, flush, stream)
    total_ms = sum(durs)
    with torch.no_grad():  # reference-algorithm work of the current state
        wd = torch.clamp(aa, min=1e-4)
        b = render.bin_primitives(cn.detach(), offs, depths, wd, h, w, sc.samples,
                                  colors=colors.detach(), opacities=opac,
                                  inv_sigma2s=render._inv_sigma2(wd), stroke_widths=widths.detach())
        _, fts, fidx = render.forward_raster(b, bg, h, w)
        pe_f, vis_f, pe_b, vis_b = binning_work(b, fts, fidx, h, w)
        xe_f, xv_f, xe_b, xv_b = executed_work(
            b.tile_bins.cpu().numpy(), b.isect_strips.cpu().numpy(), None, b.imeta.cpu().numpy(),
            fidx.cpu().numpy(), fts.cpu().numpy(), h, w, b.tile_bounds[0], int(b.num_intersects),
            b.visit_lists.cpu().numpy())
        # the two stroke raster kernels on this frame, timed with CUDA events on
        # their stream (launches queued behind a sleep, so host work is hidden;
        # the backward's time includes zeroing its gradient buffers)
        v_out = scenes.seeded_grad(7, h, w).to(dev)
        t_fwd = statistics.median(time_device_calls(
            lambda: render.forward_raster(b, bg, h, w), 20, flush, stream))
        t_bwd = statistics.median(time_device_calls(
            lambda: render.raster_backward(b, p, bg, fts, fidx, v_out, h, w), 20, flush, stream))
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    if rank != 0:
        return None
    clocks = clk.summary()
    peak = 148 * 128 * 2 * (clocks.get("sm_mhz") or 1965.0) * 1e6 / 1e12
    flop_b = 18 * pe_b + 30 * vis_b
    flop_f = 14 * pe_f + 12 * vis_f
    return {
        "metric": "stroke fwd+bwd iters/s at 1024x1024, 2048 strokes (manbo API)",
        "value": round(world * args.steps / (total_ms / 1e3), 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config4: 1024x1024 RGB target of 256 lines, 2048 open cubic "
                               "strokes (1 segment), width U[1,4], S=16, fwd+MSE+bwd+Adam "
                               "through manbo.ops.render_cubic_polyline_splat_tilelang",
                   "l2": "flushed before every step (256 MiB write), outside the step events"},
        "clocks": clocks,
        "roofline": {"kernel": "raster_backward (stroke)", "bound": "fp32",
                     "traffic": ncu_traffic("raster_backward_kernel", "raster_stroke_config4.md"),
                     "traffic_note": "dram read+write bytes per launch from one ncu capture "
                                     "(profiles/raster_stroke_config4.md)",
                     "achieved": round(flop_b / (t_bwd * 1e-3) / 1e12, 3),
                     "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(flop_b / (t_bwd * 1e-3) / 1e12 / peak, 4),
                     "flop_model": "reference-algorithm work: 18 FLOP per pixel-edge pair up to "
                                   "final_idx + 30 per pixel-intersect visit",
                     "launch_ms": round(t_bwd, 4),
                     "forward": {"launch_ms": round(t_fwd, 4),
                                 "achieved": round(flop_f / (t_fwd * 1e-3) / 1e12, 3)},
                     "executed": executed_roofline(18 * xe_b + 30 * xv_b, t_bwd,
                                                   14 * xe_f + 12 * xv_f, t_fwd, peak)},
    }


def run_sweep(args, rank, world, local_rank):
    """Config 5: path-count x samples sweep of the fused step, one scene per
    rank, and standalone MSE / SSIM kernel bandwidth.  Yields JSON lines."""
    import json as _json

    import torch
    import torch.distributed as dist

    from repo_b200 import metric as mt
    from repo_b200 import scenes
    from repo_b200.train import FillTrainer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    lines = []
    steps = max(10, args.steps // 4)
    for paths in (256, 1024, 4096, 16384):
        for samples in (4, 8, 16, 32):
            tr = FillTrainer(scenes.config5(rank, paths, samples), dev)
            tr.capture(warmup=3)
            for _ in range(max(3, args.warmup)):
                tr.step()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            durs = time_steps(tr.step, steps, flush, stream)
            t = torch.tensor([sum(durs)], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            n_isect, status = tr.check_status()
            lines.append({"metric": "fwd+bwd iters/s at 768x512 (config 5 sweep)",
                          "value": round(world * steps / (float(t.item()) / 1e3), 3),
                          "unit": UNIT, "n_gpus": world, "steps": steps,
                          "ms_per_step": round(float(t.item()) / steps, 4),
                          "higher_is_better": True, "scaling": "weak", "dtype": "f32",
                          "data": "synthetic",
                          "config": {"workload": "config5", "paths": paths, "samples": samples,
                                     "intersects": n_isect, "status": status}})
            del tr
    # standalone metric kernels: one 768x512 RGB pair (9.4 MB, launch-latency
    # bound) and the sweep's 64 scenes as one [64, 3, 512, 768] batch (604 MB,
    # HBM bound); L2 flushed before every call
    for batch in (1, 64):
        x = torch.rand(batch, 3, 512, 768, device=dev)
        y = torch.rand(batch, 3, 512, 768, device=dev)
        n = x.numel()
        for name, fn, nbytes in (("mse", lambda: mt.sse_mse(x.view(-1), y.view(-1)), 8 * n),
                                 ("ssim", lambda: mt.ssim_per_plane(x, y, 11, 1.5, 1e-4, 9e-4),
                                  8 * n)):
            for _ in range(5):
                fn()
            ms = statistics.median(time_device_calls(fn, 30 if batch == 1 else 10, flush, stream))
            line = {"metric": f"standalone {name} kernel bandwidth, {batch}x3x512x768 fp32 pair",
                    "value": round(nbytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms": round(ms, 5), "bytes": nbytes, "peak_hbm_gbs": hbm,
                    "frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                    "l2": "flushed before every call"}
            if name == "ssim":
                # SSIM is bound by the FP32 pipe: 5 moments x 11 taps x 2 passes
                # = 110 FMAs (220 FLOP) per valid output
                flop = 220.0 * batch * 3 * (512 - 10) * (768 - 10)
                tf = flop / (ms * 1e-3) / 1e12
                line["fp32"] = {"tflops": round(tf, 3), "peak_tflops": FP32_PEAK_TFLOPS,
                                "frac": round(tf / FP32_PEAK_TFLOPS, 4),
                                "flop": flop, "model": "220 FLOP per valid output"}
            lines.append(line)
        del x, y
    if rank != 0:
        return None
    return [_json.dumps(line) for line in lines]


class E2EStep:
    """The config-2 training step as a user writes it against the drop-in API:
    ring points gathered into cubics, manbo.ops.render_cubic_fill_splat_tilelang,
    clamp + CHW, manbo.mse_loss_tilelang, manbo.ssim (forward metric),
    backward, torch Adam (lr 0.5 points / 0.01 colours).  Every step copies
    its target image from pinned host memory (on a copy stream, overlapping
    the render; the loss waits for it) and reads the loss and SSIM back into
    pinned host memory."""

    def __init__(self, scene, dev, capturable=False):
        import torch

        from repo_b200 import scenes as sc_mod
        self.h, self.w, self.s = scene.height, scene.width, scene.samples
        self.ring = scene.ring.to(dev).clone().requires_grad_(True)
        self.colors = scene.colors.to(dev).clone().requires_grad_(True)
        self.opac, self.depths = scene.opacities.to(dev), scene.depths.to(dev)
        self.rules = scene.fill_rules.to(dev)
        self.aa, self.bg = scene.aa_widths.to(dev), scene.background.to(dev)
        self.offs = scene.seg_offsets().to(dev)
        self.gidx = sc_mod.ring_gather_index(scene.segs_per_path).to(dev)
        self.half = torch.tensor([0.5 * self.w, 0.5 * self.h], device=dev)
        self.target_host = scene.target.clone().pin_memory()
        self.target_dev = torch.empty_like(self.target_host, device=dev)
        self.loss_host = torch.empty((2,), dtype=torch.float32).pin_memory()
        self.capturable = capturable
        self.opt = torch.optim.Adam([{"params": [self.ring], "lr": 0.5},
                                     {"params": [self.colors], "lr": 0.01}], fused=True,
                                    capturable=capturable)
        self.copy_stream = torch.cuda.Stream(dev)
        self.h2d_bytes = int(self.target_host.numel() * 4)
        self.d2h_bytes = 8

    def __call__(self, marks=None):
        """One step; with a list `marks`, appends (phase, time.perf_counter())
        after each phase (host-time profile)."""
        import torch

        import manbo

        def mark(label):
            if marks is not None:
                marks.append((label, time.perf_counter()))

        mark("start")
        main = torch.cuda.current_stream()
        self.copy_stream.wait_stream(main)  # last step's readers of the target are done
        with torch.cuda.stream(self.copy_stream):
            self.target_dev.copy_(self.target_host, non_blocking=True)
        self.opt.zero_grad(set_to_none=not self.capturable)
        cn = self.ring[:, self.gidx, :].reshape(-1, 4, 2) / self.half - 1.0
        mark("user prep (copy, zero_grad, gather)")
        out = manbo.ops.render_cubic_fill_splat_tilelang(
            cn, self.offs, self.colors, self.opac, self.depths, self.h, self.w, 16, 16, self.bg,
            fill_rules=self.rules, aa_widths=self.aa, distance_samples=self.s)
        mark("render forward (API)")
        img = torch.clamp(out, 0, 1).permute(2, 0, 1).unsqueeze(0).contiguous()
        main.wait_stream(self.copy_stream)
        mark("user clamp/permute")
        loss = manbo.mse_loss_tilelang(img, self.target_dev)
        mark("mse (API)")
        with torch.no_grad():
            sv = manbo.ssim(img.detach(), self.target_dev)
        mark("ssim (API)")
        loss.backward()
        mark("backward (autograd + API backward)")
        self.opt.step()
        mark("torch Adam")
        self.loss_host[0:1].copy_(loss.detach().view(1), non_blocking=True)
        self.loss_host[1:2].copy_(sv.view(1), non_blocking=True)
        mark("loss read-back (enqueue)")


def run_e2e(scene, dev, args, flush, stream, world):
    """Training steps through the manbo API, timed with CUDA events: eagerly
    (as train.py runs), and the same calls captured once into a CUDA graph by
    the caller and replayed (the API is capture-safe: under capture it reads
    nothing back)."""
    import torch
    step = E2EStep(scene, dev)
    # the caching allocator and the host-side caches of the API path take a
    # few dozen steps to settle; time the steady state
    warm = max(E2E_MIN_WARMUP, args.warmup)
    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    total_ms = sum(time_steps(step, args.steps, flush, stream))

    gstep = E2EStep(scene, dev, capturable=True)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(5):
            gstep()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gstep()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    g_ms = sum(time_steps(graph.replay, args.steps, flush, stream))
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([total_ms, g_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, g_ms = (float(v) for v in t.tolist())
    del graph
    return {"value": round(world * args.steps / (total_ms / 1e3), 3), "unit": UNIT,
            "h2d_bytes_per_step": step.h2d_bytes, "d2h_bytes_per_step": step.d2h_bytes,
            "warmup": warm, "path": "manbo.ops.render_cubic_fill_splat_tilelang + "
            "manbo.mse_loss_tilelang + manbo.ssim + autograd + torch Adam, eager (train.py)",
            "ms_per_step": round(total_ms / args.steps, 4),
            "graph": {"value": round(world * args.steps / (g_ms / 1e3), 3), "unit": UNIT,
                      "ms_per_step": round(g_ms / args.steps, 4),
                      "h2d_bytes_per_step": gstep.h2d_bytes,
                      "d2h_bytes_per_step": gstep.d2h_bytes,
                      "path": "the same API calls captured once into a CUDA graph by the "
                              "caller (torch Adam capturable), replayed every step"}}


def run_host_profile(args):
    """Where the drop-in API step's time goes (config 2, one GPU): host time
    per phase of the eager E2EStep (synchronised at the end of every step,
    the wait counted as its own phase), and the device kernels of the step
    from the torch profiler (CUDA activity, averaged per step)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from repo_b200 import scenes
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    step = E2EStep(scenes.config2(), dev)
    for _ in range(max(E2E_MIN_WARMUP, args.warmup)):
        step()
    torch.cuda.synchronize()
    phases, walls = {}, []
    for _ in range(args.steps):
        marks = []
        step(marks)
        torch.cuda.current_stream().synchronize()
        marks.append(("wait for the device (sync)", time.perf_counter()))
        for (_, a), (label, b) in zip(marks, marks[1:]):
            phases[label] = phases.get(label, 0.0) + (b - a)
        walls.append(marks[-1][1] - marks[0][1])
    n = args.steps
    host = {k: round(v / n * 1e6, 1) for k, v in phases.items()}
    prof_steps = 20
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(prof_steps):
            step()
        torch.cuda.synchronize()
    kernels = []
    for ev in prof.key_averages():
        t = getattr(ev, "device_time_total", None)
        if t is None:
            t = getattr(ev, "cuda_time_total", 0.0)
        if t and t > 0:
            kernels.append({"name": ev.key[:120], "calls_per_step": round(ev.count / prof_steps, 2),
                            "us_per_step": round(t / prof_steps, 1)})
    kernels.sort(key=lambda k: -k["us_per_step"])
    return {"metric": "drop-in API step (config 2): host time per phase and device kernels",
            "steps": n, "wall_us_per_step": round(statistics.mean(walls) * 1e6, 1),
            "host_us_per_step": host, "device_kernels_per_step": kernels[:25],
            "profiled_steps": prof_steps}


# --------------------------------------------------------------------------
# GPU reference: the reference's own TileLang renderer, same loop, same box

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def gpu_reference_child(args):
    """Runs in a child process: the E2EStep loop on the unmodified reference
    package installed in baseline/_ref (its TileLang kernels), eager, timed
    like the B200 arm.  Prints one JSON object."""
    sys.path.insert(0, REF_DIR)
    import torch

    import manbo
    import tilelang
    from repo_b200 import scenes
    mpath = os.path.abspath(manbo.__file__)
    if not mpath.startswith(os.path.abspath(REF_DIR)):
        raise RuntimeError(f"manbo resolved to {mpath}, not the reference install")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=dev)
    step = E2EStep(scenes.config2(), dev)
    t0 = time.perf_counter()
    step()  # TileLang compiles its kernels here
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    for _ in range(max(E2E_MIN_WARMUP, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(20, min(args.steps, 200))
    total_ms = sum(time_steps(step, steps, flush_buf.zero_, stream))
    print(json.dumps({"value": round(steps / (total_ms / 1e3), 3), "unit": UNIT,
                      "ms_per_step": round(total_ms / steps, 4), "steps": steps,
                      "first_step_s": round(compile_s, 1),
                      "tilelang": getattr(tilelang, "__version__", "?"),
                      "manbo": os.path.relpath(mpath, ROOT),
                      "final_loss": float(step.loss_host[0])}), flush=True)


def run_gpu_reference(args):
    """The reference renderer's training step on this GPU (child process),
    or why it could not run."""
    if not os.path.isdir(os.path.join(REF_DIR, "manbo")):
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    cmd = [sys.executable, os.path.abspath(__file__), "--gpu-reference-child",
           "--steps", str(args.steps), "--warmup", str(args.warmup)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": "the reference step did not finish within 900 s"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            out = json.loads(line)
            out["path"] = ("reference manbo.ops.render_cubic_fill_splat_tilelang (TileLang) + "
                           "manbo.mse_loss_tilelang + manbo.ssim + autograd + torch Adam, eager, "
                           "the same loop as e2e")
            return out
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"reference step failed (rc {r.returncode}): {tail[0][:200]}"}


# --------------------------------------------------------------------------
# CPU reference arm (the C oracle restating the reference algorithm)

def cpu_iteration(state, scene):
    """One config-2 training iteration on the host: render, MSE, SSIM, backward,
    Adam.  Returns the loss."""
    import numpy as np

    import oracle
    from repo_b200 import scenes as sc_mod
    ring, colors, m, v, t = state["ring"], state["colors"], state["m"], state["v"], state["t"]
    h, w, s = scene.height, scene.width, scene.samples
    gi = sc_mod.ring_gather_index(scene.segs_per_path).numpy()
    cub = ring[:, gi, :].reshape(-1, 4, 2)
    half = np.array([0.5 * w, 0.5 * h], np.float32)
    cn = (cub / half - np.float32(1.0)).astype(np.float32)
    st = oracle.render_fill(cn, scene.seg_offsets().numpy(), colors, scene.opacities.numpy(),
                            scene.depths.numpy(), h, w, scene.background.numpy(),
                            fill_rules=scene.fill_rules.numpy(), aa_widths=scene.aa_widths.numpy(),
                            samples=s)
    out = st["image"]
    img = np.clip(out, 0.0, 1.0).transpose(2, 0, 1)[None]
    tgt = state["target"]
    loss = oracle.mse(img, tgt)
    oracle.ssim(img, tgt)
    g_img = oracle.mse_grad(img, tgt)[0].transpose(1, 2, 0)
    g_out = np.where((out >= 0) & (out <= 1), g_img, 0).astype(np.float32)
    gr = oracle.fill_backward(st, g_out)
    v_cub = (gr["v_cubics_norm"] / half).reshape(ring.shape[0], -1, 2)
    g_ring = np.zeros_like(ring)
    np.add.at(g_ring, (slice(None), gi), v_cub)
    t += 1
    for key, p, g, lr in (("ring", ring, g_ring, 0.5), ("colors", colors, gr["v_colors"], 0.01)):
        m[key] = 0.9 * m[key] + 0.1 * g
        v[key] = 0.999 * v[key] + 0.001 * g * g
        mh = m[key] / (1 - 0.9 ** t)
        vh = v[key] / (1 - 0.999 ** t)
        p -= (lr * mh / (np.sqrt(vh) + 1e-8)).astype(np.float32)
    state["t"] = t
    return loss


def run_cpu(seconds_budget: float, max_iters: int):
    import numpy as np

    import oracle
    from repo_b200 import scenes
    scene = scenes.config2()
    state = {"ring": scene.ring.numpy().copy(), "colors": scene.colors.numpy().copy(),
             "target": scene.target.numpy(), "t": 0,
             "m": {"ring": np.zeros_like(scene.ring.numpy()), "colors": np.zeros_like(scene.colors.numpy())},
             "v": {"ring": np.zeros_like(scene.ring.numpy()), "colors": np.zeros_like(scene.colors.numpy())}}
    cpu_iteration(state, scene)  # warm-up (library load, first touch)
    t0 = time.perf_counter()
    iters = 0
    while iters < max_iters:
        cpu_iteration(state, scene)
        iters += 1
        if time.perf_counter() - t0 > seconds_budget:
            break
    dt = time.perf_counter() - t0
    return iters / dt, iters, dt, oracle.num_threads()


def run_reference(args, rank, world):
    if rank != 0:
        return None
    budget = min(120.0, max(10.0, 1.5 * args.cpu_seconds))
    value, iters, dt, cores = run_cpu(budget, max(1, args.steps))
    sample = (f"{iters} full config-2 training iterations (render fwd, MSE, SSIM, bwd, Adam) "
              f"in {dt:.1f} s; each --steps step is one iteration, capped to ~{budget:.0f} s")
    return {"metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world,
            "steps": iters, "warmup": 1, "ms_per_step": round(1e3 * dt / iters, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD_CONFIG2, "device": "host CPU"},
            "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# --------------------------------------------------------------------------

def main(argv=None):
    args = parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpu_reference_child:
        gpu_reference_child(args)
        return 0
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return 0
    if args.host_profile:
        if world > 1:
            raise SystemExit("--host-profile runs on one GPU")
        print(json.dumps(run_host_profile(args)), flush=True)
        return 0
    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "config3":
            res, tr = run_bands(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps(res), flush=True)
            tr.release_graphs()  # graphs holding collectives go before the process group
            del tr
            return 0
        if args.workload == "config4":
            res = run_stroke(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps(res), flush=True)
            return 0
        if args.workload == "config5":
            out = run_sweep(args, rank, world, local_rank)
            if rank == 0:
                for line in out:
                    print(line, flush=True)
            return 0
        res, tr = run_b200(args, rank, world, local_rank)
        del tr
        if not args.no_strong:
            # config 3 at the same N: one 2040x1356 image in tile-row bands
            # with a gradient all-reduce per step (strong scaling)
            sres, btr = run_bands(args, rank, world, local_rank)
            btr.release_graphs()  # graphs holding collectives go before the process group
            del btr
            if rank == 0:
                res["strong_config3"] = {
                    k: sres[k] for k in ("metric", "value", "unit", "ms_per_step", "n_gpus",
                                         "scaling", "final_loss", "final_ssim")}
                res["strong_config3"]["bands"] = sres["config"]["bands"]
                res["strong_config3"]["collective"] = sres["config"]["collective"]
                res["strong_config3"]["clocks"] = sres["clocks"]
        if rank == 0 and world == 1 and not args.no_gpu_reference:
            ref = run_gpu_reference(args)
            res["gpu_reference"] = ref
            if "value" in ref:
                rv = ref["value"]
                res["vs_gpu_reference"] = {
                    "value": round(res["value"] / rv, 2),
                    "e2e": round(res["e2e"]["value"] / rv, 2) if "e2e" in res else None,
                    "e2e_graph": round(res["e2e"]["graph"]["value"] / rv, 2)
                    if "e2e" in res else None}
        if rank == 0 and not args.no_cpu_baseline:
            value, iters, dt, cores = run_cpu(args.cpu_seconds, 1000)
            res["cpu_baseline"] = {
                "value": round(value, 5), "unit": UNIT, "cores": cores, "kind": "port",
                "sample": f"{iters} full config-2 training iterations on the host in {dt:.1f} s "
                          f"(C oracle, {cores} threads)"}
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
