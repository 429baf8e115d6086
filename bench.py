#!/usr/bin/env python3
"""MH1 inference throughput on B200: atoms*evals/s of energy + forces + virial.

Workload: config C3 -- 10,000-atom perturbed-FCC cube, 46.4 A, ~85 neighbours per atom
within 6 A -- with the seeded synthetic MH1-shaped archive.  One step = one full evaluation
(neighbour list, both interaction layers, readouts, analytical backward, forces and virial).

N = 1: one GPU evaluates the structure.  N > 1 GPUs (one process per GPU, torchrun): the SAME
structure is split across the GPUs by spatial domain decomposition (NCCL halo exchange of
layer-1 features and their gradients, all-reduce of the per-atom outputs): strong scaling,
the job time is the max over ranks.  --replicas restores one independent structure per GPU.
Each line also carries sub-results for the configurations the north star sets its multi-GPU
target on: "c5_decomposed" (~200,000-atom slab, decomposed over the N GPUs) and "c4_batched"
(4,096 independent cells, LPT-sharded over the N GPUs); --no-subconfigs skips them.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value  inputs already resident in HBM (mace_calculate_device), per-step CUDA events,
       L2 flushed (256 MiB write) between steps outside the timed windows.
e2e    the reference-facing C ABI (mace_calculate) with host buffers: the host-to-device
       copy of the inputs and the device-to-host copy of energies/forces are inside.
--impl reference   the reference's own implementation of this path -- its CUDA build
       compiled from its sources (oracle/_ref/libmace_ref.so) -- through its C ABI on the
       same config, on rank 0; falls back to the float64 CPU oracle if that build is absent.
--host  host-side input work instead (no GPU): ARC reads of C1, C2, C3 and C5 and the
       conversion of the seeded synthetic MH1 checkpoint, each the median of --steps runs on
       one pinned core (bin/mace-host-bench; with --impl reference the reference's own
       chemio and converter code, oracle/_ref/host-bench-ref).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "lasp-pis_b200" / "python")]
DATA = ROOT / "lasp-pis_b200" / "data"
METRIC = "atoms*evals/s (E+F+virial), MH1-shape, C3 10k-atom cell"
CONFIG_LABEL = {"C1": "C1 64-atom cell", "C2": "C2 1,000-atom cell", "C3": "C3 10k-atom cell",
                "C5": "C5 ~200k-atom cell"}


def metric_for(config: str) -> str:
    """The headline metric's name, with the cell the run actually measured."""
    return METRIC.replace("C3 10k-atom cell", CONFIG_LABEL.get(config, config))
WORKLOADS = {"C1": "64-atom simple-cubic cell (a = 9 A)", "C2": "1,000-atom triclinic Poisson-disk cell",
             "C3": "10,000-atom perturbed FCC cube, 46.4 A", "C5": "~200,000-atom perturbed BCC Fe/Ni/Cr slab"}
UNIT = "atoms*evals/s"
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# DRAM read + write bytes per edge of the roofline kernel, from an ncu capture of the C2
# workload (edge_proj_kernel<1, backward>: dram__bytes_read.sum 1,048,964,608 +
# dram__bytes_write.sum 188,064,512 over 97,006 edges; profiles/edge_backward1_C2.md), scaled
# by the edge count.
TRAFFIC_PER_EDGE = (1048964608 + 188064512) / 97006
TRAFFIC_SOURCE = "ncu capture of C2 (97,006 edges), scaled by the edge count"


def edge_backward1_bytes(edges: int, paths: int = 10) -> float:
    """Algorithmic HBM bytes of the layer-1 edge tensor-product backward per launch.

    Per directed edge: the cutoff-scaled radial projection row and its r-derivative (2 x paths
    x 128 fp32), Y and dY/dd (16 + 48 fp32), the edge geometry (d, r: 16 B), cutoff and density
    pairs (8 + 8 B), the sender index (4 B), the edge force written (16 B) and the edge's
    up-gradient row written for the sender gather (4 x 128 fp32).  The sender's up-projected
    features stay in L2 and are not counted.
    """
    return edges * (2.0 * paths * 128 * 4 + 64 + 192 + 16 + 8 + 8 + 4 + 16 + 4 * 128 * 4)


def edge_backward1_flops(edges: int, terms: int = 86, groups: int = 22, paths: int = 10) -> float:
    """FP32 operations (an FMA counts 2) of the layer-1 edge backward per launch, per edge and
    channel (128 channels): w_p = cut b_p + R_p (2 P); per tensor-product term a_t = cg G[out]
    (1), S += a_t Y (2, 1 for a group's first term) and T_sh += a_t (u w) (2); per (path, input)
    group u w (1), Q_p += u S (2) and ug += w S (2); dE/dr = sum_p Q_p (dcut b_p + dR_p) (4 P);
    dE/dd = sum_sh T_sh dY_sh (48 FMAs).  Layer 1 of MH1: 86 terms in 22 groups over 10 paths."""
    per_channel = 2 * paths + 5 * terms - groups + 5 * groups + 4 * paths + 96
    return float(edges) * 128 * per_channel


def linear_flops(archive_path, name: str, nodes: int) -> float:
    """FP32 FLOP of one equivariant linear over `nodes` nodes: 2 in_mul out_mul (2l + 1) per
    path (the archive's `<name>.paths`, 6 ints per path: in/out offsets, in_mul, out_mul, dim,
    weight offset)."""
    sys.path.insert(0, str(ROOT / "lasp-pis_b200" / "python"))
    from lasp_b200 import archive as arc
    paths = arc.read(archive_path)[name + ".paths"].reshape(-1, 6)
    return float(nodes) * float(sum(2 * int(p[2]) * int(p[3]) * int(p[4]) for p in paths))


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running.

    mark_start() / mark_end() bracket the timed region; summary() then keeps the samples
    taken within one sampling period of it (the GPU is busy with the warm-up right before and
    the profiled calls right after), so a timed region shorter than the period still gets its
    samples.  Without marks every sample counts."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.2

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.start = self.end = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", str(int(self.PERIOD_S * 1000))],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.time() + 5.0  # the first sample, so the timed region is covered
            while not self.lines and time.time() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark_start(self):
        self.start = time.time()

    def mark_end(self):
        self.end = time.time()
        time.sleep(self.PERIOD_S * 1.5)  # the sample that follows the region

    def __exit__(self, *args):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                t = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clock, clock_max = float(f[2]), float(f[3])
            except ValueError:
                continue
            if self.start is not None and not (self.start - self.PERIOD_S <= t <= (self.end or t) + self.PERIOD_S):
                continue
            sm.append(clock)
            mx = clock_max
            for name, flag in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    if PEAKS.exists():
        p = json.loads(PEAKS.read_text())
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


def cpu_baseline(archive):
    """Float64 CPU oracle (a restatement of the reference path) on a bounded sample: one
    evaluation of a 4,096-atom cube at C3 density (about 10-30 s on the box's host cores)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from lasp_b200 import structures
    cores = oracle.threads(os.cpu_count() or 1)
    s = structures.density_sample(4096)
    model = oracle.Oracle(archive)
    t = time.perf_counter()
    model.calculate(s.positions, s.numbers, s.cell)
    dt = time.perf_counter() - t
    return {"value": s.size / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"one E+F+virial evaluation of a {s.size}-atom cube at C3 density (same generator, "
                      f"{dt:.1f} s) by the float64 oracle"}


def workload_config(config: str, atoms: int, world: int, decompose: bool) -> dict:
    """The `config` object of a line: identical for this build and the reference arm at N = 1."""
    if world == 1:
        parallelism = "one GPU"
    elif decompose:
        parallelism = f"spatial domain decomposition of one structure over {world} GPUs (NCCL halo exchange)"
    else:
        parallelism = f"{world} independent replicas (one structure per GPU)"
    return {"workload": f"{config}: {WORKLOADS.get(config, config)}, cutoff 6 A, seeded synthetic MH1-shaped "
                        "archive (seed 20261201)",
            "atoms": atoms, "parallelism": parallelism,
            "l2": "256 MiB buffer written between timed steps (outside the per-step timing)"}


def io_bytes(n: int) -> tuple[int, int]:
    """Host bytes per evaluation through mace_calculate: xyz (12 n) + Z (4 n) + cell (36) in;
    per-atom energies (4 n) + forces (12 n) + energy (8) + virial (36) out."""
    return 16 * n + 36, 16 * n + 44


def reference_arm(args, archive, structure):
    import ctypes as ct
    lib_path = ROOT / "oracle" / "_ref" / "libmace_ref.so"
    n = structure.size
    h2d, d2h = io_bytes(n)
    if not lib_path.exists():
        base = cpu_baseline(archive)
        line = {"impl": "reference", "metric": metric_for(args.config), "value": base["value"], "unit": UNIT,
                "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": True, "data": "synthetic",
                "config": {"workload": "C3 density sample (reference CUDA build absent)"},
                "cpu_baseline": base, "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                              "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return
    import torch
    lib = ct.CDLL(str(lib_path))
    lib.mace_create_mh1.argtypes = [ct.c_char_p, ct.c_int]
    lib.mace_create_mh1.restype = ct.c_void_p
    lib.mace_last_error.restype = ct.c_char_p
    lib.mace_calculate.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 7
    lib.mace_destroy.argtypes = [ct.c_void_p]
    lib.mace_diagnostics.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t]
    lib.mace_diagnostics.restype = ct.c_int
    h = lib.mace_create_mh1(str(archive).encode(), 0)
    if not h:
        print(json.dumps({"impl": "reference", "unavailable": lib.mace_last_error().decode()}))
        return
    s = structure
    e = np.zeros(1)
    a = np.zeros(n, np.float32)
    f = np.zeros((n, 3), np.float32)
    v = np.zeros((3, 3), np.float32)
    ptrs = [x.ctypes.data for x in (s.positions, s.numbers, s.cell, e, a, f, v)]
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MiB > L2
    for _ in range(args.warmup):
        assert lib.mace_calculate(h, n, *ptrs) == 0, lib.mace_last_error()
    times, device = [], []
    diag = ct.create_string_buffer(1 << 16)
    with ClockSampler(0) as clocks:
        for _ in range(args.steps):
            flush.fill_(1.0)
            torch.cuda.synchronize()
            t = time.perf_counter()
            assert lib.mace_calculate(h, n, *ptrs) == 0
            times.append(time.perf_counter() - t)
            # The reference's own CUDA-event time of the call (lapis/src/runtime.cu:287), read
            # outside the timed window.
            if lib.mace_diagnostics(h, diag, len(diag)) == 0:
                try:
                    device.append(float(json.loads(diag.value)["device_ms"]))
                except (ValueError, KeyError):
                    pass
    lib.mace_destroy(h)
    total = float(np.sum(times))
    value = n * args.steps / total
    line = {"impl": "reference", "metric": metric_for(args.config), "value": value, "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.config, n, 1, False),
            "implementation": "reference CUDA build (LipidL/LASP-PIS libmace) compiled for sm_100a from its "
                              "sources, called through its C ABI with host buffers (wall clock per blocking call)",
            "reference_device_ms": float(np.median(device)) if device else None,
            "clocks": clocks.summary(),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "reference",
                             "sample": f"full {args.config} workload per step; the reference has no CPU inference "
                                       "path, its host code (prepare/finish) is single-threaded and the model runs "
                                       "on one B200"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}}
    print(json.dumps(line))


C4_METRIC = "atoms*evals/s (E+F+virial), MH1-shape, C4 batch of 4,096 independent cells"
C5_METRIC = "atoms*evals/s (E+F+virial), MH1-shape, C5 ~200k-atom cell"


def c4_reference(args, archive):
    """The reference has no batched call: its callers loop over mace_calculate.  Time that
    loop (reference CUDA build, C ABI, host buffers) over the first 512 C4 cells."""
    import ctypes as ct
    from lasp_b200 import structures
    lib_path = ROOT / "oracle" / "_ref" / "libmace_ref.so"
    if not lib_path.exists():
        print(json.dumps({"impl": "reference", "unavailable": "reference CUDA build absent (oracle/_ref)"}))
        return
    cells = structures.load_c4(DATA)[:512]
    lib = ct.CDLL(str(lib_path))
    lib.mace_create_mh1.argtypes = [ct.c_char_p, ct.c_int]
    lib.mace_create_mh1.restype = ct.c_void_p
    lib.mace_last_error.restype = ct.c_char_p
    lib.mace_calculate.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 7
    lib.mace_destroy.argtypes = [ct.c_void_p]
    h = lib.mace_create_mh1(str(archive).encode(), 0)
    e = np.zeros(1)
    v = np.zeros((3, 3), np.float32)

    def run():
        for c in cells:
            a = np.zeros(c.size, np.float32)
            f = np.zeros((c.size, 3), np.float32)
            assert lib.mace_calculate(h, c.size, c.positions.ctypes.data, c.numbers.ctypes.data,
                                      c.cell.ctypes.data, e.ctypes.data, a.ctypes.data, f.ctypes.data,
                                      v.ctypes.data) == 0, lib.mace_last_error()
    for _ in range(args.warmup):
        run()
    t = time.perf_counter()
    for _ in range(args.steps):
        run()
    total = time.perf_counter() - t
    lib.mace_destroy(h)
    atoms = sum(c.size for c in cells)
    value = atoms * args.steps / total
    print(json.dumps({"impl": "reference", "metric": C4_METRIC, "value": value, "unit": UNIT, "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic",
                      "config": {"workload": "C4: first 512 of the 4,096 cells (32-256 atoms each), sequential "
                                             "mace_calculate calls -- the reference has no batched call",
                                 "atoms": atoms},
                      "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "reference",
                                       "sample": "512 C4 cells per step"},
                      "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 16 * atoms + 36 * len(cells),
                              "d2h_bytes_per_step": 16 * atoms + 44 * len(cells)}}))


class Ranks:
    """One process per GPU (torchrun env), NCCL process group for the host-side plumbing."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))

    def init(self):
        import torch
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))

    def barrier(self):
        import torch
        if self.world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max(self, *values):
        import torch
        if self.world == 1:
            return list(values)
        t = torch.tensor(values, device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return [float(x) for x in t]

    def model(self, archive, lib_path, decompose: bool):
        """A NativeMH1 on this rank's GPU; decomposed over all ranks when asked (a fresh NCCL
        communicator per handle, its id made by rank 0)."""
        import torch
        from mace_inference import NativeMH1
        if decompose and self.world > 1:
            from mace_inference import nccl_unique_id
            box = [nccl_unique_id(lib_path) if self.rank == 0 else None]
            torch.distributed.broadcast_object_list(box, src=0)
            return NativeMH1(archive, backend=0, library=lib_path, device=self.local,
                             domain=(self.rank, self.world, box[0]))
        return NativeMH1(archive, backend=0, library=lib_path, device=self.local)

    def close(self):
        if self.world > 1:
            import torch
            torch.distributed.destroy_process_group()


def c4_batched(ranks: Ranks, archive, lib_path, cells, steps: int, warmup: int) -> dict:
    """C4 through mace_calculate_batch: the 4,096 cells split across the ranks by LPT on
    estimated work (strong scaling: the job is fixed), timed end to end on each rank (host
    buffers, every H2D/D2H inside) and reported as the max over ranks."""
    from mace_inference.batch import estimated_work, lpt_partition
    items = [(c.positions, c.numbers, c.cell) for c in cells]
    shards = lpt_partition([estimated_work(len(z), h) for _, z, h in items], ranks.world)
    mine = [items[i] for i in shards[ranks.rank]]
    model = ranks.model(archive, lib_path, False)
    for _ in range(warmup):
        model.calculate_batch(mine)
    ranks.barrier()
    t = time.perf_counter()
    for _ in range(steps):
        model.calculate_batch(mine)
    elapsed = time.perf_counter() - t
    launches = int(model.diagnostics["launches"])
    model.close()
    (elapsed,) = ranks.max(elapsed)
    atoms = sum(len(z) for _, z, _ in items)
    value = atoms * steps / elapsed
    return {"metric": C4_METRIC, "value": value, "unit": UNIT, "n_gpus": ranks.world, "steps": steps,
            "warmup": warmup, "ms_per_step": 1e3 * elapsed / steps, "scaling": "strong", "atoms": atoms,
            "parallelism": f"LPT over {ranks.world} GPU(s), no data-path collective",
            "timing": "end to end (mace_calculate_batch with host buffers), max over ranks",
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": atoms * 16 + 36 * len(items),
                    "d2h_bytes_per_step": atoms * 16 + 44 * len(items)},
            "gpu_launches_last_sub_batch": launches}


def c5_decomposed(ranks: Ranks, archive, lib_path, structure, steps: int, warmup: int) -> dict:
    """C5 (~200,000 atoms) split across the ranks by spatial domain decomposition (one GPU
    evaluates all of it at N = 1): device-resident inputs, per-step CUDA events, max over ranks."""
    import torch
    s = structure
    model = ranks.model(archive, lib_path, True)
    xyz = torch.from_numpy(s.positions).cuda()
    z = torch.from_numpy(s.numbers).cuda()
    for _ in range(warmup):
        model.calculate_device(s.size, xyz.data_ptr(), z.data_ptr(), s.cell)
    ranks.barrier()
    total = 0.0
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.calculate_device(s.size, xyz.data_ptr(), z.data_ptr(), s.cell)
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    diag = model.diagnostics
    model.close()
    del xyz, z
    torch.cuda.empty_cache()
    (total,) = ranks.max(total)
    return {"metric": C5_METRIC, "value": s.size * steps / (total * 1e-3), "unit": UNIT, "n_gpus": ranks.world,
            "steps": steps, "warmup": warmup, "ms_per_step": total / steps, "scaling": "strong", "atoms": s.size,
            "edges": int(diag["edges"]),
            "parallelism": ("spatial domain decomposition over %d GPUs (NCCL halo exchange)" % ranks.world)
            if ranks.world > 1 else "one GPU",
            "timing": "device-resident inputs (mace_calculate_device), CUDA events per step, max over ranks"}


def host_arm(args):
    """One JSON line of host-side input timings (rank 0 only; no GPU)."""
    import tempfile
    import torch
    from lasp_b200 import checkpoint, structures
    if args.impl == "reference":
        exe = ROOT / "oracle" / "_ref" / "host-bench-ref"
        if not exe.exists():
            print(json.dumps({"impl": "reference", "unavailable": "reference host tools absent (oracle/_ref)"}))
            return
    else:
        exe = ROOT / "lasp-pis_b200" / "bin" / "mace-host-bench"
        if not exe.exists():
            raise SystemExit("mace-host-bench is not built: run __graft_entry__.build() (make -C lasp-pis_b200)")
    pin = ["taskset", "-c", str(min(os.sched_getaffinity(0)))] if subprocess.run(
        ["which", "taskset"], capture_output=True).returncode == 0 else []
    steps = {}
    with tempfile.TemporaryDirectory() as tmp:
        jobs = []
        for name in ("C1", "C2", "C3", "C5"):
            path = Path(tmp) / f"{name}.arc"
            structures.write_arc(path, [structures.load(name, DATA)])
            jobs.append((f"arc_{name}", "arc", path))
        model = checkpoint.write_checkpoint(Path(tmp) / "mh1.model", checkpoint.SEED, torch.float64)
        jobs.append(("convert_checkpoint", "convert", model))
        for key, step, path in jobs:
            r = subprocess.run(pin + [str(exe), step, str(path), str(args.steps)], capture_output=True, text=True,
                               check=True)
            steps[key] = json.loads(r.stdout)
    cpu = next((line.split(":", 1)[1].strip() for line in Path("/proc/cpuinfo").read_text().splitlines()
                if line.startswith("model name")), "unknown")
    print(json.dumps({"impl": args.impl, "metric": "host input work (ARC read, MH1 checkpoint conversion)",
                      "unit": "ms", "higher_is_better": False, "cores": 1, "pinned": bool(pin), "cpu": cpu,
                      "nproc": os.cpu_count(), "repeat": args.steps,
                      "steps": {k: {"median_ms": v["median_ms"], "min_ms": v["min_ms"], "units": v["units"]}
                                for k, v in steps.items()},
                      "data": "synthetic (C1-C5 ARC files; seeded torch.save MH1-shaped checkpoint, 54 MB float64)"}))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="C3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1 GPUs, one independent structure per GPU (weak scaling) instead of one "
                         "structure split across the GPUs")
    ap.add_argument("--no-subconfigs", action="store_true", help="skip the C5-decomposed and C4-batched results")
    ap.add_argument("--host", action="store_true",
                    help="time the host-side input work (ARC reads, checkpoint conversion) instead; no GPU")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.host:
        if int(os.environ.get("RANK", 0)) == 0:
            host_arm(args)
        return
    ranks = Ranks()
    from lasp_b200 import structures, synth
    archive = DATA / "mh1_synth.pwm"
    if ranks.rank == 0:
        synth.write_archive(archive)
    if args.config == "C4":
        if args.impl == "reference":
            if ranks.rank == 0:
                c4_reference(args, archive)
            return
        cells = structures.load_c4(DATA)
        ranks.init()
        line = c4_batched(ranks, archive, ROOT / "lasp-pis_b200" / "lib" / "libmace.so", cells, args.steps,
                          args.warmup)
        if ranks.rank == 0:
            line.update({"higher_is_better": True, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                         "config": {"workload": "C4: 4,096 cells, 32-256 atoms, Z 1-20, seed 104",
                                    "atoms": line["atoms"], "parallelism": line["parallelism"]}})
            print(json.dumps(line))
        ranks.close()
        return
    structure = structures.load(args.config, DATA)
    if args.impl == "reference":
        if ranks.rank == 0:
            reference_arm(args, archive, structure)
        return
    subconfigs = not args.no_subconfigs
    # Inputs are made on the host before any GPU work (the C4 generator uses a process pool).
    c5 = structures.load("C5", DATA) if subconfigs else None
    c4 = structures.load_c4(DATA) if subconfigs else None
    import torch
    ranks.init()
    lib_path = ROOT / "lasp-pis_b200" / "lib" / "libmace.so"
    if not lib_path.exists():
        raise SystemExit("libmace.so is not built: run __graft_entry__.build() (make -C lasp-pis_b200)")
    world = ranks.world
    decompose = world > 1 and not args.replicas
    model = ranks.model(archive, lib_path, decompose)
    s = structure
    n = s.size
    xyz_d = torch.from_numpy(s.positions).cuda()
    z_d = torch.from_numpy(s.numbers).cuda()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MiB > L2
    xyz_h = torch.from_numpy(s.positions).pin_memory()
    z_h = torch.from_numpy(s.numbers).pin_memory()
    xyz_h_np, z_h_np = xyz_h.numpy(), z_h.numpy()

    for _ in range(args.warmup):
        model.calculate_device(n, xyz_d.data_ptr(), z_d.data_ptr(), s.cell)
        model.calculate(xyz_h_np, z_h_np, s.cell)

    def timed(fn, steps):
        times, stages, graph = [], {}, set()
        for _ in range(steps):
            flush.fill_(1.0)
            ranks.barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
            diag = model.diagnostics
            graph.add(diag["graph"])
            for name, ms in diag["stages"]:
                stages.setdefault(name, []).append(ms)
        return times, stages, graph

    device_call = lambda: model.calculate_device(n, xyz_d.data_ptr(), z_d.data_ptr(), s.cell)
    with ClockSampler(ranks.local) as clocks:
        for _ in range(2):  # keeps the GPU busy while the sampler starts
            device_call()
        ranks.barrier()
        clocks.mark_start()
        dev_times, _, graph_modes = timed(device_call, args.steps)
        ranks.barrier()
        e2e_times, _, _ = timed(lambda: model.calculate(xyz_h_np, z_h_np, s.cell), args.steps)
        clocks.mark_end()
        ranks.barrier()
        # Per-stage CUDA events (the roofline kernels' times) from separate, untimed calls:
        # profiling records events between the stages and runs the kernels directly.
        model.profile(True)
        _, stages, _ = timed(device_call, 3)
        model.profile(False)
        ranks.barrier()
    diag = model.diagnostics
    model.close()
    del flush
    torch.cuda.empty_cache()
    dev_ms, e2e_ms = ranks.max(float(np.sum(dev_times)), float(np.sum(e2e_times)))
    structures_per_step = world if (world > 1 and not decompose) else 1
    sub = {}
    if subconfigs:
        sub["c5_decomposed"] = c5_decomposed(ranks, archive, lib_path, c5, min(args.steps, 3), 2)
        sub["c4_batched"] = c4_batched(ranks, archive, lib_path, c4, min(args.steps, 2), 1)
    if ranks.rank == 0:
        pk, kind = peaks()
        edges = int(diag["edges"])
        clk = clocks.summary()
        mhz = clk["sm_mhz"] or clk["sm_max_mhz"] or float(pk.get("sm_max_mhz", 1965.0))
        sms = torch.cuda.get_device_properties(ranks.local).multi_processor_count
        k_ms = float(np.mean(stages.get("backward1.edges", [float("nan")])))
        flops = edge_backward1_flops(edges)
        fp32_peak = sms * 128 * 2 * mhz * 1e6 / 1e12
        achieved = flops / (k_ms * 1e-3) / 1e12
        gbs = edge_backward1_bytes(edges) / (k_ms * 1e-3) / 1e9
        hbm = float(pk["hbm_gbs"])
        g_ms = float(np.mean(stages.get("forward0.linear_2", [float("nan")])))
        # Rank 0 owns the first n // world atoms of the bin-sorted order in a decomposed run.
        g_flop = linear_flops(archive, "layer0.linear_2", n // world if decompose else n)
        f16_peak = float(pk["bf16_tflops"])
        g_fp32 = g_flop / (g_ms * 1e-3) / 1e12
        line = {
            "metric": metric_for(args.config), "value": structures_per_step * n * args.steps / (dev_ms * 1e-3),
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "weak" if structures_per_step > 1 else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.config, n, world, decompose),
            "edges": edges,
            "e2e": {"value": structures_per_step * n * args.steps / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": io_bytes(n)[0] * structures_per_step,
                    "d2h_bytes_per_step": io_bytes(n)[1] * structures_per_step},
            "roofline": {
                "kernel": "edge_proj_kernel<1, backward> (layer-1 edge tensor-product backward: adjoints, "
                          "r-tangent, per-edge force, per-edge up-gradient rows)" + (" on rank 0" if world > 1 else ""),
                "bound": "fp32", "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": achieved / fp32_peak,
                "peak_source": f"{sms} SMs x 128 FP32 lanes x 2 FLOP x {mhz:.0f} MHz (median SM clock sampled "
                               "during the timed steps)",
                "algorithmic_flop_per_launch": flops, "kernel_ms": k_ms,
                "traffic": TRAFFIC_PER_EDGE * edges if TRAFFIC_PER_EDGE else None,
                "traffic_source": TRAFFIC_SOURCE,
                "hbm": {"achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                        "algorithmic_bytes_per_launch": edge_backward1_bytes(edges),
                        "peak_source": f"hbm_gbs ({kind})"},
                "limiter": "FP32 issue: three FP32 instructions per tensor-product term and channel plus three "
                           "per (path, input) group; one third of them are multiplies (1 FLOP), so the FLOP "
                           "fraction sits below the issue fraction"},
            "roofline_tc_gemm": {
                "kernel": "tc_gemm_kernel, layer-0 linear_2 (4 paths 512 x 512, 16 components per node: one "
                          "grouped tcgen05 launch)" + (" on rank 0" if world > 1 else ""),
                "bound": "tensor", "achieved": 3 * g_fp32, "peak": f16_peak, "unit": "TFLOP/s",
                "frac": 3 * g_fp32 / f16_peak, "f16_passes": 3,
                "fp32_flop_per_launch": g_flop, "fp32_tflops": g_fp32, "kernel_ms": g_ms,
                "peak_source": f"bf16_tflops ({kind}): the dense fp16 rate equals the bf16 rate",
                "note": "achieved counts the three fp16 MMA passes (A_lo B_hi + A_hi B_lo + A_hi B_hi) of the "
                        "split that keeps fp32 accuracy"},
            "stages_ms": {k: float(np.mean(v)) for k, v in stages.items()},
            "gpu_launches": int(diag["launches"]) * args.steps,
            "cuda_graph": sorted(graph_modes),
            "clocks": clk,
        }
        line.update(sub)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(archive)
        print(json.dumps(line))
    ranks.close()


if __name__ == "__main__":
    main()
