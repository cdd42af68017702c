"""Benchmark of the B200 VCSR SpMM engine.

`python bench.py --gpus N --steps K --warmup W` prints one JSON line.  A step
is one C = A*B over the workload's matrix with inputs resident in HBM; L2 is
flushed (256 MB write) before every timed step and each step is timed with
CUDA events on the launching stream.  Under torchrun each rank owns one GPU;
the reported time is the max over ranks.

Default workload: the north star's scaling configuration, R-MAT 2^22 at
O = 256: A cut into N nnz-balanced row panels (one per rank),
B replicated once by an NCCL broadcast (timed apart: `bcast_ms`), C panels
disjoint, strong scaling.  At N = 1 the line also carries `fem_o128`, the
FEM-banded O = 128 record (configs[1], the configuration the north star's
roofline and cuSPARSE targets are stated on) with its own roofline, peers and
end-to-end figure.

Other workloads (`--workload`; synthetic stand-ins with the benchmark
configurations' shapes):
  fem            62,451 x 62,451 FEM-style banded, ~4.0M nnz, O = 128.  With
                 N GPUs every rank owns one such panel: weak scaling.
  fem_o32 / fem_o512, uniform (O=32), powerlaw_o8 / powerlaw_o64 /
  powerlaw_o128,
  blockdense (O=512): single-panel variants (weak scaling under N GPUs).
  blockdense_tf32  the same matrix with its dense 16x16 blocks on the
                 tensor cores in TF32 (VCSR_PLAN_TF32_PANELS).
  rmat_bf16, fem_bf16, rmat_f16, fem_f16  B held in bfloat16 / float16,
                 widened to FP32 as it is loaded, FP32 sums.

`--impl reference` times the reference's CSR algorithm (src/kernels.cu:15-33,
restated in oracle/oracle.c) on the host cores instead, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vcsr-spmm_b200"))

METRIC = "SpMM GFLOP/s (2*nnz*O/t)"
L2_NOTE = "flushed before every timed GPU step (256 MB write)"

WORKLOADS = {
    # name: (generator config, size_param, O, scaling, label)
    "rmat": ("rmat", 22, 256, "strong", "rmat_s22_O256"),
    "fem": ("fem", 0, 128, "weak", "fem_banded_62451_O128"),
    "fem_o32": ("fem", 0, 32, "weak", "fem_banded_62451_O32"),
    "fem_o512": ("fem", 0, 512, "weak", "fem_banded_62451_O512"),
    "uniform": ("uniform", 0, 32, "weak", "uniform_4096_16pr_O32"),
    "powerlaw_o8": ("powerlaw", 0, 8, "weak", "powerlaw_321821_O8"),
    "powerlaw_o64": ("powerlaw", 0, 64, "weak", "powerlaw_321821_O64"),
    # the north star states its roofline and cuSPARSE targets for the
    # power-law matrix at O = 128
    "powerlaw_o128": ("powerlaw", 0, 128, "weak", "powerlaw_321821_O128"),
    "blockdense": ("blockdense", 0, 512, "weak", "blockdense_65536_O512_fp32"),
    "blockdense_tf32": ("blockdense", 0, 512, "weak", "blockdense_65536_O512_tf32"),
    "rmat_bf16": ("rmat", 22, 256, "strong", "rmat_s22_O256_bf16in"),
    "fem_bf16": ("fem", 0, 128, "weak", "fem_banded_62451_O128_bf16in"),
    "rmat_f16": ("rmat", 22, 256, "strong", "rmat_s22_O256_f16in"),
    "fem_f16": ("fem", 0, 128, "weak", "fem_banded_62451_O128_f16in"),
}
# workloads whose dense 16x16 blocks run on the tcgen05 TF32 path
TF32_WORKLOADS = {"blockdense_tf32"}
# workloads whose B is held in a 16-bit type (FP32 sums: vcsr_spmm_bf16 / _f16)
HALF_WORKLOADS = {"rmat_bf16": "bfloat16", "fem_bf16": "bfloat16",
                  "rmat_f16": "float16", "fem_f16": "float16"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="rmat")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--size", type=int, default=None,
                    help="override the workload's size parameter (rows, or the R-MAT "
                         "scale); for small profiling captures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-peers", action="store_true")
    ap.add_argument("--no-fem-record", action="store_true",
                    help="leave out the FEM O=128 sub-record of the N=1 R-MAT line")
    ap.add_argument("--sub-steps", type=int, default=400,
                    help="timed steps of the FEM sub-record (short steps: a window "
                         "long enough for the clock sampler)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU baseline sample length")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(label):
    """DRAM bytes per launch from the committed ncu summary of this workload
    (profiles/*.md with a line `dram_bytes_per_launch[<label>] = <n>`)."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    pat = re.compile(r"dram_bytes_per_launch\[" + re.escape(label) + r"\]\s*=\s*([0-9.eE+]+)")
    for fn in sorted(os.listdir(d)):
        if fn.endswith((".md", ".txt")):
            m = pat.search(open(os.path.join(d, fn)).read())
            if m:
                return float(m.group(1))
    return None


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class Clocks:
    """SM clock and clock-event reasons of one GPU, sampled through NVML about
    every millisecond by a child process (so the benchmark's own thread never
    delays it), written to a file; only samples inside [start, stop] count
    (or the one just before start, when the timed region is shorter)."""
    CHILD = r"""
import select, sys, time
import pynvml as N
N.nvmlInit()
h = N.nvmlDeviceGetHandleByUUID(sys.argv[1])
out = open(sys.argv[2], "w")
print("max", N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM), flush=True)
while True:
    r, _, _ = select.select([sys.stdin], [], [], 0.001)
    if r and not sys.stdin.readline():
        break
    t = time.monotonic()
    c = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
    e = N.nvmlDeviceGetCurrentClocksEventReasons(h)
    out.write(f"{t:.6f} {c} {e}\n")
out.close()
"""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown"}

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None
        self.max_mhz = None

    def launch(self):
        import subprocess
        import tempfile
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".txt")
            os.close(fd)
            self.proc = subprocess.Popen([sys.executable, "-c", self.CHILD, self.uuid, self.path],
                                         stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline().split()
            self.max_mhz = float(first[1]) if len(first) == 2 else None
        except Exception:
            self.proc = None
        return self

    def start(self):
        self.t0 = time.monotonic()

    def stop(self):
        self.t1 = time.monotonic()
        if self.proc is None:
            return None
        time.sleep(0.003)
        try:
            self.proc.communicate(input="\n", timeout=30)
            with open(self.path) as f:
                lines = f.read().splitlines()
            os.unlink(self.path)
        except Exception:
            self.proc.kill()
            return None
        samples = []
        for line in lines:
            f = line.split()
            if len(f) == 3:
                samples.append((float(f[0]), float(f[1]), int(f[2])))
        inside = [x for x in samples if self.t0 <= x[0] <= self.t1]
        if not inside:
            before = [x for x in samples if x[0] < self.t0]
            inside = before[-1:]
        if not inside:
            return None
        reasons = 0
        for x in inside:
            reasons |= x[2]
        return {"sm_mhz": float(np.median([x[1] for x in inside])),
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(v for k, v in self.REASONS.items() if reasons & k),
                "samples": len(inside), "source": "nvml, ~1 ms interval",
                "window_ms": round((self.t1 - self.t0) * 1e3, 3)}


def algorithmic_bytes(csr, O, b_bytes=4):
    """A as CSR (values + indices + row pointers), B after perfect reuse (each
    touched row once), C written once."""
    touched = int(np.count_nonzero(np.bincount(csr.col, minlength=csr.N))) if csr.nnz else 0
    return (8 * csr.nnz + 4 * (csr.M + 1) + b_bytes * O * touched + 4 * O * csr.M), touched


def sample_rows(csr, O, flops_cap):
    """Every k-th row of A, k chosen so that the sample holds at most about
    flops_cap flops (all rows when A is small enough): a sample with the
    matrix's own mix of short and long rows.  Returns (row_ptr, col, val,
    rows, description)."""
    total = 2.0 * csr.nnz * O
    if total <= flops_cap:
        return csr.row_ptr, csr.col, csr.val, csr.M, f"all {csr.M} rows"
    k = int(np.ceil(total / flops_cap))
    rows = np.arange(0, csr.M, k)
    lens = (csr.row_ptr[rows + 1] - csr.row_ptr[rows]).astype(np.int64)
    rp = np.zeros(len(rows) + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    idx = np.repeat(csr.row_ptr[rows].astype(np.int64) - rp[:-1], lens) + np.arange(rp[-1])
    return (rp.astype(np.int32), csr.col[idx], csr.val[idx], len(rows),
            f"every {k}th row ({len(rows)} of {csr.M} rows)")


def host_threads():
    # every core this process may run on: torchrun sets OMP_NUM_THREADS=1 for
    # its ranks, which must not shrink the CPU arm
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference(csr, B, seconds, min_reps=3, threads=None, flops_cap=2e9):
    """The reference CSR algorithm (src/kernels.cu:15-33, restated in the
    oracle) on the host cores, over a bounded sample of rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = threads or host_threads()
    O = B.shape[1]
    rp, cc, vv, rows, what = sample_rows(csr, O, flops_cap)
    nnz_s = int(rp[rows])
    Cm = np.empty((rows, O), np.float32)
    oracle.csr_spmm_f32_into(rows, rp, cc, vv, B, Cm, threads)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while reps < min_reps or time.perf_counter() - t0 < seconds:
        oracle.csr_spmm_f32_into(rows, rp, cc, vv, B, Cm, threads)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    gflops = 2.0 * nnz_s * O / dt / 1e9
    sample = (f"{what}, {nnz_s} of {csr.nnz} nnz, O={O}, "
              f"{reps} reps x {dt * 1e3:.2f} ms")
    return {"value": round(gflops, 3), "unit": "GFLOP/s", "cores": threads,
            "kind": "port", "sample": sample}


def cpu_baseline(csr, B, seconds):
    """All host threads, plus the same algorithm on one thread (a smaller
    sample) and the host CPU model."""
    allc = cpu_reference(csr, B, seconds)
    one = cpu_reference(csr, B, min(3.0, seconds / 3), min_reps=1, threads=1, flops_cap=2e8)
    allc["single_thread"] = {"value": one["value"], "unit": "GFLOP/s", "cores": 1,
                             "sample": one["sample"]}
    allc["cpu_model"] = cpu_model()
    return allc


def workload_config(label, csr_M, csr_N, global_nnz, O, world):
    """The workload's description, the same in both arms (no plan details)."""
    return {"workload": label, "M": csr_M, "N": csr_N, "global_nnz": global_nnz, "O": O,
            "segw": 4, "bundle": 32, "l2": L2_NOTE,
            "parallelism": (f"row panels x{world}, B broadcast once" if world > 1 else "1 GPU")}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, size, O, scaling, label = WORKLOADS[args.workload]
    if args.size is not None:
        size, label = args.size, f"{label}@size{args.size}"
    lo = 0.0 if cfg == "rmat" else -1.0
    if cfg == "rmat":
        # the same seeded inputs, restated in the oracle: this arm loads
        # nothing of the engine
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import types
        import oracle
        M, rp, col, val = oracle.gen_rmat(size, args.seed)
        csr = types.SimpleNamespace(M=M, N=M, nnz=len(col), row_ptr=rp, col=col, val=val)
        B = oracle.gen_dense(M, O, args.seed + 1000, lo, 1.0)
        inputs = "oracle restatement of the engine's seeded generators (bit-identical)"
    else:
        import vcsr_b200 as V
        csr = V.gen_csr(cfg, args.seed, size)
        B = V.gen_dense_host(csr.N, O, args.seed + 1000, lo, 1.0)
        inputs = "the engine library's seeded generators"
    per_step = max(1.0, args.cpu_seconds / max(1, args.steps))
    for _ in range(args.warmup):
        cpu_reference(csr, B, 0.0, min_reps=1)
    vals = []
    info = None
    for _ in range(args.steps):
        info = cpu_reference(csr, B, per_step, min_reps=1)
        vals.append(info["value"])
    v = float(np.median(vals))
    flops = 2.0 * csr.nnz * O
    world = args.gpus
    line = {"metric": METRIC, "value": round(v, 3), "unit": "GFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(flops / (v * 1e9) * 1e3, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": workload_config(label, csr.M, csr.N, csr.nnz, O, world),
            "algorithm": "reference CSR SpMM (src/kernels.cu:15-33) on host cores, "
                         "OpenMP over rows",
            "inputs": inputs,
            "cpu_baseline": dict(info, value=round(v, 3), cpu_model=cpu_model()),
            "e2e": {"value": round(v, 3), "unit": "GFLOP/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def timed_events(torch, fn, n, stream, flush):
    """Per-call device times (ms) of fn over n calls, L2 flushed before each."""
    ts = []
    for _ in range(n):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return ts


def library_peers(torch, V, csr, dB32, O, dC, flush, stream, flops, value, reps):
    """cuSPARSE (best of its CSR algorithms, handle and preprocessing outside
    the timed call) and the engine's own CSR row-wise kernel, same B200."""
    peers = {}
    d = V.DeviceCSR(csr)
    dCp = torch.empty_like(dC)
    best = None
    for alg in (0, 1, 2, 3):
        try:
            h = V.CuSparse(d, dB32, O, dCp, alg=alg)
        except V.VcsrError:
            continue
        for _ in range(3):
            flush.zero_()
            h.run()
        ts = timed_events(torch, h.run, reps, stream, flush)
        h.close()
        g = flops / (np.mean(ts) * 1e-3) / 1e9
        if best is None or g > best[1]:
            best = (V.CuSparse.ALGS[alg], g)
    if best:
        peers["cusparse_best"] = {"alg": best[0], "gflops": round(best[1], 2),
                                  "ours_over_cusparse": round(value / best[1], 3)}
    ts = timed_events(torch, lambda: V.run_csr_spmm_gpu(csr.M, d.row_ptr, d.col, d.val, dB32,
                                                        O, dCp, stream), reps, stream, flush)
    peers["csr_rowwise_gflops"] = round(flops / (np.mean(ts) * 1e-3) / 1e9, 2)
    # The reference's launcher run_vcsr_spmm_gpu (src/kernels.cu:120-167) on
    # the engine: the plan built on the GPU from the segment-major VCSR (per
    # call in the launcher, outside its timed region as the reference's upload
    # is), then C += A*B timed; and the segment-major kernel on the VCSR itself.
    v = V.csr_to_vcsr_spmm(d, 4, 32, stream=stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pv = V.Plan.from_vcsr(v, max_O=max(O, 512), stream=stream)
    build_ms = (time.perf_counter() - t0) * 1e3
    ts = timed_events(torch, lambda: pv.spmm(dB32, dCp, stream=stream, accumulate=True), reps,
                      stream, flush)
    ts_seg = timed_events(torch, lambda: V.run_vcsr_spmm_segmented_gpu(v, dB32, O, 64, dCp,
                                                                       stream),
                          min(reps, 5), stream, flush)
    peers["drop_in_run_vcsr_spmm_gpu"] = {
        "gflops": round(flops / (np.mean(ts) * 1e-3) / 1e9, 2),
        "plan_from_vcsr_ms": round(build_ms, 1),
        "segmented_kernel_gflops": round(flops / (np.mean(ts_seg) * 1e-3) / 1e9, 2)}
    del pv, v, d, dCp
    return peers


def reference_gpu_peers(torch, V, csr, dB32, O, flush, stream, flops, reps):
    """The reference's own kernels rebuilt for sm_100a (baseline/_ref, built
    from the reference tree by baseline/Makefile), each on the input it
    takes, its own event timing around the kernel alone: csr_spmm_kernel
    (src/kernels.cu:15-33), vcsr_spmm_kernel (src/kernels.cu:37-103),
    vcsr_opt_kernel (src/vcsr_opt.cu:115-241), vcsr_seg_prefetch_kernel
    (src/vcsr_seg.cu:124-189) and aspt_spmm_kernel (src/aspt.cu:38-142).
    The VCSR kernels read the segment-major format built by the engine's GPU
    builder (bit-exact with the reference's builder up to tie order); the
    segment kernels read whole segments of B, so B gets segw padding rows."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    try:
        import ref_gpu
    except Exception as e:  # not built here
        return {"unavailable": f"baseline/_ref not built ({type(e).__name__}: {e})"}
    try:
        return ref_gpu.time_all(torch, V, csr, dB32, O, flush, stream, flops, reps)
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}


def measure(args, ctx, workload, steps, warmup, extras):
    """One workload: plan, B (broadcast under N ranks), `steps` timed steps,
    and (extras) the roofline, peers, end-to-end figure and CPU baseline."""
    torch, V, D, dist = ctx["torch"], ctx["V"], ctx["D"], ctx["dist"]
    rank, world, dev, stream = ctx["rank"], ctx["world"], ctx["dev"], ctx["stream"]
    cfg, size, O, scaling, label = WORKLOADS[workload]
    if args.size is not None and workload == args.workload:
        size, label = args.size, f"{label}@size{args.size}"
    dd = dist if world > 1 else None
    csr, row0, strong_total = D.rank_panel(cfg, size, args.seed, rank, world, scaling, align=16)
    global_nnz = D.global_nnz(csr, scaling, world, strong_total, dd, dev)
    global_M = D.sum_over_ranks(dist, csr.M, dev) if world > 1 else csr.M
    lo = 0.0 if cfg == "rmat" else -1.0
    tf32 = workload in TF32_WORKLOADS
    if not ctx.get("warm"):  # first use of the builder kernels (module load): untimed
        V.Plan(V.gen_csr("fem", 0, 600), tf32_panels=tf32)
        ctx["warm"] = True
    plan = V.Plan(csr, segw=4, bundle=32, max_O=max(O, 512), tf32_panels=tf32, target_O=O)
    info = plan.info()

    # B: filled on rank 0, replicated by one NCCL broadcast (timed apart)
    dB = torch.empty(csr.N, O, device=dev)
    bcast_ms = None
    if rank == 0 or world == 1:
        V.gen_dense_device(dB, args.seed + 1000, lo, 1.0)
    half = HALF_WORKLOADS.get(workload)
    dB32 = dB  # FP32 copy for the peers and the CPU baseline
    if half:
        dB32 = dB.to(getattr(torch, half)).float()  # the values the 16-bit path sees
        dB = dB.to(getattr(torch, half))
    if world > 1:
        torch.cuda.synchronize()
        if half:
            D.broadcast_b(dist, dB32, 0)
        D.broadcast_b(dist, dB, 0)  # first collective on this buffer: NCCL set-up
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        D.broadcast_b(dist, dB, 0)
        e1.record(stream)
        torch.cuda.synchronize()
        bcast_ms = D.max_over_ranks(dist, e0.elapsed_time(e1), dev)
    dC = torch.empty(csr.M, O, device=dev)
    flush = ctx["flush"]

    def step():
        plan.spmm(dB, dC, stream=stream)

    clocks = Clocks(ctx["gpu_id"]).launch()
    for _ in range(warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    launches = 0
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
        launches += plan.last_launches
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = D.max_over_ranks(dist, sum(per), dev) if world > 1 else sum(per)
    ms_step = total_ms / steps
    flops_step = 2.0 * global_nnz * O
    value = flops_step / (ms_step * 1e-3) / 1e9

    # roofline of the dominant kernel, per launch, on this rank
    abytes, touched = algorithmic_bytes(csr, O, 2 if half else 4)
    avg_ms = float(np.mean(per))
    achieved = abytes / (avg_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    traffic = profile_traffic(label) if world == 1 else None
    # the FP32 kernels' other bound: FMA issue.  Useful = 2*nnz*O of this
    # rank; slots = 2*union*R*O, the FMAs the vector panels issue (zeros of a
    # vector's rows included); peak = SMs x 128 FP32 lanes x 2 x max SM clock
    fp32 = None
    if not tf32:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        mhz = (clk or {}).get("sm_max_mhz") or 1965.0
        fpk = sms * 128 * 2 * mhz * 1e6 / 1e12
        useful = 2.0 * csr.nnz * O / (avg_ms * 1e-3) / 1e12
        slots = 2.0 * info["num_union"] * info["vec_rows"] * O / (avg_ms * 1e-3) / 1e12
        fp32 = {"useful_tflops": round(useful, 2), "slot_tflops": round(slots, 2),
                "peak_tflops": round(fpk, 1),
                "peak_kind": "nominal: SMs x 128 FP32 lanes x 2 x max SM clock",
                "frac_useful": round(useful / fpk, 4), "frac_slots": round(slots / fpk, 4)}
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_kind": peak_kind, "algorithmic_bytes": int(abytes),
                "kernel_ms": round(avg_ms, 5), "fp32_fma": fp32}
    # the build proper: the same plan from the CSR already in HBM (build_ms
    # above also holds the upload of a host CSR from pageable memory)
    dcsr = V.DeviceCSR(csr, dev)
    torch.cuda.synchronize()
    dplan = V.Plan(dcsr, segw=4, bundle=32, max_O=max(O, 512), tf32_panels=tf32, target_O=O)
    build_dev_ms = dplan.info()["build_ms"]
    del dplan, dcsr
    plan_info = {"vec_rows": info["vec_rows"], "units": info["num_units"],
                 "split_units": info["num_split_units"], "long_units": info["num_long_units"],
                 "cols_touched": touched, "tf32_panel_blocks": info["num_panel_blocks"],
                 "tf32_panel_nnz": info["panel_nnz"], "build_ms": round(info["build_ms"], 1),
                 "build_from_device_csr_ms": round(build_dev_ms, 1)}

    rec = {"value": round(value, 3), "ms_per_step": round(ms_step, 5),
           "config": workload_config(label, global_M, csr.N, global_nnz, O, world),
           "scaling": scaling, "plan": plan_info, "roofline": roofline,
           "gpu_launches": int(launches), "clocks": clk,
           "dtype": "tf32" if tf32 else ((({"bfloat16": "bf16", "float16": "f16"}[half])
                                          + "-in/f32-acc") if half else "f32")}
    if world > 1:
        # every rank's panel, kernel time and roofline; the limiter of the curve
        mine = {"rank": rank, "rows": csr.M, "nnz": csr.nnz, "cols_touched": touched,
                "kernel_ms": round(avg_ms, 5), "roofline_frac": round(achieved / peak, 4),
                "achieved_gbs": round(achieved, 1), "split_units": info["num_split_units"],
                "long_units": info["num_long_units"], "build_ms": round(info["build_ms"], 1)}
        ranks = [None] * world
        dist.all_gather_object(ranks, mine)
        kms = [r["kernel_ms"] for r in ranks]
        slow = int(np.argmax(kms))
        imb = max(kms) / max(1e-9, float(np.mean(kms)))
        rec["ranks"] = ranks
        rec["bcast_ms"] = round(bcast_ms, 4)
        rec["bcast_bytes"] = int(csr.N * O * (2 if half else 4))
        if imb > 1.15:
            lim = (f"row-panel imbalance: rank {slow} takes {max(kms):.3f} ms against a mean of "
                   f"{np.mean(kms):.3f} ms")
        else:
            lim = (f"per-rank kernel time (panels within {100 * (imb - 1):.0f}% of the mean; "
                   f"slowest rank {slow})")
        rec["limiter"] = lim + (f"; the one-time B broadcast ({bcast_ms:.2f} ms) is "
                                f"{bcast_ms / ms_step:.1f} steps")

    if extras and world > 1 and not half:
        # B's broadcast overlapped with the product (row panels multiplied as
        # their chunk of B arrives), timed like the step: max over ranks of
        # the device time of broadcast + product
        ts = []
        for i in range(4):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            D.broadcast_and_multiply(dist, plan, dB, dC, src=0, stream=stream)
            e1.record(stream)
            torch.cuda.synchronize()
            if i > 0:
                ts.append(D.max_over_ranks(dist, e0.elapsed_time(e1), dev))
        rec["bcast_overlapped_ms"] = round(float(np.median(ts)), 4)

    # end to end through the host-buffer entry point (pinned buffers)
    if extras and not args.no_e2e and not half:  # the host-buffer entry point takes FP32 B
        hB = torch.empty(csr.N, O, dtype=torch.float32, pin_memory=True)
        hB.copy_(dB32)  # device to pinned host, no pageable copy of B on the way
        torch.cuda.synchronize()
        hC = torch.empty(csr.M, O, dtype=torch.float32, pin_memory=True)
        for _ in range(max(3, min(5, warmup))):
            plan.spmm_host(hB.numpy(), hC.numpy(), stream=stream)
        if world > 1:
            dist.barrier()
        n_e2e = max(5, min(steps, 20))
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            plan.spmm_host(hB.numpy(), hC.numpy(), stream=stream)
        dt = (time.perf_counter() - t0) / n_e2e
        if world > 1:
            dt = D.max_over_ranks(dist, dt, dev)
        # rows the call moves (touched B rows up, C rows holding entries
        # down; the empty C rows are zeroed on the host), over all ranks
        b_rows, c_rows = plan.host_rows(stream=stream)
        if world > 1:
            b_rows = int(D.sum_over_ranks(dist, b_rows, dev))
            c_rows = int(D.sum_over_ranks(dist, c_rows, dev))
        rec["e2e"] = {"value": round(flops_step / dt / 1e9, 3), "unit": "GFLOP/s",
                      "h2d_bytes_per_step": int(b_rows * O * 4),
                      "d2h_bytes_per_step": int(c_rows * O * 4),
                      "ms_per_step": round(dt * 1e3, 4),
                      "api": "vcsr_spmm_host (pinned host B and C)"}
        del hB, hC

    if extras and not args.no_peers and world == 1:
        reps = max(5, min(steps, 20))
        rec["peers"] = library_peers(torch, V, csr, dB32, O, dC, flush, stream, flops_step,
                                     value, reps)
        rec["peers"]["reference_kernels_sm100a"] = reference_gpu_peers(
            torch, V, csr, dB32, O, flush, stream, flops_step, min(reps, 5))
    if extras and rank == 0 and world == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_baseline(csr, dB32.cpu().numpy(), args.cpu_seconds)
    del plan, dB, dB32, dC
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return rec


def run_ours(args):
    import torch
    import torch.distributed as dist
    import vcsr_b200 as V
    from vcsr_b200 import dist as D

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU (no CPU fallback)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        D.init_ranks(dist, "nccl", timeout_s=300, device=dev)
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        gpu_id = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        gpu_id = ""
    ctx = {"torch": torch, "V": V, "D": D, "dist": dist, "rank": rank, "world": world,
           "dev": dev, "stream": torch.cuda.current_stream(), "gpu_id": gpu_id,
           "flush": torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)}  # 256 MB
    main = measure(args, ctx, args.workload, args.steps, args.warmup, extras=True)
    sub = None
    if world == 1 and args.workload == "rmat" and not args.no_fem_record and args.size is None:
        sub = measure(args, ctx, "fem", max(args.steps, args.sub_steps), args.warmup,
                      extras=True)
        sub["steps"] = max(args.steps, args.sub_steps)
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": main["value"], "unit": "GFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": main["ms_per_step"], "higher_is_better": True,
                "scaling": main["scaling"], "vs_baseline": None, "dtype": main["dtype"],
                "data": "synthetic", "config": main["config"],
                "roofline": main["roofline"], "gpu_launches": main["gpu_launches"],
                "e2e": main.get("e2e"), "clocks": main["clocks"],
                "cpu_baseline": main.get("cpu_baseline"), "peers": main.get("peers"),
                "plan": main["plan"]}
        for k in ("ranks", "bcast_ms", "bcast_bytes", "bcast_overlapped_ms", "limiter"):
            if k in main:
                line[k] = main[k]
        if sub is not None:
            line["fem_o128"] = sub
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
