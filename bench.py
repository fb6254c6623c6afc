#!/usr/bin/env python
"""Benchmark of the matvecQ8 hot path on B200s (one process per GPU).

Headline workload (second part, which at N = 1 is the
1-GPU 28672 x 8192 target GEMV 80 times over): a stack of 80 Q8 matrices
[28672 x 8192] (W ~ N(0, 0.02^2), per-row absmax scales) applied to one
x ~ N(0, 1).  Rows are sharded across the N GPUs (28672 / N rows of every
matrix per GPU) and the output slices are gathered with an NCCL all-gather,
so total work is fixed as N grows (strong scaling).  A step is one pass over
the whole stack.  The weights (18.8 GB / N per GPU) are far larger than L2,
so no flush is needed between steps.

Metric: achieved HBM GB/s of algorithmic bytes (codes + scales + x + y of
every matrix; x counted once per GPU), whole job.  Also reported:
  - e2e: the same metric through the C ABI with host buffers: each step
    copies x from pinned host memory, runs the stack and the gather, and
    reads y back to pinned host memory;
  - roofline of the GEMV kernel (bytes per launch / average launch time,
    CUDA events on the launching stream) against MEASURED_PEAKS.json;
  - cpu_baseline (N = 1): the CPU oracle, a restatement of the reference's
    reference.ts, single-threaded like JavaScript, on one of the matrices;
  - decode: Q8 decode tokens/s of a ~1.1B Llama (config 4) from a 2048
    position context, 128 greedy steps, replicated on every GPU.

`--impl reference` times the reference's CPU implementation of the path
(the oracle port; the TypeScript cannot run here) with every host thread.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "web-xpu-ops_b200"))
sys.path.insert(0, str(ROOT))

MATRICES, ROWS, COLS = 80, 28672, 8192
SPEC_GBS = 8000.0  # B200 HBM3e data-sheet bandwidth
METRIC = "matvecQ8 achieved HBM GB/s vs B200 peak; Q8 decode tokens/s, 1-8 GPUs"


def parse():
    global ROWS, COLS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--matrices", type=int, default=MATRICES)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--decode-steps", type=int, default=128)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--oracle-tokens", type=int, default=4)
    ap.add_argument("--gemv", metavar="NxK", default=None,
                    help="time single matvecQ8 launches of one N x K shape instead (a profiling case)")

    ap.add_argument("--rows", type=int, default=ROWS, help=argparse.SUPPRESS)
    ap.add_argument("--cols", type=int, default=COLS, help=argparse.SUPPRESS)
    args = ap.parse_args()
    ROWS, COLS = args.rows, args.cols
    return args


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def algorithmic_bytes(rows: int, K: int, matrices: int) -> int:
    """codes + scales + y of `rows` rows per matrix, and x once (the per-launch bytes of matvecQ8, x shared)."""
    W = (K + 3) // 4
    return matrices * (rows * W * 4 + rows * 4 + rows * 4) + K * 4


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_cores_serve(M, R, K):
    """Whether XPU_MATVEC_AUTO sends this stack to the tensor cores: rows of
    whole 16-byte slots, K <= 65536, and at least 512 MiB of weights (64 MiB
    when K >= 16384) -- the library's rule; torch allocations are 16-byte
    aligned."""
    W = (K + 3) // 4
    b = M * R * W * 4
    return W % 4 == 0 and (R * W) % 4 == 0 and K <= 65536 and (b >= 512 << 20 or (K >= 16384 and b >= 64 << 20))


def ncu_traffic(kernel: str, rows: int, cols: int):
    """DRAM bytes (read + write) of one launch over this rank's rows, from
    the ncu capture summarised in profiles/ncu_traffic.json (taken on one
    GPU over all 28672 rows; traffic scales with the rows streamed), and
    the capture's command.  (None, None) when there is no capture."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None, None
    e = json.loads(p.read_text()).get(f"{kernel}_{ROWS}x{cols}")
    if not e:
        return None, None
    return round(e["bytes_per_launch"] * rows / ROWS), e["command"]


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.idx = {str(i) for i in gpu_indices}
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) == 9 and f[0] in self.idx:
                rows.append(f)
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


# ------------------------------------------------------------- our arm ---

def build_stack(torch, ops, rank, world, matrices, stream):
    """This GPU's row shard of every matrix, generated and quantized on the
    device: rows [rank*R, (rank+1)*R) of matrix m are elements
    [rank*R*K, (rank+1)*R*K) of the seed-m stream, the same for any N."""
    from xpuops.synth import tensor_seed

    R, K, W = ROWS // world, COLS, COLS // 4
    dev = torch.device("cuda", torch.cuda.current_device())
    weights = torch.empty(matrices * R * W, dtype=torch.int32, device=dev)
    scales = torch.empty(matrices * R, dtype=torch.float32, device=dev)
    tmp = torch.empty(R * K, dtype=torch.float32, device=dev)
    for m in range(matrices):
        ops.fill_normal_dev(tmp, R * K, tensor_seed(0, m), 0.0, 0.02, stream=stream, start=rank * R * K)
        ops.quantizePackQ8_dev(tmp, R, K, weights.data_ptr() + 4 * m * R * W, scales.data_ptr() + 4 * m * R,
                               stream=stream)
    x = torch.empty(K, dtype=torch.float32, device=dev)
    ops.fill_normal_dev(x, K, tensor_seed(1, 0), 0.0, 1.0, stream=stream)
    torch.cuda.synchronize()
    del tmp
    return weights, scales, x, R


def check_stack_output(torch, dist, ops, rank, world, weights, scales, x, M, R, K, y_dev, to_host):
    """The last timed step's output against the oracle
    (ops/matvec/reference.ts:117-131): 8 rows of this rank's shard in the
    first and the last matrix, from the weights this GPU streamed, checked
    in every rank's copy of the output (at N > 1 the rows other GPUs'
    epilogues wrote into it) within 1e-5 * |scale| * sum|code * x| plus one
    f32 ulp."""
    import oracle.oracle as orc

    W = K // 4
    xh = x.cpu().numpy()
    mine = []
    for m in sorted({0, M - 1}):
        for i in np.linspace(0, R - 1, 8).astype(np.int64):
            r = m * R + int(i)
            wrow = weights[r * W:(r + 1) * W].cpu().numpy().view(np.uint32)
            srow = scales[r:r + 1].cpu().numpy()
            want = float(orc.matvec_q8(wrow, srow, xh, 1, K)[0])
            bound = float(orc.matvec_q8_bound(wrow, srow, xh, 1, K)[0])
            mine.append((m * world * R + rank * R + int(i), want, bound))
    rows = [mine]
    if world > 1:
        rows = [None] * world
        dist.all_gather_object(rows, mine)
    yh = torch.empty(world * M * R, dtype=torch.float32).pin_memory()
    to_host(yh, y_dev)
    torch.cuda.synchronize()
    yh = yh.numpy()
    worst, n = 0.0, 0
    for part in rows:
        for idx, want, bound in part:
            lim = 1e-5 * bound + float(np.spacing(np.float32(abs(want))))
            worst = max(worst, abs(float(yh[idx]) - want) / lim)
            n += 1
    verdicts = [(worst, n)]
    if world > 1:
        verdicts = [None] * world
        dist.all_gather_object(verdicts, (worst, n))
    w = max(v[0] for v in verdicts)
    return {"rows_checked": int(sum(v[1] for v in verdicts)), "within_bound": bool(w <= 1.0),
            "worst_error_over_bound": round(w, 6),
            "what": "sampled rows of the first and last matrix of every shard, against the oracle, read from "
                    "every GPU's copy of the output"}


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist

    from xpuops import ops

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    M, K = args.matrices, COLS
    # This GPU's own read ceiling, measured now (harness/roofline.ts
    # measureRoofline): one pass over a hash-filled 2 GiB buffer, fastest of 5.
    probe = ops.measureRoofline()
    weights, scales, x, R = build_stack(torch, ops, rank, world, M, sp)
    W = K // 4
    y_local = torch.empty(M * R, dtype=torch.float32, device="cuda")
    y_full = torch.empty(world * M * R, dtype=torch.float32, device="cuda")
    # N > 1: the all-gather is fused into the GEMV (xpu_matvec_q8_stack_allgather_dev):
    # its epilogue writes every row into every GPU's output over NVLink, the
    # outputs mapped across the processes with CUDA IPC; two output buffers
    # in turn, as a rank may run one call ahead.
    fused = None
    if world > 1:
        outs = [ops.DeviceBuffer(4 * world * M * R) for _ in range(2)]
        flags = ops.DeviceBuffer(4 * world)
        flags.upload(np.zeros(world, np.uint32))
        every = [None] * world
        dist.all_gather_object(every, [ops.ipcHandle(o) for o in outs] + [ops.ipcHandle(flags)])
        maps = [[ops.ipcOpen(h) for h in every[r]] if r != rank else [o.ptr for o in outs] + [flags.ptr]
                for r in range(world)]
        fused = {"outs": outs, "flags": flags, "maps": maps, "epoch": 0}

    def gemv():
        if fused is None:
            ops.matvecQ8Stack_dev(weights, R * W, scales, x, M, R, K, y_local, sp)
            return y_local
        fused["epoch"] += 1
        b = fused["epoch"] % 2
        ops.matvecQ8StackAllGather_dev(weights, R * W, scales, x, M, R, K, rank, world,
                                       [fused["maps"][r][b] for r in range(world)],
                                       [fused["maps"][r][2] for r in range(world)], fused["epoch"], sp)
        return fused["outs"][b]

    def step():
        return gemv()

    def to_host(dst, src):
        if isinstance(src, torch.Tensor):
            dst.copy_(src, non_blocking=True)
        else:  # a library buffer (the fused path's outputs)
            from xpuops._lib import check, lib
            check(lib().xpu_memcpy_d2h(dst.data_ptr(), src.ptr, dst.numel() * 4, sp))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        step()
    sampler = ClockSampler([physical_gpu(i) for i in range(world)]) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0.record(stream)
    last = None
    for i in range(args.steps):
        g_events[i][0].record(stream)
        last = gemv()
        g_events[i][1].record(stream)
    t1.record(stream)
    barrier()
    clocks = sampler.stop() if sampler else None
    total_ms = max_over_ranks(t0.elapsed_time(t1))
    gemv_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in g_events))
    output_check = check_stack_output(torch, dist, ops, rank, world, weights, scales, x, M, R, K, last, to_host)

    # The same stack with an NCCL all-gather after each GEMV (the unfused
    # form; comparison only).
    nccl = None
    if world > 1:
        for _ in range(2):
            ops.matvecQ8Stack_dev(weights, R * W, scales, x, M, R, K, y_local, sp)
            dist.all_gather_into_tensor(y_full, y_local)
        barrier()
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_steps = max(3, args.steps // 2)
        n0.record(stream)
        for _ in range(n_steps):
            ops.matvecQ8Stack_dev(weights, R * W, scales, x, M, R, K, y_local, sp)
            dist.all_gather_into_tensor(y_full, y_local)
        n1.record(stream)
        barrier()
        nccl_ms = max_over_ranks(n0.elapsed_time(n1)) / n_steps
        nccl = {"ms_per_step": round(nccl_ms, 4),
                "value": round(algorithmic_bytes(R, K, M) * world / (nccl_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "what": "the same stack, then one NCCL all-gather per step (unfused)"}

    bytes_rank = algorithmic_bytes(R, K, M)
    bytes_job = bytes_rank * world
    value = bytes_job * args.steps / (total_ms / 1e3) / 1e9
    # One persistent GEMV launch per step over the stack, on the tensor-core
    # path preceded by its vector-statistics kernel (inside the same events).
    avg_launch_s = gemv_ms / 1e3 / args.steps
    achieved = bytes_rank / avg_launch_s / 1e9
    peak, peak_src = measured_peaks()
    on_tc = tensor_cores_serve(M, R, K)
    kname = "mv_tc_kernel" if on_tc else "mv_bulk_kernel"
    traffic, traffic_cmd = ncu_traffic(kname, R, K)
    launches_per_step = 2 if on_tc or world > 1 else 1  # mv_xstat_kernel + mv_tc_kernel

    # The other matvecQ8 path, pinned, on the same stack (comparison only).
    ops.setMatvecPath(ops.MATVEC_CUDA_CORES if on_tc else ops.MATVEC_TENSOR_CORES)
    try:
        for _ in range(2):
            ops.matvecQ8Stack_dev(weights, R * W, scales, x, M, R, K, y_local, sp)
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        alt_steps = max(3, args.steps // 2)
        a0.record(stream)
        for _ in range(alt_steps):
            ops.matvecQ8Stack_dev(weights, R * W, scales, x, M, R, K, y_local, sp)
        a1.record(stream)
        barrier()
        alt_ms = max_over_ranks(a0.elapsed_time(a1)) / alt_steps
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)
    alt = {"path": "cuda_cores (mv_bulk_kernel)" if on_tc else "tensor_cores (mv_tc_kernel)",
           "value": round(bytes_job / (alt_ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(alt_ms, 4),
           "steps": alt_steps}

    # e2e: host x in, host y out, through the C ABI, per step
    x_host = torch.empty(K, dtype=torch.float32).pin_memory()
    x_host.copy_(x.cpu())
    y_host = torch.empty(world * M * R, dtype=torch.float32).pin_memory()
    for _ in range(3):
        x.copy_(x_host, non_blocking=True)
        to_host(y_host, step())
        stream.synchronize()
    e2e_steps = max(10, args.steps // 4)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        x.copy_(x_host, non_blocking=True)
        to_host(y_host, step())
        stream.synchronize()  # the host reads y every step
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = bytes_job * e2e_steps / (e2e_ms / 1e3) / 1e9

    target = None
    if world == 1 and M >= 8:
        target = run_target_gemv(torch, ops, weights, scales, x, R, K, sp, probe["bandwidth"] / 1e9)

    quant = run_quantize(torch, ops, sp) if world == 1 and rank == 0 else None
    small = run_small_configs(torch, ops, sp) if world == 1 and rank == 0 else None
    lm_head = run_lm_head(args, torch, ops, dist, rank, world, sp, barrier, max_over_ranks)

    decode = None
    if not args.no_decode:
        decode = run_decode(args, torch, world, max_over_ranks, barrier)

    cpu = None
    if world == 1 and rank == 0:
        cpu = cpu_baseline(weights, scales, x, R, K, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int8*f32",
            "data": "synthetic (seeded N(0, 0.02^2) weights quantized per row, x ~ N(0, 1))",
            "config": {
                "workload": f"matvecQ8 stack: {M} x [{ROWS} x {COLS}] Q8 on one x, rows sharded over {world} GPU(s)"
                            + (", NCCL all-gather of y" if world > 1 else ""),
                "matrices": M, "N": ROWS, "K": COLS, "rows_per_gpu": R,
                "bytes_per_step": bytes_job, "l2": "no flush: 18.8 GB / N of weights per step >> 126 MB L2",
                "parallelism": f"row-shard x{world}",
                "gather": ("fused into the GEMV: its epilogue writes every row into every GPU's output over NVLink "
                           "(CUDA IPC mappings), then a flag per GPU") if world > 1 else None,
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "stream_probe": {"gbs": round(probe["bandwidth"] / 1e9, 1),
                                          "frac": round(achieved / (probe["bandwidth"] / 1e9), 4),
                                          "load_gbs": round(probe["loadBandwidth"] / 1e9, 1),
                                          "bulk_gbs": round(probe["bulkBandwidth"] / 1e9, 1),
                                          "how": "xpu_measure_roofline in this run: one read pass over a "
                                                 "hash-filled 2 GiB buffer, fastest of 5 after a warm-up; the "
                                                 "faster of 16-byte loads and bulk copies"},
                         "spec": {"gbs": SPEC_GBS, "frac": round(achieved / SPEC_GBS, 4)},
                         "traffic": traffic, "traffic_source": traffic_cmd,
                         "kernel": ("mv_tc_kernel (matvecQ8 on tcgen05 tensor cores, x as exact int8 limbs): one "
                                    "persistent stream-K launch per step over the stack" if on_tc else
                                    "mv_bulk_kernel (matvecQ8, bulk-copy path): one launch per step over the contiguous stack"),
                         "launch_ms": round(avg_launch_s * 1e3, 5)},
            "other_path": alt,
            "nccl_gather": nccl,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": K * 4,
                    "d2h_bytes_per_step": world * M * R * 4, "ms_per_step": round(e2e_ms / e2e_steps, 4)},
            "gpu_launches": args.steps * world * launches_per_step,
            "gpu_launches_per_rank": args.steps * launches_per_step,
            "target_gemv": target,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "decode": decode,
            "quantize": quant,
            "output_check": output_check,
            "configs_1_3": small,
            "lm_head": lm_head,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # no rank still writes into a mapped output
        if fused is not None:
            for r in range(world):
                if r != rank:
                    for ptr in fused["maps"][r]:
                        ops.ipcClose(ptr)
        dist.barrier()
        dist.destroy_process_group()


def run_target_gemv(torch, ops, weights, scales, x, R, K, sp, stream_gbs):
    """The BASELINE target: single matvecQ8 GEMVs, each its own launch (no
    fusion), 28672 x 8192 (matrices of the stack) and 8192 x 28672 (eight
    fresh matrices), plus config 2's rows that are not whole 16-byte slots,
    11008 x 4097 and 8192 x 28676, rotating over the matrices so that L2 never
    holds the weights being read.  CUDA events on the launching stream.  The
    aligned shapes are timed under the library's default choice
    (XPU_MATVEC_AUTO) and on each path pinned; every entry names the kernel
    AUTO ran and adds `graph_us`, the same launches replayed from a CUDA graph
    (no host submission between them), which separates the fixed cost of a
    launch from the kernel's streaming rate."""
    from xpuops.synth import tensor_seed

    peak, _ = measured_peaks()
    out = {}
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

    def time_launches(launch, n, reps=5):
        for i in range(n):
            launch(i, sp)
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(reps):
            for i in range(n):
                launch(i, sp)
        ev[1].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) / 1e3 / (reps * n)

    def time_graph(launch, n, reps=5):
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                for _ in range(reps):
                    for i in range(n):
                        launch(i, cs.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        ev[0].record()
        g.replay()
        ev[1].record()
        torch.cuda.synchronize()
        t = ev[0].elapsed_time(ev[1]) / 1e3 / (reps * n)
        del g
        return t

    def fig(b, t):
        return {"us": round(t * 1e6, 2), "GBs": round(b / t / 1e9, 1), "frac": round(b / t / 1e9 / peak, 4),
                "frac_stream_probe": round(b / t / 1e9 / stream_gbs, 4),
                "frac_spec": round(b / t / 1e9 / SPEC_GBS, 4)}

    def kernel_name(N, Kx):
        Wx = (Kx + 3) // 4
        if Wx % 4 == 0:
            return "mv_tc_kernel" if tensor_cores_serve(1, N, Kx) else "mv_bulk_kernel"
        # the planner's rule for rows off the 16-byte grid (csrc/matvec.cu)
        uc = (Wx + 6) // 4
        ncw = min(max(-(-uc // 32), 1), 16)
        cpt = -(-uc // (32 * ncw))
        if cpt >= 4:
            cpt = -(-uc // (32 * 14))
        return "mv_ragged_kernel" if N * Wx * 4 >= (16 << 20) and cpt <= 4 else "mv_gen_kernel"

    def entry(N, Kx, launch, n, paths=True):
        b = algorithmic_bytes(N, Kx, 1)
        res = {}
        for name, path in (("auto", ops.MATVEC_AUTO), ("cuda_cores", ops.MATVEC_CUDA_CORES),
                           ("tensor_cores", ops.MATVEC_TENSOR_CORES)):
            if name != "auto" and not paths:
                continue
            ops.setMatvecPath(path)
            try:
                res[name] = fig(b, time_launches(launch, n))
            finally:
                ops.setMatvecPath(ops.MATVEC_AUTO)
        res["auto"]["kernel"] = kernel_name(N, Kx)
        res["auto"]["graph_us"] = round(time_graph(launch, n) * 1e6, 2)
        res["auto"]["graph_frac"] = round(b / (res["auto"]["graph_us"] * 1e-6) / 1e9 / peak, 4)
        return res

    def fresh(N2, K2, count, seed):
        W2 = (K2 + 3) // 4
        w2 = torch.empty(count * N2 * W2, dtype=torch.int32, device="cuda")
        s2 = torch.empty(count * N2, dtype=torch.float32, device="cuda")
        tmp = torch.empty(N2 * K2, dtype=torch.float32, device="cuda")
        for i in range(count):
            ops.fill_normal_dev(tmp, N2 * K2, tensor_seed(seed, i), 0.0, 0.02, stream=sp)
            ops.quantizePackQ8_dev(tmp, N2, K2, w2.data_ptr() + 4 * i * N2 * W2, s2.data_ptr() + 4 * i * N2,
                                   stream=sp)
        del tmp
        x2 = torch.empty(K2, dtype=torch.float32, device="cuda")
        ops.fill_normal_dev(x2, K2, tensor_seed(seed + 1, 0), stream=sp)
        y2 = torch.empty(N2, dtype=torch.float32, device="cuda")

        def launch(i, st):
            ops.matvecQ8_dev(w2.data_ptr() + 4 * i * N2 * W2, s2.data_ptr() + 4 * i * N2, x2, N2, K2, y2, st)
        return launch, (w2, s2, x2, y2)

    W = K // 4
    y = torch.empty(R, dtype=torch.float32, device="cuda")
    n = min(16, weights.numel() // (R * W))
    out[f"{R}x{K}"] = entry(R, K, lambda i, st: ops.matvecQ8_dev(weights.data_ptr() + 4 * i * R * W,
                                                                 scales.data_ptr() + 4 * i * R, x, R, K, y, st), n)
    for (N2, K2, count, seed, paths) in ((K, R, 8, 2, True), (11008, 4097, 16, 20, False),
                                         (8192, 28676, 8, 22, False)):
        launch, keep = fresh(N2, K2, count, seed)
        out[f"{N2}x{K2}"] = entry(N2, K2, launch, count, paths)
        del keep
    out["note"] = ("each GEMV its own launch (xpu_matvec_q8_dev), rotating over 8-16 matrices; auto = the "
                   "library's default path choice, whose kernel is named; frac of measured HBM peak; graph_us = "
                   "the same launches replayed from one CUDA graph; 11008x4097 and 8192x28676 (config 2, rows off "
                   "the 16-byte grid) have no tensor-core path")
    return out


def run_lm_head(args, torch, ops, dist, rank, world, sp, barrier, max_over_ranks):
    """Config 5(i): the LM-head shape, one Q8 GEMV of N = 128256 rows and
    K = 8192 (1.05 GB of codes), rows sharded over the N GPUs and the output
    slices all-gathered every step: at N > 1 both by the tensor-core GEMV
    itself (xpu_matvec_q8_stack_allgather_dev, outputs mapped over CUDA IPC;
    the line's figure) and, for comparison, by the library default GEMV then
    one NCCL all-gather.  Weights are generated on the device, each GPU its
    own rows of the same seeded matrix."""
    from xpuops.synth import tensor_seed

    N, K = 128256, 8192
    if N % world:
        return None
    R, W = N // world, K // 4
    w = torch.empty(R * W, dtype=torch.int32, device="cuda")
    s = torch.empty(R, dtype=torch.float32, device="cuda")
    tmp = torch.empty(R * K, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(tmp, R * K, tensor_seed(5, 0), 0.0, 0.02, stream=sp, start=rank * R * K)
    ops.quantizePackQ8_dev(tmp, R, K, w, s, stream=sp)
    del tmp
    x = torch.empty(K, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(x, K, tensor_seed(5, 1), stream=sp)
    y = torch.empty(R, dtype=torch.float32, device="cuda")
    y_full = torch.empty(N, dtype=torch.float32, device="cuda")

    def step():
        ops.matvecQ8_dev(w, s, x, R, K, y, sp)
        if world > 1:
            dist.all_gather_into_tensor(y_full, y)

    def timed(fn):
        for _ in range(5):
            fn()
        barrier()
        steps = max(20, args.steps // 4)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        barrier()
        return steps, max_over_ranks(e0.elapsed_time(e1)) / steps

    byts = algorithmic_bytes(R, K, 1) * world
    steps, ms = timed(step)
    nccl = {"workload": f"matvecQ8 LM head [{N} x {K}], rows sharded over {world} GPU(s)"
                        + (", NCCL all-gather of y every step" if world > 1 else ""),
            "steps": steps, "ms_per_step": round(ms, 4), "GBs": round(byts / (ms / 1e3) / 1e9, 1),
            "rows_per_gpu": R, "kernel": "mv_tc_kernel" if tensor_cores_serve(1, R, K) else "mv_bulk_kernel"}
    if world == 1:
        del w, s
        return nccl
    # The all-gather fused into the tensor-core GEMV: two output buffers in
    # turn and a flag array of its own, mapped into every rank.
    outs = [ops.DeviceBuffer(4 * N) for _ in range(2)]
    flags = ops.DeviceBuffer(4 * world)
    flags.upload(np.zeros(world, np.uint32))
    every = [None] * world
    dist.all_gather_object(every, [ops.ipcHandle(o) for o in outs] + [ops.ipcHandle(flags)])
    maps = [[ops.ipcOpen(h) for h in every[r]] if r != rank else [o.ptr for o in outs] + [flags.ptr]
            for r in range(world)]
    state = {"epoch": 0}

    def fused_step():
        state["epoch"] += 1
        b = state["epoch"] % 2
        ops.matvecQ8StackAllGather_dev(w, R * W, s, x, 1, R, K, rank, world, [maps[r][b] for r in range(world)],
                                       [maps[r][2] for r in range(world)], state["epoch"], sp)

    fsteps, fms = timed(fused_step)
    torch.cuda.synchronize()
    dist.barrier()  # no rank still writes into a mapped output
    for r in range(world):
        if r != rank:
            for ptr in maps[r]:
                ops.ipcClose(ptr)
    dist.barrier()
    del w, s
    return {"workload": f"matvecQ8 LM head [{N} x {K}], rows sharded over {world} GPU(s), the all-gather fused into "
                        "the tensor-core GEMV (every row stored into every GPU's output over NVLink)",
            "steps": fsteps, "ms_per_step": round(fms, 4), "GBs": round(byts / (fms / 1e3) / 1e9, 1),
            "rows_per_gpu": R, "kernel": "mv_tc_kernel", "nccl_gather": nccl}


def run_quantize(torch, ops, sp):
    """ops/quantize/reference.ts `quantize` + ops/matvec/reference.ts `packQ8`
    fused on the device (xpu_quantize_pack_q8_dev), config 1's 4096 x 4096 f32
    weights, rotating over 8 matrices (512 MB, past L2); bytes = f32 read +
    packed words and scales written.  Beside it the oracle's quantize + pack
    of the same matrix on one thread."""
    import oracle.oracle as orc
    from xpuops.synth import tensor_seed

    N = K = 4096
    W = K // 4
    f = torch.empty(8, N * K, dtype=torch.float32, device="cuda")
    for i in range(8):
        ops.fill_normal_dev(f[i], N * K, tensor_seed(0, i), 0.0, 0.02, stream=sp)
    w = torch.empty(N * W, dtype=torch.int32, device="cuda")
    s = torch.empty(N, dtype=torch.float32, device="cuda")
    for i in range(8):
        ops.quantizePackQ8_dev(f[i], N, K, w, s, stream=sp)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        for i in range(8):
            ops.quantizePackQ8_dev(f[i], N, K, w, s, stream=sp)
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / (8 * reps)
    b = 4 * N * K + 4 * N * W + 4 * N
    peak, _ = measured_peaks()
    host = f[7].cpu().numpy()
    c0 = time.perf_counter()
    codes, sc = orc.quantize(host, N, K)
    packed = orc.pack_q8(codes, N, K)
    ct = time.perf_counter() - c0
    exact = bool(np.array_equal(packed, w.cpu().numpy().view(np.uint32)) and np.array_equal(sc, s.cpu().numpy()))
    return {"workload": "quantize + packQ8 of config 1 (4096 x 4096 f32, N(0, 0.02^2))",
            "us": round(t * 1e6, 2), "GBs": round(b / t / 1e9, 1), "frac": round(b / t / 1e9 / peak, 4),
            "bit_exact_vs_oracle": exact,
            "cpu_baseline": {"us": round(ct * 1e6, 1), "GBs": round(b / ct / 1e9, 4), "cores": 1, "kind": "port",
                             "sample": "the oracle's quantize + pack of the same matrix, one pass, one thread"}}


def run_small_configs(torch, ops, sp):
    """BASELINE configs 1 and 3 as GPU launches with the oracle beside them
    (one thread, as JavaScript runs reference.ts): config 1's single
    4096 x 4096 matvecQ8, and config 3's decoder-layer GEMVs (hidden 2048,
    16 query / 4 KV heads of 128: q 2048 x 2048, k and v 512 x 2048, o
    2048 x 2048, gate/up 5632 x 2048 as one matvecQ8Ffn, down 2048 x 5632).
    Each GPU figure rotates over 8 copies of its matrices (past L2) with
    CUDA events around 5 rounds; each result is checked against the oracle
    within the matvecQ8 bound."""
    import oracle.oracle as orc
    from xpuops.synth import tensor_seed

    peak, _ = measured_peaks()

    def weights(N, K, seed, copies=8):
        W = (K + 3) // 4
        w = torch.empty(copies, N * W, dtype=torch.int32, device="cuda")
        sc = torch.empty(copies, N, dtype=torch.float32, device="cuda")
        tmp = torch.empty(N * K, dtype=torch.float32, device="cuda")
        for i in range(copies):
            ops.fill_normal_dev(tmp, N * K, tensor_seed(seed, i), 0.0, 0.02, stream=sp)
            ops.quantizePackQ8_dev(tmp, N, K, w[i], sc[i], stream=sp)
        return w, sc

    def timed(launch, reps=5, copies=8):
        for i in range(copies):
            launch(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for i in range(copies):
                launch(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / (reps * copies)

    out = {}
    # Config 1.
    N = K = 4096
    w, sc = weights(N, K, 50)
    x = torch.empty(K, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(x, K, tensor_seed(51, 0), stream=sp)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    t = timed(lambda i: ops.matvecQ8_dev(w[i], sc[i], x, N, K, y, sp))
    wh, sh, xh = w[7].cpu().numpy().view(np.uint32), sc[7].cpu().numpy(), x.cpu().numpy()
    c0 = time.perf_counter()
    want = orc.matvec_q8(wh, sh, xh, N, K)
    ct = time.perf_counter() - c0
    ops.matvecQ8_dev(w[7], sc[7], x, N, K, y, sp)
    got = y.cpu().numpy()
    lim = 1e-5 * orc.matvec_q8_bound(wh, sh, xh, N, K) + np.spacing(np.abs(want).astype(np.float32))
    ok = bool(np.all(np.abs(got.astype(np.float64) - want) <= lim))
    b = algorithmic_bytes(N, K, 1)
    out["config1"] = {"workload": "matvecQ8 4096 x 4096 (seeded N(0, 0.02^2) weights, x ~ N(0, 1))",
                      "us": round(t * 1e6, 2), "GBs": round(b / t / 1e9, 1), "frac": round(b / t / 1e9 / peak, 4),
                      "within_bound_of_oracle": ok,
                      "cpu_baseline": {"us": round(ct * 1e6, 1), "GBs": round(b / ct / 1e9, 4), "cores": 1,
                                       "kind": "port", "sample": "the oracle's matvecQ8 of the same matrix, once"}}
    del w, sc
    # Config 3.
    h, kv, ffn = 2048, 512, 5632
    layer = [("q", h, h), ("k", kv, h), ("v", kv, h), ("o", h, h), ("gate", ffn, h), ("up", ffn, h),
             ("down", h, ffn)]
    mats = {name: weights(n, k, 60 + j) for j, (name, n, k) in enumerate(layer)}
    xs = {k: torch.empty(k, dtype=torch.float32, device="cuda") for k in (h, ffn)}
    for k, v in xs.items():
        ops.fill_normal_dev(v, k, tensor_seed(70, k), stream=sp)
    ys = {n: torch.empty(n, dtype=torch.float32, device="cuda") for n in (h, kv, ffn)}

    rows = {name: n for name, n, _ in layer}

    def layer_launch(i, st=None):
        st = st or sp
        for name in ("q", "k", "v", "o"):
            ops.matvecQ8_dev(mats[name][0][i], mats[name][1][i], xs[h], rows[name], h, ys[rows[name]], st)
        ops.matvecQ8Ffn_dev(mats["gate"][0][i], mats["gate"][1][i], mats["up"][0][i], mats["up"][1][i], xs[h], ffn,
                            h, ys[ffn], st)
        ops.matvecQ8_dev(mats["down"][0][i], mats["down"][1][i], xs[ffn], h, ffn, ys[h], st)

    t = timed(layer_launch)
    # The same launches replayed from one CUDA graph (no host submission
    # between them).
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    with torch.cuda.stream(cs):
        with torch.cuda.graph(g, stream=cs):
            for _ in range(5):
                for i in range(8):
                    layer_launch(i, cs.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    tg = e0.elapsed_time(e1) / 1e3 / 40
    del g
    b = sum(algorithmic_bytes(n, k, 1) for _, n, k in layer)
    host = {name: (m[0][7].cpu().numpy().view(np.uint32), m[1][7].cpu().numpy()) for name, m in mats.items()}
    xh = {k: v.cpu().numpy() for k, v in xs.items()}
    c0 = time.perf_counter()
    for name, n, k in layer:
        if name == "gate":
            orc.matvec_q8_ffn(host["gate"][0], host["gate"][1], host["up"][0], host["up"][1], xh[h], n, k)
        elif name != "up":
            orc.matvec_q8(host[name][0], host[name][1], xh[k], n, k)
    ct = time.perf_counter() - c0
    out["config3"] = {"workload": "one decoder layer's decode GEMVs: q 2048x2048, k/v 512x2048, o 2048x2048, "
                                  "gate/up 5632x2048 (one matvecQ8Ffn), down 2048x5632; 6 launches",
                      "us": round(t * 1e6, 2), "GBs": round(b / t / 1e9, 1), "frac": round(b / t / 1e9 / peak, 4),
                      "graph_us": round(tg * 1e6, 2), "graph_frac": round(b / tg / 1e9 / peak, 4),
                      "cpu_baseline": {"us": round(ct * 1e6, 1), "GBs": round(b / ct / 1e9, 4), "cores": 1,
                                       "kind": "port", "sample": "the oracle's GEMVs of the same layer, once"}}
    return out


def cpu_baseline(weights, scales, x, R, K, seconds):
    """The oracle (a restatement of ops/matvec/reference.ts#matvecQ8, f64,
    single-threaded like JavaScript) on matrix 0, repeated for ~`seconds`."""
    import oracle.oracle as orc

    W = K // 4
    w = weights[: R * W].cpu().numpy().view(np.uint32)
    s = scales[:R].cpu().numpy()
    xv = x.cpu().numpy()
    passes, t0 = 0, time.perf_counter()
    while True:
        orc.matvec_q8(w, s, xv, R, K)
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds or passes >= 200:
            break
    gbs = algorithmic_bytes(R, K, 1) * passes / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"matrix 0 of the stack ([{R} x {K}]), {passes} passes, {el:.1f} s, single thread",
            "cpu": _cpu_model()}


def _cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip() + f" x{os.cpu_count()}"
    except OSError:
        pass
    return f"{os.cpu_count()} cpus"


def decode_bytes_per_token(cfg, pos: int) -> int:
    """Algorithmic bytes of one decode step at position `pos` (the cache
    holds pos + 1 entries once this step's K/V are written)."""
    c = cfg
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    per_layer_rows = q + 2 * kv + c.hiddenSize + 2 * c.ffnHidden + c.hiddenSize
    per_layer_codes = (q + 2 * kv) * c.hiddenSize + c.hiddenSize * q + 2 * c.ffnHidden * c.hiddenSize + \
        c.hiddenSize * c.ffnHidden
    codes = c.numLayers * per_layer_codes + c.vocabSize * c.hiddenSize
    scales = 4 * (c.numLayers * per_layer_rows + c.vocabSize)
    norms = 4 * c.hiddenSize * (2 * c.numLayers + 1)
    kv_read = c.numLayers * 2 * c.numKvHeads * (pos + 1) * c.headDim * 4
    kv_write = c.numLayers * 2 * kv * 4
    return codes + scales + norms + kv_read + kv_write + c.hiddenSize * 2


def random_q8_linear_dev(torch, ops, rows, cols, seed, std=0.02):
    """Seeded N(0, std^2) weights quantized on the device, returned as host
    int8 codes + f32 scales (the engine's QuantizedLinear input)."""
    from xpuops.llama import QuantizedLinear

    f = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(f, rows * cols, seed, 0.0, std, stream=torch.cuda.current_stream().cuda_stream)
    codes = torch.empty(rows * cols, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    ops.quantize_dev(f, rows, cols, codes, sc, stream=torch.cuda.current_stream().cuda_stream)
    return QuantizedLinear(codes.to(torch.int8).cpu().numpy(), sc.cpu().numpy())


def run_decode(args, torch, world, max_over_ranks, barrier):
    """Config 4: random-init ~1.1B Llama, f32 KV cache prefilled with N(0, 1)
    to 2048 positions, 128 greedy steps from a random token id."""
    from xpuops import LLAMA_1B_DECODE_CONFIG, LlamaEngineQ8Resident, ops
    from xpuops.llama import LlamaLayerWeightsQ8, LlamaWeightsQ8
    from xpuops.synth import tensor_seed

    cfg = LLAMA_1B_DECODE_CONFIG
    c = cfg
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    idx = iter(range(100_000))
    lin = lambda n, k: random_q8_linear_dev(torch, ops, n, k, tensor_seed(40, next(idx)))
    ones = np.ones(c.hiddenSize, np.float32)  # HF default RMSNorm init
    layers = [LlamaLayerWeightsQ8(attnNorm=ones, wq=lin(q, c.hiddenSize), wk=lin(kv, c.hiddenSize),
                                  wv=lin(kv, c.hiddenSize), wo=lin(c.hiddenSize, q), ffnNorm=ones,
                                  wGate=lin(c.ffnHidden, c.hiddenSize), wUp=lin(c.ffnHidden, c.hiddenSize),
                                  wDown=lin(c.hiddenSize, c.ffnHidden)) for _ in range(c.numLayers)]
    weights = LlamaWeightsQ8(embedTokens=random_q8_linear_dev(torch, ops, c.vocabSize, c.hiddenSize,
                                                              tensor_seed(40, next(idx))),
                             layers=layers, finalNorm=ones, lmHead=lin(c.vocabSize, c.hiddenSize))
    ctx = 2048
    rng = np.random.default_rng(41)
    eng = LlamaEngineQ8Resident.create(cfg, weights, torch.cuda.current_device())
    try:
        kvs = []
        for l in range(c.numLayers):
            k = rng.standard_normal(c.numKvHeads * ctx * c.headDim, dtype=np.float32)
            v = rng.standard_normal(c.numKvHeads * ctx * c.headDim, dtype=np.float32)
            eng.setKv(l, k, v, ctx)
            kvs.append((k, v))
        kv0 = kvs[0]
        first = int(rng.integers(0, c.vocabSize))
        warm = 3
        es = torch.cuda.ExternalStream(eng.stream())

        def timed(path):
            # setKv of one layer puts the position back to ctx; the other
            # layers' rows >= ctx are rewritten before they are read.
            eng.setDecodePath(path)
            eng.setKv(0, kv0[0], kv0[1], ctx)
            eng.greedySteps(first, warm)
            barrier()
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record(es)
            toks = eng.greedySteps(first, args.decode_steps)
            d1.record(es)
            d1.synchronize()
            return max_over_ranks(d0.elapsed_time(d1)), toks

        from xpuops import XpuInvalidArgument

        default = eng.decodePath
        GRAPH, PERSISTENT = LlamaEngineQ8Resident.DECODE_GRAPH, LlamaEngineQ8Resident.DECODE_PERSISTENT
        paths = [default]
        try:
            other = PERSISTENT if default == GRAPH else GRAPH
            eng.setDecodePath(other)
            paths.append(other)
        except XpuInvalidArgument:
            pass
        res = {pth: timed(pth) for pth in reversed(paths)}
        eng.setDecodePath(default)
        ms, toks = res[default]
        # host-API decode (forward(), logits copied to the host every token)
        h0 = time.perf_counter()
        n_host = min(32, args.decode_steps)
        tok = int(toks[-1])
        for _ in range(n_host):
            (logits,) = eng.forward([tok])
            tok = int(np.argmax(logits))
        host_ms = max_over_ranks((time.perf_counter() - h0) * 1e3)
        pos0 = ctx + warm
        byts = sum(decode_bytes_per_token(cfg, pos0 + i) for i in range(args.decode_steps))
        peak, src = measured_peaks()
        tps = args.decode_steps / (ms / 1e3)
        persistent = default == PERSISTENT
        out = {
            "tokens_per_s": round(tps * world, 1),
            "tokens_per_s_per_gpu": round(tps, 1),
            "ms_per_token": round(ms / args.decode_steps, 4),
            "path": "persistent (one cooperative launch per token)" if persistent else "graph (per-kernel)",
            "config": "22 layers, hidden 2048, 32q/4kv heads, head_dim 64, FFN 5632, vocab 32000; context "
                      f"{pos0}..{pos0 + args.decode_steps}; greedy; replicas on each GPU",
            "bytes_per_token": byts // args.decode_steps,
            "achieved_gbs": round(byts / (ms / 1e3) / 1e9, 1),
            "roofline_frac": round(byts / (ms / 1e3) / 1e9 / peak, 4),
            "gpu_launches_per_token": 1 if persistent else 5 * c.numLayers + 3,
            "e2e_host_forward": {"tokens_per_s": round(n_host / (host_ms / 1e3) * world, 1),
                                 "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4 * c.vocabSize},
        }
        # The same decode with llm/sampler.ts top-p sampling on the device
        # (temperature 1, topP 0.9) choosing every token; the rng is a seeded
        # generator whose values are the steps' draws.
        draws = iter(np.random.default_rng(44).random(warm + args.decode_steps).tolist())
        opts = {"temperature": 1.0, "topP": 0.9, "rng": lambda: next(draws)}
        eng.setKv(0, kv0[0], kv0[1], ctx)
        eng.sampleSteps(first, warm, opts)
        barrier()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(es)
        stoks = eng.sampleSteps(first, args.decode_steps, opts)
        d1.record(es)
        d1.synchronize()
        sms = max_over_ranks(d0.elapsed_time(d1))
        out["sampled"] = {
            "tokens_per_s_per_gpu": round(args.decode_steps / (sms / 1e3), 1),
            "ms_per_token": round(sms / args.decode_steps, 4),
            "sampler_us_per_token": round((sms - ms) / args.decode_steps * 1e3, 1),
            "mode": "top-p on the device: temperature 1.0, topP 0.9, seeded draws",
            "distinct_tokens": int(len(set(np.asarray(stoks).tolist()))),
            "gpu_launches_per_token": (1 if persistent else 5 * c.numLayers + 3) + 3,
        }
        # Prefill: a 512-token prompt through the batched prefill (tensor-core
        # matmulQ8 GEMMs), measured on the engine stream; forward() also
        # returns the final logits to the host.
        n_prompt = min(512, c.maxSeqLen)
        prompt = np.random.default_rng(43).integers(0, c.vocabSize, n_prompt).tolist()
        eng.reset()
        eng.forward(prompt)  # warm-up (workspace, modules)
        p_ms, p_wall = [], []
        for _ in range(3):
            eng.reset()
            barrier()
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            w0 = time.perf_counter()
            d0.record(es)
            eng.forward(prompt)
            d1.record(es)
            d1.synchronize()
            p_wall.append((time.perf_counter() - w0) * 1e3)
            p_ms.append(d0.elapsed_time(d1))
        pms = max_over_ranks(float(np.mean(p_ms)))
        pwall = max_over_ranks(float(np.mean(p_wall)))
        out["prefill"] = {
            "prompt_tokens": n_prompt,
            "ms": round(pms, 3),
            "tokens_per_s": round(n_prompt / (pms / 1e3) * world, 1),
            "e2e_ms": round(pwall, 3),
            "path": "batched prefill: tcgen05 matmulQ8 GEMMs (int8 weights x int8 activation limbs)",
        }
        if world == 1 and args.oracle_tokens > 0:
            out["oracle"] = decode_oracle_check(cfg, weights, kvs, ctx, first, warm, toks, args.oracle_tokens)
        for pth in paths[1:]:
            oms, otoks = res[pth]
            out["persistent_path" if pth == PERSISTENT else "graph_path"] = {
                "tokens_per_s_per_gpu": round(args.decode_steps / (oms / 1e3), 1),
                "gpu_launches_per_token": 1 if pth == PERSISTENT else 5 * c.numLayers + 3,
                "same_tokens": int(np.sum(np.asarray(otoks) == np.asarray(toks)))}
        return out
    finally:
        eng.close()


def decode_oracle_check(cfg, weights, kvs, ctx, first, warm, toks, n):
    """The decode benchmark's first `n` greedy tokens against the oracle (a C
    restatement of llm/engine-q8-resident.ts:1774-1892, f64, one thread like
    JavaScript), replaying the benchmark's sequence: the cache prefilled to
    `ctx`, `warm` greedy steps from `first`, then the timed steps from `first`
    again.  Also the oracle's decode rate: the CPU baseline of decode
    tokens/s."""
    import oracle.oracle as orc

    t0 = time.perf_counter()
    o = orc.LlamaOracle(cfg, weights)
    for l, (k, v) in enumerate(kvs):
        o.set_kv(l, k, v, ctx)
    build_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    tok = first
    for _ in range(warm):
        tok = orc.argmax(o.forward([tok]))
    want, margins, tok = [], [], first
    for _ in range(n):
        logits = o.forward([tok])
        srt = np.sort(logits.astype(np.float64))
        margins.append(float(srt[-1] - srt[-2]) / float(np.max(np.abs(logits))))
        tok = orc.argmax(logits)
        want.append(int(tok))
    el = time.perf_counter() - t0
    o.close()
    got = [int(t) for t in toks[:n]]
    decided = [i for i in range(n) if margins[i] > 1e-3]
    return {"tokens": n, "oracle": want, "ours": got, "equal": int(sum(a == b for a, b in zip(got, want))),
            "equal_where_margin_exceeds_1e-3": all(got[i] == want[i] for i in decided),
            "top2_margins_rel": [round(m, 6) for m in margins],
            "cpu_baseline": {"tokens_per_s": round((warm + n) / el, 4), "cores": 1, "kind": "port",
                             "sample": f"{warm + n} decode steps of the benchmark model at context {ctx}.."
                                       f"{ctx + warm + n} on the oracle, one thread ({el:.1f} s; model build "
                                       f"{build_s:.1f} s untimed)"}}


# ------------------------------------------------------- reference arm ---

def run_reference(args, rank, world):
    """The reference's CPU path for this workload: ops/matvec/reference.ts
    `matvecQ8`, restated in C (oracle/), the TypeScript itself having no
    runtime on this image.  Inputs are built on the host by the oracle (the
    same seeded recipe as the GPU arm), so this arm loads no GPU code.  Timed
    with every host thread on one whole matrix of the stack per step, and
    once single-threaded as JavaScript runs it."""
    if rank != 0:
        return
    import oracle.oracle as orc

    K, R = COLS, ROWS  # one whole matrix of the stack per step
    threads = os.cpu_count() or 1
    g0 = time.perf_counter()
    w, s, x = reference_sample(R, K, threads)
    gen_s = time.perf_counter() - g0
    for _ in range(max(1, min(args.warmup, 3))):
        orc.matvec_q8(w, s, x, R, K, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.matvec_q8(w, s, x, R, K, threads=threads)
    el = time.perf_counter() - t0
    value = algorithmic_bytes(R, K, 1) * args.steps / el / 1e9
    t1 = time.perf_counter()
    orc.matvec_q8(w, s, x, R, K)
    one = time.perf_counter() - t1
    single = algorithmic_bytes(R, K, 1) / one / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8*f64 (reference.ts accumulates in f64)",
        "data": "synthetic (seeded N(0, 0.02^2) weights quantized per row, x ~ N(0, 1))",
        "config": {"workload": f"matvecQ8 stack: {args.matrices} x [{ROWS} x {COLS}] Q8 on one x; "
                               f"each step one [{R} x {K}] matrix of it on the CPU",
                   "matrices": args.matrices, "N": ROWS, "K": COLS, "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"one [{R} x {K}] matrix per step, {args.steps} steps, {threads} threads "
                                   f"(rows split over POSIX threads)",
                         "single_thread": {"value": round(single, 4), "unit": "GB/s", "cores": 1,
                                           "sample": f"one pass over the same matrix, {one:.2f} s"},
                         "inputs": f"built on the host by the oracle in {gen_s:.1f} s, untimed",
                         "cpu": _cpu_model()},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference.ts cannot run here (no JavaScript runtime on the image); the C restatement of "
                "ops/matvec/reference.ts:117-131 stands in.  JavaScript runs it on one thread: that figure is "
                "cpu_baseline.single_thread.",
    }
    print(json.dumps(line), flush=True)


def reference_sample(R, K, threads):
    """Matrix 0 of the stack and x, built on the host by the oracle's C
    restatement of the seeded recipe (xpuops/synth.py; the GPU arm's device
    fill follows the same recipe), quantized and packed by the oracle."""
    import oracle.oracle as orc
    from xpuops.synth import tensor_seed

    wf = orc.fill_normal(R * K, tensor_seed(0, 0), 0.0, 0.02, threads=threads)
    codes, sc = orc.quantize_mt(wf, R, K, threads)
    del wf
    packed = orc.pack_q8(codes, R, K)
    del codes
    return packed, sc, orc.fill_normal(K, tensor_seed(1, 0))


def run_gemv(args):
    """`--gemv NxK`: single matvecQ8 launches (xpu_matvec_q8_dev, library
    default path) of one shape, rotating over enough matrices (up to 16, at
    least 1 GB) that L2 never holds the weights read; --warmup rounds over the
    matrices untimed, then --steps timed rounds.  Prints one JSON line.  This
    is the small, self-contained case the kernel profiles are captured on."""
    import torch

    from xpuops import ops
    from xpuops.synth import tensor_seed

    N, K = (int(v) for v in args.gemv.lower().split("x"))
    W = (K + 3) // 4
    torch.cuda.set_device(0)
    sp = torch.cuda.current_stream().cuda_stream
    count = max(2, min(16, -(-(1 << 30) // (4 * N * W))))
    w = torch.empty(count * N * W, dtype=torch.int32, device="cuda")
    sc = torch.empty(count * N, dtype=torch.float32, device="cuda")
    tmp = torch.empty(N * K, dtype=torch.float32, device="cuda")
    for i in range(count):
        ops.fill_normal_dev(tmp, N * K, tensor_seed(30, i), 0.0, 0.02, stream=sp)
        ops.quantizePackQ8_dev(tmp, N, K, w.data_ptr() + 4 * i * N * W, sc.data_ptr() + 4 * i * N, stream=sp)
    del tmp
    x = torch.empty(K, dtype=torch.float32, device="cuda")
    ops.fill_normal_dev(x, K, tensor_seed(31, 0), stream=sp)
    y = torch.empty(N, dtype=torch.float32, device="cuda")

    def rounds(n):
        for _ in range(n):
            for i in range(count):
                ops.matvecQ8_dev(w.data_ptr() + 4 * i * N * W, sc.data_ptr() + 4 * i * N, x, N, K, y, sp)

    rounds(max(1, args.warmup))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    rounds(args.steps)
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / (args.steps * count)
    b = algorithmic_bytes(N, K, 1)
    peak, _ = measured_peaks()
    print(json.dumps({"metric": "matvecQ8 single GEMV, each its own launch", "workload": f"{N}x{K}",
                      "matrices": count, "launches": args.steps * count, "us": round(t * 1e6, 2),
                      "GBs": round(b / t / 1e9, 1), "frac": round(b / t / 1e9 / peak, 4),
                      "bytes_per_launch": b}), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.gemv:
        run_gemv(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
