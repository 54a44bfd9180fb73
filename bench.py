#!/usr/bin/env python
"""Benchmark of the Q4_K decode GEMV path on B200 (one JSON line on rank 0).

Workload (the reference's Q8_0/Q4_K matvec sweep, Q4_K half): batch-1 GEMVs
over the four Llama-7B projection shapes (4096x4096, 11008x4096, 4096x11008,
32000x4096), weights ~N(0, 0.02) quantized to Q4_K by this project's
quantizer (the reference has none), activations ~N(0, 1).  One step = one
GEMV per shape, activation packing included.  Weights rotate over R copies
(4 x 133.9 MB) so every step streams them from HBM, not from the 126 MB L2.

  value   device throughput, algorithmic bytes (weights + 4k + 4n per GEMV)
          per second; inputs resident in HBM; K steps replayed from one CUDA
          graph; timed with CUDA events; max over ranks.
  e2e     the same metric through the C ABI's host-pointer entry point
          (eosi_cuda_matmul_q: host activations in, host outputs back,
          weights cached on the device as the backend does for a model).
  roofline  per-launch CUDA-event times of the GEMV (+ its packing kernel)
          inside the timed graph vs the measured HBM copy bandwidth.
  cpu_baseline  the reference's own x86 kernel (compiled from its sources
          into oracle/_ref) on the host cores, same workload;
          cpu_baseline_1core the same on one core.
  q8_0_sweep  the Q8_0 half of the sweep (same shapes, the reference's Q8_0
          weight format), with its own roofline and CPU baseline.

Multi-GPU (torchrun): weak scaling -- every rank streams its own row shard
of N-times-taller matrices (rows are independent; no collective on the data
path), value = all ranks' bytes / max-over-ranks time.

`--impl reference` runs the reference's CPU implementation (eosi_avx2_matmul_q,
the x86_avx2 backend's matmul_q slot) with all host threads on rank 0.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]  # (n, k)
METRIC = "Q4_K GEMV HBM GB/s (batch-1 sweep 4096x4096, 11008x4096, 4096x11008, 32000x4096)"
DT_Q4_K = 33


def q4k_bytes(n: int, k: int) -> int:
    return n * (k // 256) * 144


def algo_bytes(n: int, k: int) -> int:
    """Algorithmic bytes of one GEMV: weights + f32 activations + f32 outputs."""
    return q4k_bytes(n, k) + 4 * k + 4 * n


STEP_BYTES = sum(algo_bytes(n, k) for n, k in SHAPES)
DT_Q8_0 = 32


def q80_bytes(n: int, k: int) -> int:
    return n * (k // 32) * 34


def algo_bytes_q80(n: int, k: int) -> int:
    """Algorithmic bytes of one Q8_0 GEMV: weights + f32 activations + f32 outputs."""
    return q80_bytes(n, k) + 4 * k + 4 * n


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--copies", type=int, default=4, help="rotating weight copies (L2 defeat)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample length")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-q8", action="store_true", help="skip the Q8_0 half of the sweep")
    p.add_argument("--workload", choices=["all", "sweep", "decode", "prefill"], default="all",
                   help="sweep: the GEMV sweep line only; decode: the 7B decode line; prefill: the GEMM line")
    p.add_argument("--no-prefill", action="store_true", help="skip the tensor-core prefill measurement")
    p.add_argument("--no-decode", action="store_true", help="skip the 7B-shape decode measurement")
    p.add_argument("--decode-prompt", type=int, default=512)
    p.add_argument("--decode-gen", type=int, default=256)
    p.add_argument("--decode-cpu-steps", type=int, default=2, help="reference-engine decode steps timed on the host (cpu_baseline)")
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks: NVML sampled during the timed region (read-only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._th = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self.nv = None
            self.err = str(e)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def _sample(self):
        try:
            mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.samples.append((mhz, rs))
        except Exception:  # noqa: BLE001
            pass

    def start(self):
        if self.nv is not None:
            self._sample()
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()

    def stop(self):
        if self._th is not None:
            self._stop.set()
            self._th.join()
            self._sample()

    def summary(self):
        if self.nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s[0] for s in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for b, name in self.REASONS.items() if bits & b and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(backend: str):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device=None) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_done(world):
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def measured_hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the GEMV from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "q4k_gemv_sweep.ncu.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch_avg:"):
                    return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# CPU: the reference's own kernel (oracle/_ref), row-sharded over threads
# ---------------------------------------------------------------------------
class CpuSweep:
    """eosi_avx2_matmul_q of the reference (or the oracle port when the
    reference build is absent) over the sweep, rows split across threads;
    ctypes releases the GIL so the threads run in parallel."""

    def __init__(self, threads: int | None = None, row_fraction: float = 1.0, dtype: int = DT_Q4_K):
        from oracle.oracle import REF_KERNELS, Oracle, RefKernels
        if RefKernels.available():
            self.kind = "reference"
            lib = RefKernels().lib
            self.fn = lib.eosi_avx2_matmul_q
        else:
            self.kind = "port"
            lib = Oracle().lib
            self.fn = lib.orc_matmul_q
        self.oracle = Oracle()
        self.dtype = dtype
        self.threads = threads or os.cpu_count() or 1
        self.pool = cf.ThreadPoolExecutor(self.threads)
        self.data = []
        quant = self.oracle.q4_k_quantize if dtype == DT_Q4_K else self.oracle.q8_0_quantize
        for s, (n, k) in enumerate(SHAPES):
            rows = max(self.threads, int(n * row_fraction))
            w = quant(self.oracle.gauss(rows * k, s, 0.02))
            x = self.oracle.gauss(k, 10 + s, 1.0)
            c = np.empty(rows, np.float32)
            self.data.append((rows, k, w, x, c))
        ab = algo_bytes if dtype == DT_Q4_K else algo_bytes_q80
        self.step_bytes = sum(ab(rows, k) for rows, k, *_ in self.data)
        self.row_fraction = row_fraction

    def _part(self, rows, k, w, x, c, lo, hi):
        rb = (k // 256) * 144 if self.dtype == DT_Q4_K else (k // 32) * 34
        rc = self.fn(x.ctypes.data, w.ctypes.data + lo * rb, self.dtype, c.ctypes.data + 4 * lo, 1, hi - lo, k)
        if rc != 0:
            raise RuntimeError(f"reference matmul_q failed: {rc}")

    def step(self):
        futs = []
        for rows, k, w, x, c in self.data:
            for t in range(self.threads):
                lo, hi = rows * t // self.threads, rows * (t + 1) // self.threads
                if hi > lo:
                    futs.append(self.pool.submit(self._part, rows, k, w, x, c, lo, hi))
        for f in futs:
            f.result()

    def describe(self):
        sample = "full sweep" if self.row_fraction >= 1.0 else f"{self.row_fraction:.3f} of each matrix's rows"
        return f"{sample}, batch 1, {self.threads} threads over output rows"


def host_cpu() -> dict:
    """The host CPU every CPU number was measured on: model string and the
    logical cores the OS offers."""
    name = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu": name, "nproc": os.cpu_count() or 1}


def sweep_config(copies: int) -> dict:
    """The workload of the headline sweep, identical in both arms."""
    return {"workload": "q4k_gemv_sweep", "shapes": SHAPES, "batch": 1,
            "weights": "Q4_K, ~N(0,0.02) (Irwin-Hall), own quantizer", "activations": "~N(0,1)",
            "l2": f"inputs larger than the last-level cache: on the GPU {copies} rotating weight copies "
                  f"({copies * sum(q4k_bytes(n, k) for n, k in SHAPES) / 1e6:.1f} MB) > 126 MB L2; the host "
                  f"sweep's {sum(q4k_bytes(n, k) for n, k in SHAPES) / 1e6:.1f} MB > its L3"}


def cpu_baseline(seconds: float, threads: int | None = None, dtype: int = DT_Q4_K,
                 row_fraction: float = 1.0) -> dict:
    """The reference's matmul_q slot on the host cores for `seconds`: Q4_K
    goes to its int8 AVX2 kernel, Q8_0 to its scalar kernel (the x86
    backend's dispatch, src/kernels/avx2/matmul_q4_k.c:155-171)."""
    cpu = CpuSweep(threads=threads, dtype=dtype, row_fraction=row_fraction)
    cpu.step()
    steps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        cpu.step()
        steps += 1
    dt = time.perf_counter() - t0
    path = "Q4_K -> int8 AVX2 path" if dtype == DT_Q4_K else "Q8_0 -> scalar path"
    return {"value": round(cpu.step_bytes * steps / dt / 1e9, 3), "unit": "GB/s", "cores": cpu.threads,
            "kind": cpu.kind, **host_cpu(), "sample": f"{steps} sweeps ({cpu.describe()}) in {dt:.1f} s, "
                                                      f"eosi_avx2_matmul_q ({path})"}


def run_reference(args):
    world, rank, _ = dist_setup("gloo")
    if rank != 0:
        dist_done(world)
        return
    # size the sample so K + W steps stay within about two minutes
    probe = CpuSweep(row_fraction=1.0)
    t0 = time.perf_counter()
    probe.step()
    per_step = time.perf_counter() - t0
    frac = min(1.0, 120.0 / max(per_step * (args.steps + args.warmup), 1e-9))
    cpu = probe if frac >= 1.0 else CpuSweep(row_fraction=frac)
    for _ in range(args.warmup):
        cpu.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.step()
    dt = time.perf_counter() - t0
    gbs = cpu.step_bytes * args.steps / dt / 1e9
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": sweep_config(max(1, args.copies)),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu.threads, "kind": cpu.kind,
                         **host_cpu(), "sample": cpu.describe()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    dist_done(world)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch

    from eosllm_b200 import backend as B

    world, rank, local = dist_setup("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B.load()
    if B.load().eosi_cuda_probe() != 0:
        raise SystemExit(f"CUDA backend unavailable: {B.last_error()}")
    B.set_devices([local])
    if args.workload == "prefill":
        d = run_prefill(args, dev)
        if rank == 0:
            line = dict(d, n_gpus=world, steps=20, warmup=3, ms_per_step=d["per_m"][str(PREFILL_M[-1])]["ms"],
                        higher_is_better=True, scaling="weak", vs_baseline=None, dtype="int8 (bit-exact; exact bf16 MMA, f32 rescale)",
                        data="synthetic", gpu_launches=2 * 20 * len(PREFILL_M),
                        config={"workload": "q4k_prefill_gemm", "m": list(PREFILL_M), "n": PREFILL_NK[0],
                                "k": PREFILL_NK[1]})
            print(json.dumps(line), flush=True)
        dist_done(world)
        return
    if args.workload == "decode":
        d = run_decode(args, dev, world, rank)
        if rank == 0:
            line = dict(d, steps=args.decode_gen, warmup=16, ms_per_step=d["ms_per_token"], higher_is_better=True,
                        scaling="strong",
                        vs_baseline=None, dtype="int8", data="synthetic",
                        gpu_launches=args.decode_gen * d.pop("launches_per_token"))
            line["config"] = dict(line["config"], workload="llama_7b_shape_q4k_decode")
            print(json.dumps(line), flush=True)
        dist_done(world)
        return
    R = max(1, args.copies)

    # ---- inputs resident in HBM: rank r owns rows [r*n, (r+1)*n) of N-times-taller matrices
    weights, acts, outs, scratch = [], [], [], []
    # activations with the same k are rows of one matrix, packed in one launch
    ks = sorted({k for _, k in SHAPES})
    xmat = {k: torch.empty((sum(1 for _, kk in SHAPES if kk == k), k), dtype=torch.float32, device=dev) for k in ks}
    # packed activations, double-buffered: step i reads set i % 2 while the
    # packing of step i + 1 fills the other set
    smats = [{k: torch.empty(B.q4_k_scratch_bytes(xmat[k].shape[0], k), dtype=torch.uint8, device=dev) for k in ks}
             for _ in range(2)]
    smat = smats[0]
    row_of = {}
    for s, (n, k) in enumerate(SHAPES):
        row_of[s] = sum(1 for kk in [kk for _, kk in SHAPES[:s]] if kk == k)
    for s, (n, k) in enumerate(SHAPES):
        copies = []
        for r in range(R):
            w = torch.empty(q4k_bytes(n, k), dtype=torch.uint8, device=dev)
            B.q4_k_from_gauss_dev(w, n * k, seed=1000 * rank + 100 * r + s, sigma=0.02)
            copies.append(w)
        weights.append(copies)
        x = xmat[k][row_of[s]]
        B.fill_gauss_dev(x, k, 10 + s, 0, 1.0)
        acts.append(x)
        outs.append(torch.empty(n, dtype=torch.float32, device=dev))
        scratch.append(smat[k].data_ptr() + row_of[s] * B.q4_k_scratch_bytes(1, k))
    torch.cuda.synchronize()

    def scratch_of(s: int, i: int) -> int:
        n, k = SHAPES[s]
        return smats[i % 2][k].data_ptr() + row_of[s] * B.q4_k_scratch_bytes(1, k)

    def capture(steps: int):
        """One step: pack the four activation vectors (exact quantize_sub32
        packing; one launch per distinct k, the vectors being rows of one
        matrix), then the four GEMVs back to back (PDL-chained).  The
        packing of step i + 1 runs on a second stream while the GEMVs of step
        i run (double-buffered packed activations; graph edges order each
        packing after the GEMVs that last read its buffer and before the
        GEMVs that read it), so the GEMV chain is not interrupted."""
        g = torch.cuda.CUDAGraph()
        main = torch.cuda.Stream(device=dev)
        packer = torch.cuda.Stream(device=dev)
        packed = [torch.cuda.Event() for _ in range(steps + 1)]
        gemvs_done = [torch.cuda.Event() for _ in range(steps)]
        with torch.cuda.graph(g, stream=main, capture_error_mode="relaxed"):
            st, ps = main.cuda_stream, packer.cuda_stream
            packer.wait_stream(main)  # fork the packing stream into the capture

            def pack(i: int) -> None:
                for k in ks:
                    B.q4_k_pack_act_dev(xmat[k], xmat[k].shape[0], k, smats[i % 2][k], ps)
                packed[i].record(packer)

            pack(0)
            for i in range(steps):
                if i + 1 < steps:
                    if i >= 1:
                        packer.wait_event(gemvs_done[i - 1])  # step i - 1 read the buffer step i + 1 fills
                    pack(i + 1)
                main.wait_event(packed[i])
                for s, (n, k) in enumerate(SHAPES):
                    B.q4_k_gemv_dev(scratch_of(s, i), weights[s][i % R], outs[s], n, k, st)
                gemvs_done[i].record(main)
            main.wait_stream(packer)  # join
        return g

    def capture_train(s: int, launches: int):
        """`launches` GEMVs of shape s back to back (rotating weight copies,
        PDL-chained): the kernel's average launch duration in a stream of
        its own launches."""
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device=dev)
        n, k = SHAPES[s]
        with torch.cuda.graph(g, stream=side, capture_error_mode="relaxed"):
            st = torch.cuda.current_stream().cuda_stream
            for i in range(launches):
                B.q4_k_gemv_dev(scratch[s], weights[s][i % R], outs[s], n, k, st)
        return g

    g_warm = capture(max(args.warmup, 3))
    g_timed = capture(args.steps)
    train_n = max(args.steps, 100)
    g_trains = [capture_train(s, train_n) for s in range(len(SHAPES))]
    g_warm.replay()
    # one untimed replay of the timed graph itself: a graph's first launch
    # uploads it to the device (~1.6 ms for 6000 nodes), which is not a step
    g_timed.replay()
    for g in g_trains:
        g.replay()
    torch.cuda.synchronize()
    assert B.take_device_errors() == 0

    # ---- timed region: K steps from one graph, events on the capture stream's
    # replay stream, barrier + synchronize on both sides
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t0.record()
    g_timed.replay()
    t1.record()
    torch.cuda.synchronize()
    clocks.stop()
    barrier(world)
    if B.take_device_errors() != 0:
        raise SystemExit("device-side bounded wait reported an error")
    total_ms = t0.elapsed_time(t1)

    # ---- the GEMV kernel's average launch duration per shape: a train of
    # launches of that shape alone, CUDA events on the replay stream around
    # the whole train (inputs > L2: rotating copies)
    per_shape_ms = []
    for g in g_trains:
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        g.replay()
        a1.record()
        torch.cuda.synchronize()
        per_shape_ms.append(a0.elapsed_time(a1) / train_n)
    t_max = max_over_ranks(total_ms, world, dev)
    value = world * STEP_BYTES * args.steps / (t_max * 1e-3) / 1e9
    achieved = STEP_BYTES / (sum(per_shape_ms) * 1e-3) / 1e9
    peak, peak_kind = measured_hbm_peak()
    traffic = profiled_traffic()

    # ---- e2e through the host-pointer C ABI (the backend vtable slot)
    e2e = None
    if not args.no_e2e:
        host_w = [[weights[s][r].cpu().numpy() for r in range(R)] for s in range(len(SHAPES))]
        host_x = [acts[s].cpu().numpy() for s in range(len(SHAPES))]
        host_c = [np.empty((1, n), np.float32) for n, _ in SHAPES]
        for s, (n, k) in enumerate(SHAPES):
            for r in range(R):
                B.cache_preload(host_w[s][r], DT_Q4_K, n, k)
        lib = B.load()

        def e2e_step(i):
            r = i % R
            for s, (n, k) in enumerate(SHAPES):
                rc = lib.eosi_cuda_matmul_q(host_x[s].ctypes.data, host_w[s][r].ctypes.data, DT_Q4_K,
                                            host_c[s].ctypes.data, 1, n, k)
                if rc != 0:
                    raise RuntimeError(B.last_error())

        for i in range(max(args.warmup, 3)):
            e2e_step(i)
        e2e_steps = max(args.steps, 10)
        barrier(world)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            e2e_step(i)
        dt = max_over_ranks(time.perf_counter() - t0, world, dev)
        # check the e2e outputs against the device path (same kernels, same bits)
        for s, (n, k) in enumerate(SHAPES):
            B.matmul_q4_k_dev(acts[s], weights[s][(e2e_steps - 1) % R], outs[s], 1, n, k, scratch[s],
                              torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            assert np.array_equal(outs[s].cpu().numpy().view(np.uint32), host_c[s][0].view(np.uint32))
        e2e = {"value": round(world * STEP_BYTES * e2e_steps / dt / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": sum(4 * k for _, k in SHAPES),
               "d2h_bytes_per_step": sum(4 * n for n, _ in SHAPES)}

    q80 = None
    if not args.no_q8:
        q80 = run_q80_sweep(args, dev, world, rank, R)

    cpu = cpu_1core = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)
        # one core, on an eighth of each matrix's rows (rows are independent)
        cpu_1core = cpu_baseline(args.cpu_seconds / 2, threads=1, row_fraction=0.125)
        if q80 is not None:  # the reference's scalar Q8_0 kernel on every host core, a quarter of the rows
            q80["cpu_baseline"] = cpu_baseline(args.cpu_seconds / 2, dtype=DT_Q8_0, row_fraction=0.25)

    prefill = None
    if args.workload == "all" and not args.no_prefill:
        prefill = run_prefill(args, dev)

    decode = None
    if args.workload == "sweep":
        pass
    elif not args.no_decode:
        del g_timed, g_warm, g_trains
        weights.clear()
        torch.cuda.empty_cache()
        decode = run_decode(args, dev, world, rank)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_max / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": sweep_config(R),
            "timing": f"CUDA graph of K steps (2 packing launches, one per distinct k, + 4 PDL-chained GEMVs "
                      f"each; the packing of step i + 1 on a second stream during the GEMVs of step i) over {R} "
                      "rotating weight copies, CUDA events, max over ranks",
            "parallelism": f"row shards x{world}, no collective",
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "kernel": "q4k_gemv_cols_kernel<8,2,2> (rows of k = 11008 staged in 16-super-block chunks): "
                                   "mean launch time of a 100+-launch train per shape "
                                   "(rotating copies), bytes = weights + 4k + 4n per launch, summed over the sweep",
                         "per_shape_us": {f"{n}x{k}": round(ms * 1e3, 3) for (n, k), ms in zip(SHAPES, per_shape_ms)},
                         "per_shape_frac": {f"{n}x{k}": round(algo_bytes(n, k) / (ms * 1e-3) / 1e9 / peak, 4)
                                            for (n, k), ms in zip(SHAPES, per_shape_ms)}},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "cpu_baseline_1core": cpu_1core,
            "q8_0_sweep": q80,
            "gpu_launches": args.steps * (len(ks) + len(SHAPES)),
            "clocks": clocks.summary(),
            "decode_7b": decode,
            "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    dist_done(world)


LLAMA_7B = dict(n_embd=4096, n_layer=32, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=32000)
PREFILL_M = (128, 512, 2048)
PREFILL_NK = (11008, 4096)


def run_q80_sweep(args, dev, world, rank, R: int) -> dict:
    """The Q8_0 half of the reference's matvec sweep on the same four shapes:
    weights ~N(0, 0.02) quantized on the device by the reference's Q8_0
    quantizer (q8_0.c:58-93, bit for bit), activations ~N(0, 1); one step =
    one eosi_cuda_matmul_q8_0_dev GEMV per shape, K steps replayed from one
    CUDA graph, R rotating weight copies (> L2), CUDA events on the replay
    stream, max over ranks.  The per-shape trains give the kernel's mean
    launch time for the roofline."""
    import torch

    from eosllm_b200 import backend as B
    tmp = torch.empty(max(n * k for n, k in SHAPES), dtype=torch.float32, device=dev)
    weights, acts, outs = [], [], []
    for s, (n, k) in enumerate(SHAPES):
        copies = []
        for r in range(R):
            w = torch.empty(q80_bytes(n, k), dtype=torch.uint8, device=dev)
            B.fill_gauss_dev(tmp, n * k, 5000 + 1000 * rank + 100 * r + s, 0, 0.02)
            B.q8_0_quantize_dev(tmp, w, n * k)
            copies.append(w)
        weights.append(copies)
        x = torch.empty(k, dtype=torch.float32, device=dev)
        B.fill_gauss_dev(x, k, 10 + s, 0, 1.0)
        acts.append(x)
        outs.append(torch.empty(n, dtype=torch.float32, device=dev))
    torch.cuda.synchronize()
    del tmp

    def graph(launch, count):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device=dev)
        with torch.cuda.graph(g, stream=side, capture_error_mode="relaxed"):
            st = torch.cuda.current_stream().cuda_stream
            for i in range(count):
                launch(i, st)
        return g

    def gemv(s, i, st):
        n, k = SHAPES[s]
        B.matmul_q8_0_dev(acts[s], weights[s][i % R], outs[s], 1, n, k, st)

    def step(i, st):
        for s in range(len(SHAPES)):
            gemv(s, i, st)

    train_n = max(args.steps, 100)
    g_warm, g_timed = graph(step, max(args.warmup, 3)), graph(step, args.steps)
    trains = [graph(lambda i, st, s=s: gemv(s, i, st), train_n) for s in range(len(SHAPES))]
    g_warm.replay()
    g_timed.replay()  # the graph's upload, untimed
    for g in trains:
        g.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev.index)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t0.record()
    g_timed.replay()
    t1.record()
    torch.cuda.synchronize()
    clocks.stop()
    barrier(world)
    per_shape_ms = []
    for g in trains:
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        g.replay()
        a1.record()
        torch.cuda.synchronize()
        per_shape_ms.append(a0.elapsed_time(a1) / train_n)
    if B.take_device_errors() != 0:
        raise SystemExit("q8_0 sweep: device-side error bits set")
    t_max = max_over_ranks(t0.elapsed_time(t1), world, dev)
    step_bytes = sum(algo_bytes_q80(n, k) for n, k in SHAPES)
    peak, peak_kind = measured_hbm_peak()
    achieved = step_bytes / (sum(per_shape_ms) * 1e-3) / 1e9
    return {
        "metric": "Q8_0 GEMV HBM GB/s (same batch-1 sweep)", "unit": "GB/s",
        "value": round(world * step_bytes * args.steps / (t_max * 1e-3) / 1e9, 2),
        "ms_per_step": round(t_max / args.steps, 5), "steps": args.steps, "dtype": "f32 (int8 weights)",
        "gpu_launches": args.steps * len(SHAPES),
        "config": {"workload": "q80_gemv_sweep", "shapes": SHAPES, "batch": 1,
                   "weights": "Q8_0 by the reference's quantizer (on the device), ~N(0,0.02)",
                   "l2": f"{R} rotating weight copies ({R * sum(q80_bytes(n, k) for n, k in SHAPES) / 1e6:.1f} MB)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "kernel": "q80_gemv_kernel: mean launch time of a 100+-launch train per shape",
                     "per_shape_us": {f"{n}x{k}": round(ms * 1e3, 3) for (n, k), ms in zip(SHAPES, per_shape_ms)},
                     "per_shape_frac": {f"{n}x{k}": round(algo_bytes_q80(n, k) / (ms * 1e-3) / 1e9 / peak, 4)
                                        for (n, k), ms in zip(SHAPES, per_shape_ms)}},
        "clocks": clocks.summary(),
    }


def measured_bf16_peak():
    """Dense bf16 TFLOP/s measured on this pool (burst), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        for key in ("bf16_tflops", "bf16_dense_tflops"):
            if key in d:
                return float(d[key]), "measured"
    except (OSError, ValueError):
        pass
    return 1590.0, "fallback"


def run_prefill(args, dev, reps: int = 20) -> dict:
    """Q4_K W [11008 x 4096] (~N(0,0.02), seed 2) times A [M x 4096] (~N(0,1))
    for M in 128/512/2048 on the tensor cores, bit-exact with the int8
    reference.  Weights are prepared once (as for a loaded model); each timed
    call packs the activations and runs the GEMM.  FLOPs = 2 M N K.  The
    kernel's bound is its epilogue: per output and 32-element sub-block it
    applies the reference's rescale (7 f32 operations: convert, 4 multiplies,
    subtract, add) on the CUDA cores, against one int8 MMA on the tensor
    pipe; `epilogue_frac` compares those operations per second with the
    f32 issue rate (148 SMs x 128 lanes x the sampled SM clock)."""
    import torch

    from eosllm_b200 import backend as B
    n, k = PREFILL_NK
    w = torch.empty(q4k_bytes(n, k), dtype=torch.uint8, device=dev)
    B.q4_k_from_gauss_dev(w, n * k, seed=2, sigma=0.02)
    wprep = torch.empty(B.prefill_weight_bytes(n, k), dtype=torch.uint8, device=dev)
    B.prefill_prepare_weights_dev(w, n, k, wprep)
    peak, peak_kind = measured_bf16_peak()
    props = torch.cuda.get_device_properties(dev)
    out = {"metric": "Q4_K prefill GEMM TFLOP/s (tcgen05, bit-exact with the int8 reference, N=11008 K=4096)", "unit": "TFLOP/s",
           "peak_bf16_tflops": peak, "peak_kind": peak_kind, "per_m": {}}
    st = torch.cuda.current_stream().cuda_stream
    clocks = ClockSampler(dev.index)
    clocks.start()
    for m in PREFILL_M:
        a = torch.empty((m, k), dtype=torch.float32, device=dev)
        B.fill_gauss_dev(a, m * k, 1000 + m, 0, 1.0)
        scratch = torch.empty(B.prefill_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
        c = torch.empty((m, n), dtype=torch.float32, device=dev)
        for _ in range(3):
            B.prefill_dev(a, wprep, c, m, n, k, scratch, st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            B.prefill_dev(a, wprep, c, m, n, k, scratch, st)
        e1.record()
        torch.cuda.synchronize()
        if B.take_device_errors() != 0:
            raise SystemExit("prefill: device-side bounded wait reported an error")
        ms = e0.elapsed_time(e1) / reps
        tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
        # tensor_frac: against the measured dense bf16 peak (the MMAs are
        # bf16 x bf16 -> f32 over exactly 2 M N K operations)
        out["per_m"][str(m)] = {"ms": round(ms, 4), "tflops": round(tf, 1), "tensor_frac": round(tf / peak, 4),
                                "epilogue_gops": round(7.0 * m * n * (k // 32) / (ms * 1e-3) / 1e9, 1)}
    clocks.stop()
    cs = clocks.summary()
    mhz = cs["sm_mhz"] or cs["sm_max_mhz"] or 1965
    f32_rate = props.multi_processor_count * 128 * mhz * 1e6 / 1e9  # G operations / s
    for v in out["per_m"].values():
        v["epilogue_frac"] = round(v["epilogue_gops"] / f32_rate, 4)
    out["f32_issue_gops"] = round(f32_rate, 1)
    out["clocks"] = cs
    out["value"] = out["per_m"][str(PREFILL_M[-1])]["tflops"]
    return out


GREEDY_FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "greedy_7b.npz")


def token_hash(tokens) -> str:
    """sha256 of the generated token ids as little-endian uint32, first 16 hex digits."""
    import hashlib
    return hashlib.sha256(np.asarray(tokens, dtype="<u4").tobytes()).hexdigest()[:16]


def fixture_agreement(tokens, prompt_len: int):
    """Free-running picks against the reference engine's own greedy picks on
    the same model and prompt (tests/golden/greedy_7b.npz, written by
    tests/golden/make_greedy_7b.py from the reference compiled from its
    sources): picks equal position by position, and the length of the
    common prefix (after the first difference the two runs feed different
    tokens, so later positions are not comparable)."""
    if not os.path.exists(GREEDY_FIXTURE):
        return None
    g = np.load(GREEDY_FIXTURE)
    ref = g["tokens"].astype(np.int64)
    if int(g["prompt"].size) != prompt_len:
        return None
    got = np.asarray(tokens, dtype=np.int64)
    n = min(ref.size, got.size)
    eq = got[:n] == ref[:n]
    prefix = int(n if eq.all() else np.argmin(eq))
    return {"compared": int(n), "equal": int(eq.sum()), "common_prefix": prefix,
            "reference_sha256": token_hash(ref[:n])}


def run_decode(args, dev, world, rank) -> dict:
    """7B-shape Q4_K greedy decoding through the device-resident decoder:
    random-init Llama-architecture model generated on the device (weights
    ~N(0, 0.02) -> Q4_K, F16 embeddings, F32 norms, stream seed 4), prompt of
    `decode_prompt` ids uniform in [0, 32000) from seed 4, then
    `decode_gen` greedy tokens.  Device time with CUDA events on the
    decoder's stream around each phase; the whole generation goes through
    eosi_cuda_text_generate (host prompt in, host tokens out)."""
    import torch

    from eosllm_b200 import backend as B
    from eosllm_b200.text import TextDecoder, synthetic_llama, weight_bytes_per_token
    P, G = args.decode_prompt, args.decode_gen
    cfg = dict(LLAMA_7B, max_ctx=P + G)
    model = synthetic_llama(**cfg, seed=4, device=dev.index)
    dec = TextDecoder(model, device=dev.index, rank=rank, world=world)
    if world > 1:
        dec.connect()  # IPC handles all-gathered over the process group; data path: GEMV pushes over NVLink
    host_model = None
    if rank == 0 and world == 1 and args.decode_cpu_steps > 0 and not args.no_cpu_baseline:
        host_model = dict(config=model["config"], tok_embd=model["tok_embd"].cpu().numpy().view(np.uint16),
                          output_norm=model["output_norm"].cpu().numpy(), output=model["output"].cpu().numpy(),
                          layers=[{k: v.cpu().numpy() for k, v in lay.items()} for lay in model["layers"]])
    del model
    torch.cuda.empty_cache()
    prompt = np.random.default_rng(4).integers(0, cfg["n_vocab"], P).astype(np.uint32)
    st = torch.cuda.ExternalStream(dec.stream, device=dev)
    dec.generate(prompt[:64], 8)  # warm-up: graph upload, batched-prefill scratch, first-touch
    dec.reset()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    clocks = ClockSampler(dev.index)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    w0 = time.perf_counter()
    ev[0].record(st)
    first = dec.generate(prompt, 1)  # P steps; the last one picks token 0
    ev[1].record(st)
    w1 = time.perf_counter()
    ev[2].record(st)
    toks = dec.generate(first, G)  # G steps at positions P .. P+G-1
    ev[3].record(st)
    w2 = time.perf_counter()
    torch.cuda.synchronize()
    clocks.stop()
    barrier(world)
    prefill_ms = max_over_ranks(ev[0].elapsed_time(ev[1]), world, dev)
    decode_ms = max_over_ranks(ev[2].elapsed_time(ev[3]), world, dev)
    wall_decode = max_over_ranks(w2 - w1, world, dev)
    wbytes = weight_bytes_per_token(dict(cfg, wdtype=B.DT_Q4_K, out_dtype=B.DT_Q4_K))
    kv_avg = 2 * cfg["n_layer"] * cfg["n_embd"] * 4 * (P + (G + 1) / 2)  # fp32 K and V rows 0..p, mean p
    peak, peak_kind = measured_hbm_peak()
    ms_tok = decode_ms / G
    out = {
        "metric": "7B-shape Q4_K greedy decode tokens/s", "value": round(G / (decode_ms * 1e-3), 2),
        "unit": "tok/s", "ms_per_token": round(ms_tok, 4), "n_gpus": world,
        "prefill_tok_s": round(P / (prefill_ms * 1e-3), 2), "prompt": P, "generated": G,
        # prompt tokens 0..P-2 in one batched pass on the tensor cores
        # (eosi_cuda_text_prefill; tensor parallel: each rank its slices, the
        # partial rows pushed over NVLink), the last through the step graph
        "prefill_mode": "batched_tcgen05",
        # the batched prefill's GEMM layout of every layer (bf16 4-bit values
        # + per-32 scales), prepared once at the warm-up prefill and kept
        "prefill_weights_gb": round(sum(B.prefill_weight_bytes(nn, kk) for nn, kk in (
            (3 * cfg["n_embd"], cfg["n_embd"]), (cfg["n_embd"], cfg["n_embd"]), (2 * cfg["n_ff"], cfg["n_embd"]),
            (cfg["n_embd"], cfg["n_ff"]))) * cfg["n_layer"] / world / 1e9, 2),  # per rank
        "config": dict(cfg, wdtype="Q4_K", out_dtype="Q4_K", kv_cache="f32", parallelism=f"tp{world}"),
        "e2e": {"value": round(G / wall_decode, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm", "bytes_per_token": int(wbytes + kv_avg), "weight_bytes_per_token": wbytes,
                     "kv_bytes_per_token_mean": int(kv_avg),
                     "achieved": round((wbytes + kv_avg) / world / (ms_tok * 1e-3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s per GPU", "peak_kind": peak_kind,
                     "frac": round((wbytes + kv_avg) / world / (ms_tok * 1e-3) / 1e9 / peak, 4),
                     "tok_s_at_peak": round(world * peak * 1e9 / (wbytes + kv_avg), 1),
                     "tok_s_weight_only_at_peak": round(world * peak * 1e9 / wbytes, 1)},
        "launches_per_token": dec.step_kernels,  # counted: the nodes of the step's CUDA graph
        "first_tokens": [int(x) for x in toks[:8]],
        # all P.. greedy picks (the one after the prompt, then G more), the
        # same on every GPU count when tensor parallelism is exact
        "tokens_sha256": token_hash(np.concatenate([first, toks])),
        "reference_agreement": fixture_agreement(np.concatenate([first, toks]), P),
        "clocks": clocks.summary(),
    }
    # the persistent step (one cooperative kernel per token) on the same
    # decoder: up to 64 tokens after the same prompt; its picks must be the
    # per-op step's (bit-identical by construction)
    n_p = min(64, G)
    if world == 1 and n_p > 0:
        from eosllm_b200.text import TextDecoder as _TD
        dec.set_step_mode(_TD.STEP_PERSISTENT)
        dec.reset()
        p_first = dec.generate(prompt, 1)
        ev2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev2[0].record(st)
        p_toks = dec.generate(p_first, n_p)
        ev2[1].record(st)
        torch.cuda.synchronize()
        p_ms = ev2[0].elapsed_time(ev2[1])
        out["persistent_step"] = {"tok_s": round(n_p / (p_ms * 1e-3), 2), "ms_per_token": round(p_ms / n_p, 4),
                                  "tokens": n_p, "launches_per_token": dec.step_kernels,
                                  "tokens_equal_per_op": bool(np.array_equal(
                                      np.concatenate([p_first, p_toks]), np.concatenate([first, toks[:n_p]])))}
        dec.set_step_mode(_TD.STEP_PER_OP)
    dec.close()
    if host_model is not None:
        out["cpu_baseline"] = decode_cpu_baseline(host_model, prompt[:args.decode_cpu_steps], P + G)
    return out


def decode_cpu_baseline(host_model: dict, tokens, max_ctx: int) -> dict:
    """The reference engine itself on the host: the same model written as a
    GGUF file, eos_model_open, then eosi_text_step with the op table the
    engine's dispatch picks on an AVX2 host (oracle/_ref/libeosllm_ref.so,
    compiled from the reference's sources; single-threaded, as the engine
    is), a few steps at positions 0...  Falls back to the C restatement of
    the same step (bit-exact with the engine) where oracle/_ref is absent."""
    import tempfile

    from oracle.oracle import REF_ENGINE
    n = len(tokens)
    if os.path.exists(REF_ENGINE):
        from oracle.gguf_writer import write_llama
        from oracle.llama import RefDecoder
        with tempfile.TemporaryDirectory() as tmp:
            path = os.path.join(tmp, "llama7b.gguf")
            write_llama(path, host_model)
            n_vocab = host_model["config"]["n_vocab"]
            host_model.clear()
            ref = RefDecoder(path, max_ctx, n_vocab)
            t0 = time.perf_counter()
            for t in tokens:
                ref.step(int(t))
            dt = time.perf_counter() - t0
            ref.close()
        return dict(value=round(n / dt, 4), unit="tok/s", cores=1, kind="reference", **host_cpu(),
                    sample=f"{n} steps of the reference engine's eosi_text_step at positions 0.. "
                           "(x86_avx2 matmul_q, scalar rmsnorm/rope/silu; the engine is single-threaded)")
    from oracle.llama import OracleDecoder
    from oracle.oracle import Oracle
    od = OracleDecoder(Oracle(), host_model)
    t0 = time.perf_counter()
    for t in tokens:
        od.step(int(t))
    dt = time.perf_counter() - t0
    od.close()
    return dict(value=round(n / dt, 4), unit="tok/s", cores=1, kind="port", **host_cpu(),
                sample=f"{n} steps of orc_text_step at positions 0.. (C restatement of eosi_text_step)")


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
