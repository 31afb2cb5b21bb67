"""Benchmark of the streaming semi-CRF scan on B200 (one JSON line on rank 0).

Workload ("batched genomic-window training"): a global
batch of B=64 sequences, T=10,000, C=24, K=300, lengths uniform in
[8000, 10000]; cum_scores = prefix sums of N(0,1)/sqrt(C) emissions,
transition / duration_bias ~ N(0, 0.1^2); one step = log-semiring forward +
backward (partition.sum().backward()) through ``semi_crf_streaming_forward``,
plus (N > 1) the NCCL all-reduce of [grad_transition | grad_duration_bias |
loss].  Metric: fwd+bwd positions/s = B * T / step time (the reference's
definition, benchmarks/benchmark_streaming_scale.py:191-193).

Scaling is strong: the same global batch is split over the N ranks (32/16/8
sequences per GPU at N = 2/4/8, longest first to the least-loaded rank), and
the step time is the maximum over ranks.  At N > 1 a "weak" sub-object also
reports B=64 sequences per rank.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

``--impl reference`` times the reference algorithm on the host CPU (the
float32 oracle port of streaming/pytorch_reference.py, all host threads) on a
bounded sample of the same workload, by the slope method (two sequence
lengths past the K ramp; their time difference is the steady-state cost).
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
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

B, T, K, C = 64, 10_000, 300, 24
METRIC = "fwd+bwd positions/sec (B*T/s) at C=24,K=300"
UNIT = "positions/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-viterbi", action="store_true")
    # smaller per-rank batches / sequences, e.g. for profiler captures of one
    # kernel; the benchmark line is only the configuration-2 number at the defaults
    # only the configuration-5 Viterbi sub-benchmark (e.g. for a profiler)
    ap.add_argument("--viterbi-only", action="store_true")
    # only the (K, C, C)-transition fwd+bwd sub-benchmark, at --batch / --seq-len
    ap.add_argument("--kcc-only", action="store_true")
    ap.add_argument("--large-c-only", action="store_true",
                    help="only configuration 4's fwd+bwd (B=32 T=4096 K=64 C=256), for "
                         "profiler captures; with --batch/--seq-len below the defaults, "
                         "that smaller shape")
    ap.add_argument("--probe-only", action="store_true",
                    help="only the float64 FMA / tensor-core rate probes")
    ap.add_argument("--batch", type=int, default=B)
    ap.add_argument("--seq-len", type=int, default=T)
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU while the timed region
    runs.  An NVML thread polls every 5 ms (queries only; nothing is set); the
    first sample is taken before start() returns, so a timed region of a few
    tens of milliseconds still gets a dozen samples.  nvidia-smi is the fallback
    when the NVML bindings are missing."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("sw_power_cap", 0x4))

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.thread = None

    def start(self):
        if self._start_nvml():
            return
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 5 and os.path.getsize(self.path) == 0:
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def _start_nvml(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None)
            if reasons is None:
                reasons = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            return False
        self.samples = []
        self.halt = threading.Event()

        def poll():
            while not self.halt.is_set():
                try:
                    self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(
                        h, pynvml.NVML_CLOCK_SM)), int(reasons(h))))
                except Exception:
                    pass
                self.halt.wait(0.005)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.samples and time.time() - t0 < 2:
            time.sleep(0.001)
        return True

    def stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join(timeout=2)
            if not self.samples:
                return None
            reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS if r & bit})
            return {"sm_mhz": statistics.median(c for c, _ in self.samples),
                    "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, 5 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi, 50 ms"}


# ---------------------------------------------------------------------------
# CPU legs: the float32 oracle port of the reference algorithm (the reference
# arm) and the reference's own PyTorch path, timed on the host cores
# ---------------------------------------------------------------------------
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class PortSample:
    """Steady-state fwd+bwd rate of the float32 oracle port on all host threads,
    by the slope method: B = threads sequences of configuration 2 at lengths T1
    and T2 (both past the K-1 ramp); one sample = B * (T2 - T1) positions in
    t(T2) - t(T1) seconds.  The thread count is passed explicitly, because
    torchrun sets OMP_NUM_THREADS=1."""

    def __init__(self, T1=400, T2=800):
        import numpy as np

        from inputs import make_streaming_inputs
        from oracle import oracle

        oracle.build()
        self.np, self.oracle = np, oracle
        self.threads = host_threads()
        self.B, self.T1, self.T2 = self.threads, T1, T2
        inp = make_streaming_inputs(self.B, T2, K, C, seed=2, gen="cfg2")
        self.cum = inp["cum_scores"].numpy()
        self.tr = inp["transition"].numpy()
        self.db = inp["duration_bias"].numpy()
        self.sample = (f"float32 oracle port, B={self.B} (one sequence per thread), K={K}, "
                       f"C={C}, fwd+bwd at T={T1} and T={T2}, slope")

    def _run(self, Tn):
        np = self.np
        t0 = time.perf_counter()
        self.oracle.forward_backward(self.cum[:, : Tn + 1], self.tr, self.db,
                                     np.full(self.B, Tn), K, dtype=np.float32,
                                     threads=self.threads)
        return time.perf_counter() - t0

    def step(self):
        """(positions, seconds) of one slope sample."""
        return self.B * (self.T2 - self.T1), self._run(self.T2) - self._run(self.T1)


def reference_pytorch_sample(T1=300, T2=340, Bs=64, budget_s=120.0):
    """The reference's own CPU streaming path (torch_semimarkov 0.2.0 installed
    offline in baseline/_ref, ``semi_crf_streaming_forward(..., use_triton=False)``
    forward + backward, float32, torch on all host threads) on configuration 2's
    inputs, by the slope method: B=64 at T1 and T2 just past the K-1 ramp,
    after a short warm-up call.  Its Python loop dispatches about ten torch
    ops per (position, duration) whatever the batch, so each length costs tens
    of seconds; if T1 alone exceeds budget_s the rate is B*T1/t(T1), which
    includes the cheaper ramp and so overstates the steady state.  Returns
    None when the reference is not installed."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "torch_semimarkov")):
        return None
    import torch

    if ref not in sys.path:
        sys.path.insert(0, ref)
    from torch_semimarkov.streaming import semi_crf_streaming_forward as ref_forward

    from inputs import make_streaming_inputs

    threads = host_threads()
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        inp = make_streaming_inputs(Bs, T2, K, C, seed=2, gen="cfg2")

        def run(Tn):
            cum = inp["cum_scores"][:, : Tn + 1].clone().requires_grad_(True)
            tr = inp["transition"].clone().requires_grad_(True)
            db = inp["duration_bias"].clone().requires_grad_(True)
            t0 = time.perf_counter()
            ref_forward(cum, tr, db, torch.full((Bs,), Tn), K, use_triton=False).sum().backward()
            return time.perf_counter() - t0

        run(8)  # warm-up: torch's lazy initialisation of the ops involved
        t1 = run(T1)
        t2 = run(T2) if t1 <= budget_s else None
    finally:
        torch.set_num_threads(old)
    base = (f"reference PyTorch path (torch_semimarkov 0.2.0, use_triton=False), float32, "
            f"B={Bs}, K={K}, C={C}, fwd+bwd")
    if t2 is not None and t2 - t1 > 0.1 * t1:
        return {"value": Bs * (T2 - T1) / (t2 - t1), "unit": UNIT, "cores": threads,
                "kind": "reference",
                "sample": f"{base} at T={T1} and T={T2}, slope ({t1:.1f} s and {t2:.1f} s)"}
    return {"value": Bs * T1 / t1, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{base} at T={T1} ({t1:.1f} s), one point: includes the K-1 ramp, "
                      "which overstates the steady-state rate"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    ps = PortSample()
    for _ in range(args.warmup):
        ps.step()
    pos = secs = 0.0
    for _ in range(args.steps):
        n, dt = ps.step()
        pos += n
        secs += dt
    value = pos / secs
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": B * T / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cfg2 genomic windows (B={B} T={T} K={K} C={C}), sampled: "
                               f"{ps.sample}", "global_batch": B, "seq_len": T, "K": K, "C": C},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": ps.threads, "kind": "port",
                         "sample": ps.sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ms_per_step extrapolates the sampled steady-state rate to one full "
                "configuration-2 step",
    }
    if args.gpus == 1:
        # the reference's own PyTorch code beside the port (informational)
        try:
            ref_pt = reference_pytorch_sample()
        except Exception as exc:
            ref_pt = {"unavailable": f"{type(exc).__name__}: {exc}"}
        if ref_pt:
            line["cpu_baseline_reference_pytorch"] = ref_pt
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def profiled_traffic():
    """DRAM bytes (read + write) per launch of the dominant kernel at B=64 from the
    committed ncu summary (profiles/lchain_ws_kernel_cfg2.txt), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", "lchain_ws_kernel_cfg2.txt")):
            if line.startswith("traffic_bytes_per_launch_full_size:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def global_workload(Bg, Tg, seed=2):
    """Configuration 2's global batch (CPU tensors): every rank generates the
    same one and keeps its shard."""
    from inputs import config_lengths, make_streaming_inputs

    inp = make_streaming_inputs(Bg, Tg, K, C, seed=seed, gen="cfg2")
    lengths = config_lengths("cfg2", Bg, Tg, seed=seed)
    return inp["cum_scores"], inp["transition"], inp["duration_bias"], lengths


def fp64_probe(dev):
    """Measured float64 FMA peak of this GPU (TFLOP/s, all SMs, 8 independent
    chains per thread) and the cycles of one dependent float64 FMA."""
    import ctypes

    import torch

    path = os.path.join(ROOT, "torch_semimarkov_b200", "libsemicrf_probe.so")
    lib = ctypes.CDLL(path)
    lib.semicrf_probe_fp64_fma.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                           ctypes.c_void_p]
    lib.semicrf_probe_fp64_latency.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p]
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    grid, iters, nt = nsm * 8, 4096, 256
    out = torch.empty(grid * nt, dtype=torch.float64, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    best = None
    for _ in range(4):
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        assert lib.semicrf_probe_fp64_fma(grid, iters, ctypes.c_void_p(out.data_ptr()), st) == 0
        b_.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b_)
        best = ms if best is None else min(best, ms)
    fmas = grid * nt * iters * 32
    cyc = torch.zeros(1, dtype=torch.int64, device=dev)
    o32 = torch.empty(32, dtype=torch.float64, device=dev)
    assert lib.semicrf_probe_fp64_latency(1024, ctypes.c_void_p(cyc.data_ptr()),
                                          ctypes.c_void_p(o32.data_ptr()), st) == 0
    torch.cuda.synchronize()
    dfma_lat = float(cyc) / (1024 * 16)
    # the float64 tensor-core path (mma.sync m8n8k4 f64), the candidate for
    # the large-C contraction: throughput and dependent latency
    lib.semicrf_probe_dmma.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p]
    lib.semicrf_probe_dmma_latency.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p]
    dbest = None
    diters = 1024
    for _ in range(4):
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        assert lib.semicrf_probe_dmma(grid, diters, ctypes.c_void_p(out.data_ptr()), st) == 0
        b_.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b_)
        dbest = ms if dbest is None else min(dbest, ms)
    dfmas = grid * (nt // 32) * diters * 16 * 256
    assert lib.semicrf_probe_dmma_latency(256, ctypes.c_void_p(cyc.data_ptr()),
                                          ctypes.c_void_p(o32.data_ptr()), st) == 0
    torch.cuda.synchronize()
    return {"fp64_tflops": 2 * fmas / (best / 1e3) / 1e12,
            "dfma_latency_cycles": dfma_lat,
            "fp64_tensor_tflops": 2 * dfmas / (dbest / 1e3) / 1e12,
            "dmma_latency_cycles": float(cyc) / (256 * 16),
            "how": f"{grid} CTAs x {nt} threads x 8 independent FMA chains x {iters * 4} "
                   "FMAs, best of 4, CUDA events (probe.cu); latency: one warp, one chain, "
                   "clock64"}


def main():
    global B, T
    args = parse()
    B, T = args.batch, args.seq_len
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from torch_semimarkov_b200 import _lib, semi_crf_streaming_forward
    from torch_semimarkov_b200.distributed import SharedGradReducer, shard_sequences

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.viterbi_only:
        if rank == 0:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            print(json.dumps(bench_viterbi(dev, flush)), flush=True)
        return
    if args.large_c_only:
        if rank == 0:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            bc = 32 if B == 64 else B
            tc = 4096 if T == 10000 else T
            print(json.dumps(bench_fwd_bwd(dev, flush, "cfg4", bc, tc, 64, 256, 4,
                                           f"cfg4: B={bc} T={tc} K=64 C=256")), flush=True)
        return
    if args.probe_only:
        if rank == 0:
            print(json.dumps(fp64_probe(dev)), flush=True)
        return
    if args.kcc_only:
        if rank == 0:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            print(json.dumps(bench_fwd_bwd(
                dev, flush, "cfg2", B, T, K, C, 2,
                f"cfg2 shape with (K, C, C) transitions: B={B} T={T} K={K} C={C}", kcc=True)),
                flush=True)
        return
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    # ---- this rank's shard of the global batch (strong scaling) ----
    cum_all, tr_h, db_h, len_all = global_workload(B, T)
    mine = shard_sequences(len_all, world, rank)
    Bl = int(mine.numel())
    cum_host = cum_all[mine].contiguous()
    lengths_h = len_all[mine].contiguous()
    del cum_all
    tr, db = tr_h.to(dev), db_h.to(dev)
    cum_pinned = cum_host.pin_memory()
    cum = cum_host.to(dev)
    lengths = lengths_h.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    reducer = SharedGradReducer(C, K, dev)

    def make_step(lengths_d):
        def step(cum_in):
            cum_l = cum_in.detach().requires_grad_(True)
            tr_l = tr.detach().requires_grad_(True)
            db_l = db.detach().requires_grad_(True)
            part = semi_crf_streaming_forward(cum_l, tr_l, db_l, lengths_d, K)
            loss = part.sum()
            loss.backward()
            if world > 1:
                # the step's one collective: [grad_tr | grad_db | loss] summed over ranks
                gt, gd, lsum = reducer(tr_l.grad, db_l.grad, loss)
                return lsum, gt, gd
            return loss, tr_l.grad, db_l.grad
        return step

    step = make_step(lengths)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        tt = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt)

    for _ in range(max(args.warmup, 3)):
        step(cum)
    barrier()

    # ---- device-resident timed region (L2 flushed between steps) ----
    sampler = ClockSampler(local)
    sampler.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush.zero_()
        evs[i][0].record()
        step(cum)
        evs[i][1].record()
    barrier()
    clocks = sampler.stop()
    t_step = max_over_ranks(statistics.mean(a.elapsed_time(b_) for a, b_ in evs) / 1e3)
    value = B * T / t_step

    # ---- end to end: pinned host -> device, fwd+bwd, result -> host ----
    # As a data loader runs it: a copy stream uploads step i+1's cum_scores
    # into the second device buffer while step i computes; every step's
    # upload and its result download are inside the timed region.
    out_host = torch.empty(2, C * C + K * C + 1, dtype=torch.float32).pin_memory()
    bufs = [cum, torch.empty_like(cum)]
    copy_stream = torch.cuda.Stream(device=dev)
    main_s = torch.cuda.current_stream(dev)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def pipeline(n):
        # step 0's upload is exposed; steps 1.. upload behind the previous step
        copy_stream.wait_stream(main_s)
        with torch.cuda.stream(copy_stream):
            bufs[0].copy_(cum_pinned, non_blocking=True)
            uploaded[0].record(copy_stream)
        for i in range(n):
            cur = i % 2
            if i + 1 < n:
                nxt = (i + 1) % 2
                with torch.cuda.stream(copy_stream):
                    if i >= 1:
                        copy_stream.wait_event(consumed[nxt])  # step i-1 is done with it
                    bufs[nxt].copy_(cum_pinned, non_blocking=True)
                    uploaded[nxt].record(copy_stream)
            main_s.wait_event(uploaded[cur])
            loss, gt, gd = step(bufs[cur])
            res = torch.cat([gt.flatten(), gd.flatten(), loss.detach().view(1)])
            out_host[cur].copy_(res, non_blocking=True)
            consumed[cur].record(main_s)

    pipeline(3)  # untimed: warms the second buffer and the allocator's blocks for it
    n_e2e = max(10, args.steps)
    flush.zero_()
    barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(main_s)
    pipeline(n_e2e)
    b_.record(main_s)
    torch.cuda.synchronize()
    te = max_over_ranks(a.elapsed_time(b_) / n_e2e / 1e3)
    e2e_value = B * T / te
    del bufs

    # ---- the kernels of one step, timed alone: the forward launch (alpha and
    # beta chains side by side, the dominant kernel) and the backward kernels
    prob = _lib.Problem(cum, tr, db, lengths, K, "log")
    lib = _lib.load()
    import ctypes

    p_off = _lib.SemicrfProblem.from_buffer_copy(prob.c)
    p_off.chunk_warmup = -1
    chunked = lib.semicrf_saved_size(prob.cref) > lib.semicrf_saved_size(ctypes.byref(p_off))
    gout = torch.ones(Bl, dtype=torch.float32, device=dev)
    saved = None
    for _ in range(2):
        _, _, saved = _lib.forward(prob, want_saved=True)
        _lib.backward(prob, saved, gout)
    fe = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(3)]
    for e0, e1, e2, e3 in fe:
        flush.zero_()
        e0.record()
        _, _, saved = _lib.forward(prob, want_saved=True)
        e1.record()
        flush.zero_()
        e2.record()
        _lib.backward(prob, saved, gout)
        e3.record()
    torch.cuda.synchronize()
    t_fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in fe) / 1e3
    t_bwd = statistics.mean(e[2].elapsed_time(e[3]) for e in fe) / 1e3
    del saved

    # ---- weak scaling beside it (N > 1): B=64 sequences per rank ----
    weak = None
    if world > 1:
        cw, _, _, lw = global_workload(B, T, seed=2 + 1000 * rank)
        cw, lw = cw.to(dev), lw.to(dev)
        step_w = make_step(lw)
        for _ in range(3):
            step_w(cw)
        barrier()
        ew = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(10)]
        for e0, e1 in ew:
            flush.zero_()
            e0.record()
            step_w(cw)
            e1.record()
        barrier()
        tw = max_over_ranks(statistics.mean(x.elapsed_time(y) for x, y in ew) / 1e3)
        weak = {"metric": METRIC, "value": world * B * T / tw, "unit": UNIT,
                "ms_per_step": tw * 1e3, "scaling": "weak",
                "config": f"B={B} sequences per rank (global {world * B}), 10 steps"}
        del cw

    probe = fp64_probe(dev)

    viterbi = None
    others = {}
    if not args.no_viterbi and world == 1:
        viterbi = bench_viterbi(dev, flush)
        others["head_cfg1"] = bench_head_cfg1(dev, flush)
        others["chromosome"] = bench_fwd_bwd(dev, flush, "cfg3", 1, 1_000_000, 1000, 8, 3,
                                             "cfg3: B=1 T=1e6 K=1000 C=8, one GPU")
        others["large_C"] = bench_fwd_bwd(dev, flush, "cfg4", 32, 4096, 64, 256, 4,
                                          "cfg4: B=32 T=4096 K=64 C=256")
        others["duration_transitions"] = bench_fwd_bwd(
            dev, flush, "cfg2", 64, 10000, 300, 24, 2,
            "cfg2 shape with (K, C, C) duration-dependent transitions ~N(0, 0.1^2): "
            "B=64 T=10000 K=300 C=24", kcc=True)

    cpu = cpu_ref = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ps = PortSample()
        ps.step()  # warm
        n, dt = ps.step()
        cpu = {"value": n / dt, "unit": UNIT, "cores": ps.threads, "kind": "port",
               "sample": ps.sample}
        try:
            cpu_ref = reference_pytorch_sample()
        except Exception as exc:  # the reference leg is informational
            cpu_ref = {"unavailable": f"{type(exc).__name__}: {exc}"}

    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    # Algorithmic bytes of one forward launch (the survey's per-position
    # figures, over this rank's actual lengths): the cum_scores stream read
    # once per pass (alpha and beta chains: 2 x 4C bytes per row) plus the
    # reference's ring checkpoints, K*C*4/S bytes per position.  The float64
    # tables this design writes for its parallel backward are reported apart
    # as design_bytes.
    lsum = int(lengths_h.sum())
    rows = lsum + Bl
    S = max(K, int(math.sqrt(T * K)))
    bytes_alg = 2 * 4 * C * rows + lsum * K * C * 4 / S
    design_bytes = 2 * 8 * (2 * C + 1) * rows + Bl * (4 + 8)
    achieved = bytes_alg / t_fwd / 1e9
    traffic = profiled_traffic()
    if traffic is not None:
        # the capture was of the B=64 launch; a shard's launch moves the same
        # bytes per row
        traffic *= rows / (int(len_all.sum()) + len(len_all))
    # float64 FMAs of the factorised recurrence per forward launch: per
    # position and chain, the C x C mat-vec and the (K-1) x C duration sums
    kcap = max(K - 1, 1)
    fmas = 2 * lsum * (C * C + kcap * C)
    fp64_tf = 2 * fmas / t_fwd / 1e12
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    launches_fwd = 4 + (7 if chunked else 0)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"cfg2 genomic windows: global B={B} T={T} K={K} C={C}, "
                               "lengths U[0.8T,T], log fwd+bwd (float32 in/out, float64 "
                               "arithmetic), batch split over the ranks",
                   "global_batch": B, "per_rank_batch": Bl, "seq_len": T, "K": K, "C": C,
                   "parallelism": f"dp{world} (batch-sharded, strong)",
                   "time_chunked": bool(chunked),
                   "l2": "flushed (256 MiB write) between timed steps"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4 * Bl * (T + 1) * C,
                "d2h_bytes_per_step": 4 * (C * C + K * C + 1),
                "note": "per rank: pinned uploads of its shard on a copy stream, "
                        "double-buffered against compute; every timed step uploads its own "
                        "inputs (step 0 exposed); max over ranks"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": bytes_alg,
                     "design_bytes_per_launch": design_bytes,
                     "kernel": "lchain_ws_kernel<32,8>: alpha and beta chains"
                               + (" in time chunks" if chunked else ", 2B CTAs"),
                     "kernel_ms": t_fwd * 1e3, "backward_kernels_ms": t_bwd * 1e3,
                     "note": "algorithmic bytes per the survey: 4C per row and pass of the "
                             "cum_scores stream plus K*C*4/S checkpoint bytes per position; "
                             "HBM is not binding (each chain is a serial recurrence); see "
                             "compute_roofline"},
        "compute_roofline": {"bound": "fp64", "unit": "TFLOP/s",
                             "fp64_fma_per_launch": fmas, "achieved": fp64_tf,
                             "peak": probe["fp64_tflops"], "frac": fp64_tf / probe["fp64_tflops"],
                             "peak_source": "measured in this run: " + probe["how"],
                             "dfma_latency_cycles": probe["dfma_latency_cycles"],
                             "fp64_tensor_tflops": probe["fp64_tensor_tflops"],
                             "dmma_latency_cycles": probe["dmma_latency_cycles"],
                             "ns_per_position_step": t_fwd / int(lengths_h.max()) * 1e9,
                             "ctas": 2 * Bl, "sms": nsm,
                             "note": "the factorised recurrence's float64 FMAs (C*C + (K-1)*C "
                                     "per position and chain) over the forward launch time"},
        # the reference's O(T K C^2) formulation does (K-1) C^2 semiring edge
        # terms per position and pass, four passes per fwd+bwd (forward, alpha
        # recompute, beta, marginals); this is the rate at which the same
        # result is produced in those units (not work this build executes)
        "reference_equivalent": {"edge_terms_per_position_pass": kcap * C * C, "passes": 4,
                                 "edge_terms_per_s": 4 * kcap * C * C * B * T / t_step},
        # per step: forward = prep_max, prep, chains, chain_fix (returns at once
        # unless a clamp clipped), and when time-chunked the boundary check,
        # prefix and fix-up per direction and the rerun of unjoined sequences;
        # backward = pos, blk, tr, db, db_fix (returns at once unless a sequence
        # was flagged), reduce
        "gpu_launches": (launches_fwd + 6) * args.steps,
        "clocks": clocks,
    }
    if weak:
        line["weak"] = weak
    if viterbi:
        line["viterbi"] = viterbi
    line.update(others)
    if cpu:
        line["cpu_baseline"] = cpu
    if cpu_ref:
        line["cpu_baseline_reference_pytorch"] = cpu_ref
    print(json.dumps(line), flush=True)


def bench_fwd_bwd(dev, flush, gen, Bc, Tc, Kc, Cc, seed, label, kcc=False):
    """fwd+bwd positions/s of another configuration (inputs resident)."""
    import torch

    from inputs import config_lengths, make_streaming_inputs
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    inp = make_streaming_inputs(Bc, Tc, Kc, Cc, seed=seed, gen=gen, kcc=kcc)
    cum = inp["cum_scores"].to(dev)
    tr = inp["transition"].to(dev)
    db = inp["duration_bias"].to(dev)
    lengths = config_lengths(gen, Bc, Tc, seed=seed).to(dev)

    def one():
        c = cum.detach().requires_grad_(True)
        t = tr.detach().requires_grad_(True)
        d = db.detach().requires_grad_(True)
        semi_crf_streaming_forward(c, t, d, lengths, Kc).sum().backward()

    for _ in range(2):
        one()
    ms = []
    for _ in range(5):
        flush.zero_()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        one()
        b_.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b_))
    # the median of five steps: on some boxes single steps of configuration 4
    # ran 2-5x slower at random iterations (its cluster launch needs 32 of the
    # 33 resident cluster slots); every step's time is reported beside it
    t = statistics.median(ms) / 1e3
    return {"metric": "fwd+bwd positions/s", "value": Bc * Tc / t, "unit": UNIT,
            "ms": t * 1e3, "ms_steps": [round(x, 3) for x in ms], "config": label}


def bench_head_cfg1(dev, flush):
    """Configuration 1 through the public module: SemiMarkovCRFHead(24, 100,
    hidden_dim=512) with a Xavier-initialised projection; one step =
    compute_loss (projection, cumsum, partition, gold score) + backward +
    decode_with_traceback, B=4, T=1000."""
    import torch

    from inputs import make_hidden
    from torch_semimarkov_b200 import SemiMarkovCRFHead

    Bh, Th, Kh, Ch, H = 4, 1000, 100, 24, 512
    h = make_hidden(Bh, Th, Ch, Kh, seed=1, gen="cfg1", hidden_dim=H)
    head = SemiMarkovCRFHead(Ch, Kh, hidden_dim=H).to(dev)
    with torch.no_grad():
        head.transition.copy_(h["transition"])
        head.duration_dist.duration_bias.copy_(h["duration_bias"])
        head.projection.weight.copy_(h["proj_weight"])
        head.projection.bias.copy_(h["proj_bias"])
    hidden = h["hidden"].to(dev)
    labels = h["labels"].to(dev)
    lengths = torch.full((Bh,), Th, dtype=torch.int64, device=dev)

    def one():
        head.zero_grad(set_to_none=True)
        head.compute_loss(hidden, lengths, labels).backward()
        return head.decode_with_traceback(hidden, lengths)

    for _ in range(3):
        one()
    ms = []
    for _ in range(5):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        one()
        torch.cuda.synchronize()
        ms.append((time.perf_counter() - t0) * 1e3)
    t = statistics.median(ms) / 1e3
    return {"metric": "head positions/s (compute_loss + backward + decode_with_traceback)",
            "value": Bh * Th / t, "unit": UNIT, "ms": t * 1e3,
            "config": "cfg1: SemiMarkovCRFHead(24, 100, hidden_dim=512), B=4 T=1000, "
                      "host wall clock around each step (decode_with_traceback returns "
                      "host Segment lists)"}


def bench_viterbi(dev, flush):
    """Configuration 5: B=512, T=2048, C=16, K=32 max fwd + backpointers + backtrace."""
    import torch

    from inputs import config_lengths, make_streaming_inputs
    from torch_semimarkov_b200 import _lib

    Bv, Tv, Kv, Cv = 512, 2048, 32, 16
    inp = make_streaming_inputs(Bv, Tv, Kv, Cv, seed=5, gen="cfg5")
    lengths = config_lengths("cfg5", Bv, Tv, seed=5).to(dev)
    prob = _lib.Problem(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                        inp["duration_bias"].to(dev), lengths, Kv, "max")
    for _ in range(2):
        _lib.viterbi(prob, 10000)
    ms = []
    for _ in range(5):
        flush.zero_()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _lib.viterbi(prob, 10000)
        b_.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b_))
    t = statistics.mean(ms) / 1e3
    return {"metric": "Viterbi positions/s (max fwd + backpointers + backtrace)",
            "value": Bv * Tv / t, "unit": UNIT, "ms": t * 1e3,
            "config": "cfg5: B=512 T=2048 K=32 C=16 lengths U[1024,2048]"}


if __name__ == "__main__":
    main()
