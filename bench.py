"""Benchmark of the streaming semi-CRF scan on B200 (one JSON line on rank 0).

Workload ("batched genomic-window training"): per rank a
batch of B=64 sequences, T=10,000, C=24, K=300, lengths uniform in
[8000, 10000]; cum_scores = prefix sums of N(0,1)/sqrt(C) emissions,
transition / duration_bias ~ N(0, 0.1^2); one step = log-semiring forward +
backward (partition.sum().backward()) through ``semi_crf_streaming_forward``,
plus (N > 1) the NCCL all-reduce of [grad_transition | grad_duration_bias |
loss].  Metric: fwd+bwd positions/s = ranks * B * T / step time (the
reference's definition, benchmarks/benchmark_streaming_scale.py:191-193).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

``--impl reference`` times the reference algorithm on the host CPU (the
float32 oracle port of streaming/pytorch_reference.py, all host threads) on a
bounded sample of the same workload.
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
# reference arm: the float32 oracle port of the reference algorithm on the host
# ---------------------------------------------------------------------------
def cpu_reference_sample(budget_s: float):
    """Time the reference algorithm (float32 oracle, all host threads) on a
    bounded sample of the configuration-2 workload.  Returns (pos/s, info)."""
    import numpy as np

    from inputs import make_streaming_inputs
    from oracle import oracle

    oracle.build()
    threads = oracle.max_threads()
    Ts = 600
    Bs = threads
    inp = make_streaming_inputs(Bs, Ts, K, C, seed=2, gen="cfg2")
    lengths = np.full(Bs, Ts)
    args = (inp["cum_scores"].numpy(), inp["transition"].numpy(), inp["duration_bias"].numpy(),
            lengths, K)
    t0 = time.perf_counter()
    oracle.forward_backward(*args, dtype=np.float32, threads=threads)
    dt = time.perf_counter() - t0
    return Bs * Ts / dt, {"threads": threads, "sample": f"B={Bs} T={Ts} K={K} C={C} fwd+bwd "
                                                        "(float32 oracle port, steady-state "
                                                        "truncated T)", "seconds": dt,
                          "fn": lambda: oracle.forward_backward(*args, dtype=np.float32,
                                                                threads=threads),
                          "positions": Bs * Ts}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    rate, info = cpu_reference_sample(budget_s=10)
    for _ in range(args.warmup):
        pass  # the calibration call above is the warm-up
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        info["fn"]()
        times.append(time.perf_counter() - t0)
    step = statistics.mean(times)
    value = info["positions"] / step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cfg2 sample ({info['sample']})", "B": B, "T": T, "K": K, "C": C},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": info["threads"],
                         "kind": "port", "sample": info["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def profiled_traffic():
    """DRAM bytes (read + write) per launch of the dominant kernel from the
    committed ncu summary (profiles/lchain_ws_kernel_cfg2.txt), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", "lchain_ws_kernel_cfg2.txt")):
            if line.startswith("traffic_bytes_per_launch_full_size:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def make_workload(rank, device):
    import torch

    from inputs import config_lengths, make_streaming_inputs

    inp = make_streaming_inputs(B, T, K, C, seed=2 + 1000 * rank, gen="cfg2")
    lengths = config_lengths("cfg2", B, T, seed=2 + 1000 * rank)
    return (inp["cum_scores"], inp["transition"].to(device), inp["duration_bias"].to(device),
            lengths)


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
    from torch_semimarkov_b200.distributed import SharedGradReducer

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.viterbi_only:
        if rank == 0:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            print(json.dumps(bench_viterbi(dev, flush)), flush=True)
        return
    if args.kcc_only:
        if rank == 0:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            print(json.dumps(bench_fwd_bwd(
                dev, flush, "cfg2", B, T, K, C,
                f"cfg2 shape with (K, C, C) transitions: B={B} T={T} K={K} C={C}", kcc=True)),
                flush=True)
        return
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    cum_host, tr, db, lengths_h = make_workload(rank, dev)
    cum_pinned = cum_host.pin_memory()
    cum = cum_host.to(dev)
    lengths = lengths_h.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    reducer = SharedGradReducer(C, K, dev)

    def step(cum_in):
        cum_l = cum_in.detach().requires_grad_(True)
        tr_l = tr.detach().requires_grad_(True)
        db_l = db.detach().requires_grad_(True)
        part = semi_crf_streaming_forward(cum_l, tr_l, db_l, lengths, K)
        loss = part.sum()
        loss.backward()
        if world > 1:
            # the step's one collective: [grad_tr | grad_db | loss] summed over ranks
            gt, gd, lsum = reducer(tr_l.grad, db_l.grad, loss)
            return lsum, gt, gd
        return loss, tr_l.grad, db_l.grad

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 1)):
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
    ms = [a.elapsed_time(b) for a, b in evs]
    t_step = statistics.mean(ms) / 1e3
    tt = torch.tensor([t_step], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_step = float(tt)
    value = world * B * T / t_step

    # ---- end to end: pinned host -> device, fwd+bwd, result -> host ----
    # As a data loader runs it: a copy stream uploads step i+1's cum_scores
    # into the second device buffer while step i computes; every step's
    # upload and its result download are inside the timed region.
    out_host = torch.empty(2, C * C + K * C + 1, dtype=torch.float32).pin_memory()
    bufs = [cum, torch.empty_like(cum)]
    copy_stream = torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream(dev)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def pipeline(n):
        # step 0's upload is exposed; steps 1.. upload behind the previous step
        copy_stream.wait_stream(main)
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
            main.wait_event(uploaded[cur])
            loss, gt, gd = step(bufs[cur])
            res = torch.cat([gt.flatten(), gd.flatten(), loss.detach().view(1)])
            out_host[cur].copy_(res, non_blocking=True)
            consumed[cur].record(main)

    pipeline(3)  # untimed: warms the second buffer and the allocator's blocks for it
    n_e2e = max(10, args.steps)
    flush.zero_()
    barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(main)
    pipeline(n_e2e)
    b_.record(main)
    torch.cuda.synchronize()
    te = torch.tensor([a.elapsed_time(b_) / n_e2e / 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * B * T / float(te)
    del bufs

    # ---- the kernels of one step, timed alone: the forward launch (alpha and
    # beta chains side by side, the dominant kernel) and the backward kernels
    prob = _lib.Problem(cum, tr, db, lengths, K, "log")
    gout = torch.ones(B, dtype=torch.float32, device=dev)
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

    viterbi = None
    others = {}
    if not args.no_viterbi and rank == 0:
        viterbi = bench_viterbi(dev, flush)
        others["chromosome"] = bench_fwd_bwd(dev, flush, "cfg3", 1, 1_000_000, 1000, 8,
                                             "cfg3: B=1 T=1e6 K=1000 C=8, one GPU")
        others["large_C"] = bench_fwd_bwd(dev, flush, "cfg4", 32, 4096, 64, 256,
                                          "cfg4: B=32 T=4096 K=64 C=256")
        others["duration_transitions"] = bench_fwd_bwd(
            dev, flush, "cfg2", 64, 10000, 300, 24,
            "cfg2 shape with (K, C, C) duration-dependent transitions ~N(0, 0.1^2): "
            "B=64 T=10000 K=300 C=24", kcc=True)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, info = cpu_reference_sample(budget_s=10)
        cpu = {"value": rate, "unit": UNIT, "cores": info["threads"], "kind": "port",
               "sample": info["sample"]}

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
    # algorithmic bytes of one forward launch over the actual lengths (rows
    # 0..L of each sequence): cum_scores read by each of the two chains, their
    # float64 tables written (2C+1 doubles per row and chain), log Z and the
    # partition written
    lsum = int(lengths_h.sum())
    rows = lsum + B
    bytes_fwd = 2 * (4 * C + 8 * (2 * C + 1)) * rows + B * (4 + 8)
    achieved = bytes_fwd / t_fwd / 1e9
    # float64 FMAs of the factorised recurrence per forward launch: per
    # position and chain, the C x C mat-vec and the (K-1) x C duration sums
    kcap = max(K - 1, 1)
    fmas = 2 * lsum * (C * C + kcap * C)
    traffic = profiled_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"cfg2 genomic windows: per rank B={B} T={T} K={K} C={C}, "
                               "lengths U[0.8T,T], log fwd+bwd (float32 in/out, float64 "
                               "arithmetic)",
                   "global_batch": B * world, "seq_len": T, "K": K, "C": C,
                   "parallelism": f"dp{world} (batch-sharded, weak)",
                   "l2": "flushed (256 MiB write) between timed steps"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4 * B * (T + 1) * C,
                "d2h_bytes_per_step": 4 * (C * C + K * C + 1),
                "note": "pinned uploads on a copy stream, double-buffered against compute; every timed step uploads its own inputs (step 0 exposed)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "peak_source": peak_src,
                     "kernel": "lchain_ws_kernel<32,8>: alpha and beta chains, 2B CTAs",
                     "kernel_ms": t_fwd * 1e3, "backward_kernels_ms": t_bwd * 1e3,
                     "note": "HBM is not binding: each chain is a serial recurrence over T "
                             "(one CTA per chain), bound by its per-position latency; see "
                             "compute_roofline"},
        "compute_roofline": {"fp64_fma_per_launch": fmas,
                             "achieved_fp64_tflops": 2 * fmas / t_fwd / 1e12,
                             "ns_per_position_step": t_fwd / T * 1e9,
                             "ctas": 2 * B, "sms": torch.cuda.get_device_properties(dev)
                             .multi_processor_count},
        # the reference's O(T K C^2) formulation does (K-1) C^2 semiring edge
        # terms per position and pass, four passes per fwd+bwd (forward, alpha
        # recompute, beta, marginals); this is the rate at which the same
        # result is produced in those units (not work this build executes)
        "reference_equivalent": {"edge_terms_per_position_pass": kcap * C * C, "passes": 4,
                                 "edge_terms_per_s": 4 * kcap * C * C * B * T / t_step},
        # per step: forward = prep (2) + chains (1) + chain_fix (returns at once
        # unless a clamp clipped); backward = pos, blk, tr, db, db_fix (returns at
        # once unless a sequence was flagged), reduce
        "gpu_launches": 10 * args.steps,
        "clocks": clocks,
    }
    if viterbi:
        line["viterbi"] = viterbi
    line.update(others)
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def bench_fwd_bwd(dev, flush, gen, Bc, Tc, Kc, Cc, label, kcc=False):
    """fwd+bwd positions/s of another configuration (inputs resident)."""
    import torch

    from inputs import config_lengths, make_streaming_inputs
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    inp = make_streaming_inputs(Bc, Tc, Kc, Cc, seed=3, gen=gen, kcc=kcc)
    cum = inp["cum_scores"].to(dev)
    tr = inp["transition"].to(dev)
    db = inp["duration_bias"].to(dev)
    lengths = torch.full((Bc,), Tc, dtype=torch.int64, device=dev)

    def one():
        c = cum.detach().requires_grad_(True)
        t = tr.detach().requires_grad_(True)
        d = db.detach().requires_grad_(True)
        semi_crf_streaming_forward(c, t, d, lengths, Kc).sum().backward()

    for _ in range(2):
        one()
    ms = []
    for _ in range(3):
        flush.zero_()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        one()
        b_.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b_))
    t = statistics.mean(ms) / 1e3
    return {"metric": "fwd+bwd positions/s", "value": Bc * Tc / t, "unit": UNIT,
            "ms": t * 1e3, "config": label}


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
