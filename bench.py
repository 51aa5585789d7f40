"""Benchmark of the fused lm_head cross-entropy head (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]
    (N > 1: launched by torchrun, one process per GPU)

Metric: "lm_head CE fwd+bwd tokens/s (Qwen2.5-1.5B head), % tcgen05 peak, peak MiB".
Workload at N=1: config 2 — Qwen2.5-1.5B tied head H=1536, V=151936, fp16, 4 rows x 512 tokens all
packed (N=2048), labels uniform with 10% = -100, W ~ N(0, 0.02); seeded synthetic data (the
reference's dataset is not available offline). One step = loss forward + backward (dX and dW) through
the public autograd API. N > 1 (weak scaling, default): the head is vocab-sharded over the N GPUs and
the global batch is N x 2048 tokens, so every GPU does the work of one config-2 step; the per-token
statistics are all-gathered over NCCL and dX is summed inside the backward kernel over NVLink SHARP
(fp32 dX of 32 MiB or more) or by an NCCL all-reduce. ``--scaling strong`` keeps 2048 tokens and
splits the vocabulary instead.

``value`` is device-timed with the inputs resident (L2 flushed between steps); ``e2e`` runs the same
steps from pinned host memory, each step's inputs copied on a copy stream while the previous step
computes, all copies, L2 flushes and loss read-backs inside one timed region.

``--impl reference`` times the reference's eager formula (full-logit F.linear in fp16 + fp32 cross
entropy + entropy + argmax + autograd dX/dW; the oracle restatement of solution/test_kernels.py:204-216)
on the host CPU with all threads, on a bounded token sample of the same workload; under torchrun only
rank 0 runs it.
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "lm_head CE fwd+bwd tokens/s (Qwen2.5-1.5B head), % tcgen05 peak, peak MiB"
CONFIGS = {
    # name: (rows, row_len, H, V, dtype, ignored fraction)
    "c2": (4, 512, 1536, 151936, torch.float16, 0.10),
    "c4": (8, 4096, 4096, 128256, torch.bfloat16, 0.0),
}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) of one forward-statistics launch at config 2, from one
# `ncu --set full` capture (dram__bytes_read.sum + dram__bytes_write.sum) of this
# script's second warm-up step.
FWD_STATS_TRAFFIC_C2 = 506_910_000 + 5_596_000
# DRAM bytes of one persistent backward launch at config 2 (same capture; pair kernel).
BWD_TRAFFIC_C2 = 1_974_155_000 + 1_095_150_000


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def make_inputs(cfg, n_tokens, device, seed=0):
    rows, row_len, H, V, dt, ign = CONFIGS[cfg]
    g = torch.Generator(device="cpu").manual_seed(seed)
    X = torch.randn(n_tokens, H, generator=g)
    if cfg == "c2":
        X = X * (1.0 + 0.1 * torch.randn(H, generator=g))
    X = X.to(dt)
    y = torch.randint(0, V, (n_tokens,), generator=g)
    if ign > 0:
        y[torch.rand(n_tokens, generator=g) < ign] = -100
    return X.to(device), y.to(device)


def make_weight(cfg, v_lo, v_hi, device, seed=1):
    rows, row_len, H, V, dt, ign = CONFIGS[cfg]
    # generate on the device shard by shard (deterministic per shard seed)
    g = torch.Generator(device=device).manual_seed(seed * 1000 + v_lo)
    return (torch.randn(v_hi - v_lo, H, generator=g, device=device) * 0.02).to(dt)


class ClockSampler:
    """SM clock and clock-event reasons sampled every 10 ms (NVML) while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            # match the CUDA device to its NVML handle by PCI domain / bus / device numbers
            props = torch.cuda.get_device_properties(self.device)
            want = (int(getattr(props, "pci_domain_id", -1)), int(getattr(props, "pci_bus_id", -1)),
                    int(getattr(props, "pci_device_id", -1)))
            h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                cand = pynvml.nvmlDeviceGetHandleByIndex(i)
                pci = pynvml.nvmlDeviceGetPciInfo(cand)
                if (int(pci.domain), int(pci.bus), int(pci.device)) == want:
                    h = cand
                    break
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    reasons = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                    self.samples.append((mhz, reasons))
                except Exception:
                    pass
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml, 10 ms"}


# ------------------------------------------------------------------ CPU side

def cpu_reference_sample(cfg, sample_tokens, iters, warmup, threads):
    """The reference eager formula on the host CPU over a token sample; returns tokens/s per iteration."""
    from oracle import lmce_oracle as orc

    torch.set_num_threads(threads)
    rows, row_len, H, V, dt, ign = CONFIGS[cfg]
    X, y = make_inputs(cfg, sample_tokens, "cpu", seed=7)
    W = (torch.randn(V, H, generator=torch.Generator().manual_seed(3)) * 0.02).to(dt)
    times = []
    for i in range(warmup + iters):
        t0 = time.perf_counter()
        orc.eager_head(X, y, W, grads=True, grad_mode="eager")
        t1 = time.perf_counter()
        if i >= warmup:
            times.append(t1 - t0)
    return [sample_tokens / t for t in times], times


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = args.cpu_sample_tokens
    tps, times = cpu_reference_sample(args.config, sample, max(args.steps, 1), max(args.warmup, 0), threads)
    value = statistics.median(tps)
    rows, row_len, H, V, dt, ign = CONFIGS[args.config]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(times) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16" if dt == torch.float16 else "bf16", "data": "synthetic",
        "config": {"workload": workload_name(args.config), "H": H, "V": V,
                   "tokens_timed_per_step": sample, "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} tokens of the {args.config} workload per step (fwd+bwd, eager "
                                   f"F.linear fp16 + fp32 CE + entropy + argmax + autograd dX/dW)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_name(cfg):
    if cfg == "c2":
        return "C2 Qwen2.5-1.5B tied head fwd+bwd, H=1536 V=151936 fp16, 4x512 tokens (N=2048), 10% labels -100"
    return "C4 Llama-3-8B head fwd+bwd, H=4096 V=128256 bf16, 8x4096 tokens (N=32768)"


# ------------------------------------------------------------------ GPU side

def stage(msg):
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak")
    ap.add_argument("--v-chunk", type=int, default=0, help="vocab chunk of the backward; 0 = library default")
    ap.add_argument("--cpu-sample-tokens", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if world != args.gpus and "RANK" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch.distributed as dist
    from rus_b200 import _lib, chunked_lm_head
    from rus_b200.sharded import shard_range, sharded_lm_head

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    group = None
    # keep stdout to the one JSON line: NCCL's version banner goes to stdout at init
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    rows, row_len, H, V, dt, ign = CONFIGS[args.config]
    n_per = rows * row_len
    n_tokens = n_per * world if (world > 1 and args.scaling == "weak") else n_per
    v_lo, v_hi = shard_range(V, rank, world) if world > 1 else (0, V)

    X, y = make_inputs(args.config, n_tokens, device)
    W = make_weight(args.config, v_lo, v_hi, device).requires_grad_(True)
    Xg = X.clone().requires_grad_(True)
    n_lab = int((y != -100).sum())
    torch.cuda.synchronize()

    def head(xx, yy):
        if world > 1:
            return sharded_lm_head(xx, yy, W, v_lo, V, group, None, args.v_chunk)
        return chunked_lm_head(xx, yy, W, None, args.v_chunk)

    def step():
        Xg.grad = None
        W.grad = None
        loss, nll, ent, arg = head(Xg, y)
        loss.backward()
        return loss

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # ---- warm-up
    stage("warm-up")
    for _ in range(args.warmup):
        step()
    barrier()

    stage("peak memory")
    # ---- peak activation memory of one step (beyond inputs and the dX/dW outputs)
    Xg.grad = None
    W.grad = None
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(device)
    base = torch.cuda.memory_allocated(device)
    step()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated(device) - base
    out_bytes = Xg.grad.numel() * Xg.grad.element_size() + W.grad.numel() * W.grad.element_size()
    peak_act_mib = max(peak - out_bytes, 0) / 2**20

    # ---- device-timed steps (inputs resident in HBM; L2 flushed between steps). The two
    # tensor-core kernels of each step are also bracketed by events recorded by the library
    # (lmce_set_timing_events) on the launching stream.
    def new_event():
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)  # create the underlying CUDA event before handing it to the library
        return e

    stage("timed steps")
    l0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    kev = {k: [(new_event(), new_event()) for _ in range(args.steps)] for k in (0, 1)}
    torch.cuda.synchronize()
    barrier()
    with ClockSampler(device) as clk:
        for i in range(args.steps):
            flush.zero_()
            for k in (0, 1):
                _lib.call("lmce_set_timing_events", k, kev[k][i][0].cuda_event, kev[k][i][1].cuda_event)
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        barrier()
    for k in (0, 1):
        _lib.call("lmce_set_timing_events", k, None, None)
    launches = _lib.launch_count() - l0
    step_ms = [a.elapsed_time(b) for a, b in ev]
    kern_ms = {k: statistics.mean(a.elapsed_time(b) for a, b in kev[k]) for k in (0, 1)}
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    ms_per_step = total_ms.item() / args.steps
    tokens_per_step = n_tokens
    value = tokens_per_step / (ms_per_step / 1e3)

    stage("end-to-end")
    # ---- end-to-end through the public API: pinned host inputs -> H2D, fwd+bwd, loss D2H.
    # Like a training loop with a prefetching loader, each step's inputs are copied on a
    # copy stream into one of two device buffers while the previous step computes; the
    # timed region (one pair of events on the compute stream) starts before the first
    # copy and ends after the last loss read-back, so every step's copies are inside it.
    # As for `value`, L2 is flushed before every step (on the compute stream, inside the
    # region here), as the layers that run before the head in a training step would.
    Xh = X.cpu().pin_memory()
    yh = y.cpu().pin_memory()
    loss_h = torch.empty(1, dtype=torch.float32).pin_memory()
    Xd = [torch.empty_like(X) for _ in range(2)]
    yd = [torch.empty_like(y) for _ in range(2)]
    copy_stream = torch.cuda.Stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(args.steps // 2, 3)

    def issue_copy(j):
        b = j % 2
        copy_stream.wait_event(done[b])  # the step that last read buffer b has finished
        with torch.cuda.stream(copy_stream):
            Xd[b].copy_(Xh, non_blocking=True)
            yd[b].copy_(yh, non_blocking=True)
            ready[b].record(copy_stream)

    def run_e2e(steps):
        for b in range(2):
            done[b].record(stream)
        issue_copy(0)
        for j in range(steps):
            if j + 1 < steps:
                issue_copy(j + 1)
            flush.zero_()
            stream.wait_event(ready[j % 2])
            xin = Xd[j % 2].detach().requires_grad_(True)
            W.grad = None
            loss, *_ = head(xin, yd[j % 2])
            loss.backward()
            loss_h.copy_(loss.detach().reshape(1), non_blocking=True)
            done[j % 2].record(stream)

    run_e2e(2)  # warm-up of the pipelined loop
    barrier()
    e2e_a = torch.cuda.Event(enable_timing=True)
    e2e_b = torch.cuda.Event(enable_timing=True)
    e2e_a.record(stream)
    copy_stream.wait_stream(stream)
    run_e2e(e2e_steps)
    e2e_b.record(stream)
    barrier()
    ev2 = [(e2e_a, e2e_b)]
    e2e_ms = torch.tensor([sum(a.elapsed_time(b) for a, b in ev2)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms_step = e2e_ms.item() / e2e_steps
    e2e_value = tokens_per_step / (e2e_ms_step / 1e3)
    h2d = Xh.numel() * Xh.element_size() + yh.numel() * yh.element_size()

    stage("report")
    dx_exchange = "none (single GPU)"
    if world > 1:
        from rus_b200.sharded import nvls_dx_exchange
        dx_exchange = ("in-kernel NVLink SHARP exchange (multimem.ld_reduce + multimem.st)"
                       if nvls_dx_exchange(n_tokens, H, dt, device, group) is not None else "NCCL all-reduce (fp32)")
    # ---- roofline of the dominant kernel (largest share of the step)
    peaks, peak_kind = load_peaks()
    v_local = v_hi - v_lo
    burst = float(peaks["bf16_tflops"])
    # Both kernels run inside a multi-millisecond step, back to back for the whole timed
    # region, where the 1 kW power cap sets the clock: the sustained figure is the ceiling.
    k_peak = float(peaks.get("bf16_tflops_sustained", burst))
    sust = k_peak
    # the library's choice of backward kernel (include/lmce.h: CTA pairs unless H < 256)
    bwd_pair = H % 64 == 0 and H >= 256 and os.environ.get("LMCE_BWD_KERNEL") != "single"
    kernels = {
        "stats": {"name": "lmce_stats_kernel (fused logits GEMM + online softmax statistics)",
                  "ms": kern_ms[0], "alg_flops": 2.0 * n_tokens * H * v_local,
                  "exec_flops": 2.0 * n_tokens * H * v_local, "traffic": FWD_STATS_TRAFFIC_C2},
        "backward": {"name": ("lmce_bwd_pair_kernel (persistent on CTA pairs" if bwd_pair else "lmce_bwd_kernel (persistent")
                             + ": recomputed logits -> G, dX and dW GEMMs)",
                     "ms": kern_ms[1], "alg_flops": 4.0 * n_lab * H * v_local,
                     "exec_flops": 6.0 * n_lab * H * v_local, "traffic": BWD_TRAFFIC_C2},
    }
    for kk in kernels.values():
        kk["achieved_tflops"] = kk["alg_flops"] / (kk["ms"] / 1e3) / 1e12
        kk["executed_tflops"] = kk["exec_flops"] / (kk["ms"] / 1e3) / 1e12
        kk["share_of_step"] = kk["ms"] / ms_per_step
    dom_key = max(kernels, key=lambda k: kernels[k]["ms"])
    dom = kernels[dom_key]
    # whole-step roofline: algorithmic flops 2*N*H*V + 4*N_lab*H*V (recompute not credited)
    step_flops = 2.0 * n_tokens * H * v_local + 4.0 * n_lab * H * v_local
    step_tflops = step_flops / (ms_per_step / 1e3) / 1e12

    if world > 1:
        dist.barrier(device_ids=[local_rank])
    err = _lib.device_error(reset=True)
    if err:
        print(f"device error word {err} on rank {rank}", file=sys.stderr)

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        tps, _ = cpu_reference_sample(args.config, args.cpu_sample_tokens, 2, 1, threads)
        cpu_base = {"value": statistics.median(tps), "unit": "tokens/s", "cores": threads, "kind": "port",
                    "sample": f"{args.cpu_sample_tokens} tokens of the workload, fwd+bwd, eager fp16 reference "
                              f"formula on the host CPU (median of 2 after 1 warm-up)"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": args.scaling if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "f16" if dt == torch.float16 else "bf16",
            "data": "synthetic",
            "config": {
                "workload": workload_name(args.config),
                "tokens_per_step": n_tokens,
                "labelled_tokens": n_lab,
                "H": H, "V": V,
                "parallelism": "single-gpu" if world == 1 else f"vocab-sharded tp{world} ({args.scaling})",
                "v_chunk": args.v_chunk,
                "dx_exchange": dx_exchange,
                "l2": "256 MiB flush written between timed steps; W (467 MB) exceeds L2 as well",
            },
            "pct_tcgen05_peak": 100.0 * step_tflops / k_peak,
            "pct_tcgen05_burst_peak": 100.0 * step_tflops / burst,
            "step_tflops": step_tflops,
            "peak_activation_mib": peak_act_mib,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": e2e_ms_step,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": loss_h.numel() * 4,
                    "api": "rus_b200.chunked_lm_head (sharded_lm_head for N>1) + loss.backward()",
                    "copies": "each step's inputs copied from pinned host memory on a copy stream "
                              "(double-buffered) while the previous step computes; one timed region "
                              "over all steps, copies, L2 flushes and loss read-backs included"},
            "gpu_launches": int(launches),
            "roofline": {
                "bound": "tensor",
                "kernel": dom["name"],
                "achieved": dom["achieved_tflops"], "peak": k_peak, "unit": "TFLOP/s",
                "frac": dom["achieved_tflops"] / k_peak,
                "peak_kind": f"{peak_kind} sustained bf16 (MEASURED_PEAKS.json); burst {burst}",
                "traffic": dom["traffic"] if (args.config == "c2" and world == 1) else None,
                "launch_ms": dom["ms"], "flops_per_launch": dom["alg_flops"],
                "executed_tflops": dom["executed_tflops"],
                "step_frac_of_sustained": step_tflops / sust,
            },
            "kernels": {k: {kk: v for kk, v in d.items() if kk != "name"} for k, d in kernels.items()},
            "clocks": clk.summary(),
            "device_error": err,
        }
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
