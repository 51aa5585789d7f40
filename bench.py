"""Benchmark of the fused lm_head cross-entropy head (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1..c5]
                    [--scaling weak|strong]
    (N > 1: launched by torchrun, one process per GPU)

Metric: "lm_head CE fwd+bwd tokens/s (Qwen2.5-1.5B head), % tcgen05 peak, peak MiB".
Workload at N=1 (default): config 2 — Qwen2.5-1.5B tied head H=1536, V=151936, fp16, 4 rows x 512
tokens all packed (N=2048), labels uniform with 10% = -100, W ~ N(0, 0.02). The other configs of
BASELINE.json are selectable (--config): c1 packed SFT batch (~880 tokens, the reference's real
call shape), c3 Qwen2.5-7B head (~11.6k tokens, H=3584), c4 Llama-3-8B head (32768 tokens,
H=4096, bf16), c5 Qwen2.5-0.5B numerics stress (~2.8k tokens, logit std ~12, exact top-2 ties).
All inputs are seeded synthetic data with the configs' shapes and distributions (the reference's
dataset is not available offline), generated on the device. One step = loss forward + backward
(dX and dW) through the public autograd API.

N > 1: the head is vocab-sharded over the N GPUs. Weak scaling (default) multiplies the global batch
by N (every GPU does the work of one single-GPU step); strong scaling (--scaling strong) keeps the
config's tokens and splits only the vocabulary. The per-token statistics are all-gathered over NCCL
and dX is summed inside the backward kernel over NVLink SHARP (fp32 dX of 32 MiB or more) or by an
NCCL all-reduce.

``value`` is device-timed with the inputs resident (L2 flushed between steps); ``e2e`` runs the same
steps from pinned host memory, each step's inputs copied on a copy stream while the previous step
computes, all copies, L2 flushes and loss read-backs inside one timed region.

``roofline`` divides by the measured burst bf16 peak unless the timed region's own clock record
shows the power cap holding the SM clock down (then the sustained figure).

``--impl reference`` times the reference's eager formula (full-logit F.linear in the input dtype +
fp32 cross entropy + entropy + argmax + autograd dX/dW; the oracle restatement of
solution/test_kernels.py:204-216) on the host CPU with all threads, on the same config's full step
when that fits a few minutes of CPU time, else on a stated token sample; under torchrun only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "lm_head CE fwd+bwd tokens/s (Qwen2.5-1.5B head), % tcgen05 peak, peak MiB"
# name: H, V, dtype, workload description
CONFIGS = {
    "c1": (1536, 151936, torch.float16,
           "C1 Qwen2.5-1.5B tied head fwd+bwd, H=1536 V=151936 fp16, 4 packed rows, lognormal lengths "
           "(median 140) clipped to [16,512], first 40% of each row -100"),
    "c2": (1536, 151936, torch.float16,
           "C2 Qwen2.5-1.5B tied head fwd+bwd, H=1536 V=151936 fp16, 4x512 tokens (N=2048), 10% labels -100"),
    "c3": (3584, 152064, torch.float16,
           "C3 Qwen2.5-7B head fwd+bwd, H=3584 V=152064 fp16, 16 packed rows, lognormal lengths (median 600) "
           "clipped to [32,2048], 10% labels -100"),
    "c4": (4096, 128256, torch.bfloat16,
           "C4 Llama-3-8B head fwd+bwd, H=4096 V=128256 bf16, 8x4096 tokens (N=32768), labels uniform"),
    "c5": (896, 151936, torch.float16,
           "C5 Qwen2.5-0.5B tied head fwd+bwd (numerics stress), H=896 V=151936 fp16, 64 rows of Zipf(1.2) "
           "lengths in [1,512], 3 rows all -100, logit std ~12, 1% exact top-2 ties"),
}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) of one forward-statistics launch and of one backward launch at
# config 2 with the default chunk, from one `ncu --set full` capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of this script's second warm-up step.
FWD_STATS_TRAFFIC_C2 = 504_412_000 + 5_608_000
BWD_TRAFFIC_C2 = 1_822_938_000 + 1_257_441_000
CPU_BUDGET_S = 150.0  # CPU seconds the reference arm may spend (warm-up + timed steps)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


# ------------------------------------------------------------------ inputs

def row_lengths(cfg: str, seed: int = 0) -> np.ndarray:
    """Packed row lengths of a config (seeded): the config descriptions' distributions."""
    rng = np.random.default_rng(seed)
    if cfg == "c1":
        return np.clip(np.round(rng.lognormal(math.log(140), 0.951, 4)), 16, 512).astype(np.int64)
    if cfg == "c2":
        return np.full(4, 512, dtype=np.int64)
    if cfg == "c3":
        return np.clip(np.round(rng.lognormal(math.log(600), 0.67, 16)), 32, 2048).astype(np.int64)
    if cfg == "c4":
        return np.full(8, 4096, dtype=np.int64)
    # c5: Zipf(1.2) truncated to 1..512, i.e. P(k) ~ k^-1.2 renormalised on that support (E[N] ~ 2.8k)
    k = np.arange(1, 513)
    pmf = k ** -1.2
    return rng.choice(k, size=64, p=pmf / pmf.sum()).astype(np.int64)


def make_config(cfg: str, device, replicas: int = 1, seed: int = 0):
    """(X [N, H], labels [N] int64, W [V, H], lengths) of a config, built on `device` from seeded
    generators, so every process (and every GPU of one type) builds the same tensors. ``replicas``
    > 1 stacks that many independently seeded batches (weak scaling's global batch)."""
    H, V, dt, _ = CONFIGS[cfg]
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    w_std = 12.0 / math.sqrt(H) if cfg == "c5" else 0.02
    W = (torch.randn(V, H, generator=g, device=dev) * w_std).to(dt)
    gamma = 1.0 + 0.1 * torch.randn(H, generator=g, device=dev)  # RMSNorm weight ~ N(1, 0.1)
    xs, ys, lens_all = [], [], []
    for r in range(replicas):
        lens = row_lengths(cfg, seed + r)
        n = int(lens.sum())
        X = torch.randn(n, H, generator=g, device=dev)
        if cfg != "c4":
            X = X * gamma
        y = torch.randint(0, V, (n,), generator=g, device=dev)
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        if cfg == "c1":
            for s0, L in zip(starts, lens):
                y[int(s0):int(s0) + int(0.4 * L)] = -100
        elif cfg in ("c2", "c3"):
            y[torch.rand(n, generator=g, device=dev) < 0.10] = -100
        elif cfg == "c5":
            rng = np.random.default_rng(1000 + seed + r)
            for row in rng.choice(len(lens), 3, replace=False):
                y[int(starts[row]):int(starts[row] + lens[row])] = -100
            # exact argmax ties on ~1% of tokens: a duplicated W row pair with x aligned to it
            for t in rng.choice(n, max(1, n // 100), replace=False):
                a, b = (int(v) for v in rng.choice(V, 2, replace=False))
                W[b] = W[a]
                X[int(t)] = W[a].float() * (40.0 / W[a].float().norm())
        xs.append(X.to(dt))
        ys.append(y)
        lens_all.extend(int(v) for v in lens)
    return torch.cat(xs), torch.cat(ys), W, lens_all


# ------------------------------------------------------------------ clocks

# NVML sampling loop run in a child process (no GIL shared with the ranks' host work): argv[1]
# lists the GPUs as domain:bus:device, argv[2] the period in seconds. It prints one JSON line
# when ready, starts sampling when a line arrives on its stdin and, once its stdin closes,
# prints one JSON line of samples per GPU.
_SAMPLER_SRC = r"""
import json, select, sys
import pynvml
pynvml.nvmlInit()
want = [tuple(int(v) for v in w.split(":")) for w in sys.argv[1].split(",")]
period = float(sys.argv[2])
found = {}
for i in range(pynvml.nvmlDeviceGetCount()):
    h = pynvml.nvmlDeviceGetHandleByIndex(i)
    pci = pynvml.nvmlDeviceGetPciInfo(h)
    found[(int(pci.domain), int(pci.bus), int(pci.device))] = h
handles = [found[w] for w in want]
mx = [float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)) for h in handles]
print(json.dumps({"max_mhz": mx}), flush=True)
sys.stdin.readline()
samples = [[] for _ in handles]
while not select.select([sys.stdin], [], [], period)[0]:
    for k, h in enumerate(handles):
        try:
            samples[k].append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                               int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))))
        except Exception:
            pass
print(json.dumps({"samples": samples}), flush=True)
"""


def pci_ids(devices) -> list:
    """domain:bus:device of each CUDA device (how the sampler finds its NVML handle)."""
    out = []
    for dev in devices:
        props = torch.cuda.get_device_properties(dev)
        out.append(f"{int(props.pci_domain_id)}:{int(props.pci_bus_id)}:{int(props.pci_device_id)}")
    return out


class ClockSampler:
    """SM clock and clock-event reasons of one or more GPUs, sampled (NVML) every ~2 ms by a
    child process between start() and stop(). The child is set up (NVML initialised, handles
    found: tens to hundreds of ms) when the sampler is entered, which must come before the
    ranks' last barrier ahead of the timed region: a rank that did that set-up inside the
    timed region would start its steps late, and under torchrun the other ranks would wait
    for it at the first collective, inflating their step times. Under torchrun rank 0 samples
    every rank's GPU and the other ranks sample none."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, devices, period_s: float = 0.002):
        self.devices = list(devices)
        self.period = period_s
        self.samples = [[] for _ in self.devices]
        self.max_mhz = [None for _ in self.devices]
        self._proc = None

    def __enter__(self):
        import subprocess

        if not self.devices:
            return self
        try:
            pci = pci_ids(self.devices)
            self._proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, ",".join(pci), str(self.period)],
                                          stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                          stderr=subprocess.DEVNULL, text=True)
            ready = json.loads(self._proc.stdout.readline())
            self.max_mhz = ready["max_mhz"]
        except Exception:
            self._stop_proc()
        return self

    def start(self):
        """Begin sampling (call at the start of the timed region)."""
        if self._proc is not None:
            try:
                self._proc.stdin.write("go\n")
                self._proc.stdin.flush()
            except Exception:
                self._stop_proc()

    def _stop_proc(self):
        if self._proc is None:
            return None
        out = None
        try:
            out, _ = self._proc.communicate(input="", timeout=10)
        except Exception:
            self._proc.kill()
            self._proc.wait()
        self._proc = None
        return out

    def stop(self):
        """End sampling and collect the samples (call at the end of the timed region)."""
        out = self._stop_proc()
        if out:
            try:
                got = json.loads(out.strip().splitlines()[-1])["samples"]
                self.samples = [[(float(m), int(r)) for m, r in g] for g in got]
            except Exception:
                pass

    def __exit__(self, *exc):
        self.stop()
        return False

    def summary(self, k: int = 0):
        samples = self.samples[k] if k < len(self.samples) else []
        mx = self.max_mhz[k] if k < len(self.max_mhz) else None
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unavailable"], "samples": 0}
        reasons = set()
        capped = 0
        for _, r in samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
            capped += 1 if r & 0x4 else 0
        return {"sm_mhz": statistics.median(m for m, _ in samples), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(samples),
                "power_capped_fraction": capped / len(samples), "source": "nvml, ~2 ms, child process"}


def choose_peak(peaks: dict, clk: dict):
    """Roofline denominator: the burst bf16 figure, unless the timed region ran power-capped
    (sw_power_cap in at least half the samples and median SM clock under 90% of max), then the
    sustained figure measured under the cap. Returns (peak, kind string)."""
    burst = float(peaks["bf16_tflops"])
    sust = float(peaks.get("bf16_tflops_sustained", burst))
    mhz, mx = clk.get("sm_mhz"), clk.get("sm_max_mhz")
    capped = (mhz is not None and mx and clk.get("power_capped_fraction", 0.0) >= 0.5 and mhz < 0.9 * mx)
    if capped:
        return sust, f"sustained bf16 {sust} (timed region power-capped: median SM {mhz:.0f} of {mx:.0f} MHz)"
    where = f"median SM {mhz:.0f} of {mx:.0f} MHz" if mhz is not None and mx else "no clock record"
    return burst, f"burst bf16 {burst} (timed region not held by the power cap: {where})"


# ------------------------------------------------------------------ CPU side

def cpu_reference(cfg: str, iters: int, warmup: int, threads: int, budget_s: float = CPU_BUDGET_S, inputs=None):
    """The reference eager formula on the host CPU over the config's step, or over its first
    tokens when `warmup + iters` whole steps would not fit `budget_s` (the per-token cost is
    calibrated on a 128-token run first). `inputs` = (X, labels, W) host tensors to use instead
    of building the config on the host (the GPU arm passes its own, so that the outputs can be
    compared). Returns (tokens/s per timed iteration, seconds per iteration, tokens timed per
    iteration, tokens of the whole step, the last iteration's outputs)."""
    from oracle import lmce_oracle as orc

    torch.set_num_threads(threads)
    if inputs is None:
        X, y, W, _ = make_config(cfg, "cpu")
    else:
        X, y, W = inputs
    n_full = int(y.numel())
    t0 = time.perf_counter()
    orc.eager_head(X[:128], y[:128], W, grads=True, grad_mode="eager")
    per_tok = (time.perf_counter() - t0) / min(128, n_full)
    fit = int(budget_s / (per_tok * (iters + warmup)))
    tokens = n_full if fit >= n_full else max(64, fit // 64 * 64)
    X, y = X[:tokens].contiguous(), y[:tokens].contiguous()
    times = []
    out = None
    for i in range(warmup + iters):
        t0 = time.perf_counter()
        out = orc.eager_head(X, y, W, grads=True, grad_mode="eager")
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return [tokens / t for t in times], times, tokens, n_full, out


def output_check(loss, nll, ent, arg, ref) -> dict:
    """The GPU head's forward outputs against the eager reference formula's on the same inputs
    (the host CPU's GEMM): `ok` = loss within 1e-3 relative and every token's nll within
    1e-3 * max(|nll|, 1), the parity tests' bars. Entropy and argmax are reported, not gated: where
    the two GEMMs round a row's top logits one fp16 ulp apart (config 5 plants exact top-2 ties
    at logits near 40, where an ulp is 0.03), that row's entropy moves by up to ln 2 and its
    argmax may flip; the GPU parity tests classify those rows against fp32 logits."""
    nll, ent, arg = nll.detach().float().cpu(), ent.detach().float().cpu(), arg.detach().cpu()
    rl, rn, re_, ra = float(ref["loss"]), ref["nll"].float(), ref["entropy"].float(), ref["argmax"]
    loss_rel = abs(float(loss) - rl) / max(abs(rl), 1e-30)
    nll_excess = float(((nll - rn).abs() / rn.abs().clamp(min=1.0)).max())
    ent_excess = float(((ent - re_).abs() / re_.abs().clamp(min=1.0)).max())
    agree = float((arg == ra).float().mean())
    return {"loss": float(loss), "loss_oracle": rl, "loss_rel_diff": loss_rel, "nll_max_rel_diff": nll_excess,
            "entropy_max_rel_diff": ent_excess, "argmax_agreement": agree,
            "ok": loss_rel <= 1e-3 and nll_excess <= 1e-3}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps, warm = max(args.steps, 1), max(args.warmup, 1)
    tps, times, tokens, n_full, _ = cpu_reference(args.config, steps, warm, threads)
    value = statistics.median(tps)
    H, V, dt, _ = CONFIGS[args.config]
    sample = ("the whole step" if tokens == n_full else f"the first {tokens} of the step's {n_full} tokens")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": statistics.median(times) * 1e3,
        "higher_is_better": True, "scaling": args.scaling if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f16" if dt == torch.float16 else "bf16", "data": "synthetic",
        "config": {"workload": CONFIGS[args.config][3], "tokens_per_step": n_full, "tokens_timed_per_step": tokens,
                   "H": H, "V": V, "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} of {args.config} per step (fwd+bwd, eager F.linear in the input dtype + "
                                   f"fp32 CE + entropy + argmax + autograd dX/dW), median of {steps} after {warm} "
                                   f"warm-up"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    H, V, dt, workload = CONFIGS[args.config]
    replicas = world if (world > 1 and args.scaling == "weak") else 1
    X, y, W_full, _ = make_config(args.config, device, replicas=replicas)
    n_tokens = int(y.numel())
    v_lo, v_hi = shard_range(V, rank, world) if world > 1 else (0, V)
    W = W_full[v_lo:v_hi].clone().requires_grad_(True)
    del W_full
    Xg = X.clone().requires_grad_(True)
    n_lab = int((y != -100).sum())
    torch.cuda.synchronize()

    def head(xx, yy):
        if world > 1:
            return sharded_lm_head(xx, yy, W, v_lo, V, group, None, args.v_chunk)
        return chunked_lm_head(xx, yy, W, None, args.v_chunk)

    host_s = [0.0, 0.0]  # host time spent issuing the forward / the backward of the timed steps

    def step(mid=None):
        Xg.grad = None
        W.grad = None
        h0 = time.perf_counter()
        loss, nll, ent, arg = head(Xg, y)
        if mid is not None:
            mid.record(stream)  # between the forward and the backward phase
        h1 = time.perf_counter()
        loss.backward()
        if mid is not None:
            host_s[0] += h1 - h0
            host_s[1] += time.perf_counter() - h1
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

    # ---- timed region. The device-timed steps (inputs resident in HBM; L2 flushed between
    # steps; the library records events around its two tensor-core kernels on the launching
    # stream, lmce_set_timing_events) run in two halves with the end-to-end block between
    # them, so both measurements see the same clock and power state under one clock record.
    stage("timed steps")
    l0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    ev_mid = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kev = {k: [(new_event(), new_event()) for _ in range(args.steps)] for k in (0, 1)}
    e2e_a = torch.cuda.Event(enable_timing=True)
    e2e_b = torch.cuda.Event(enable_timing=True)

    def value_steps(i0, i1):
        for i in range(i0, i1):
            flush.zero_()
            for k in (0, 1):
                _lib.call("lmce_set_timing_events", k, kev[k][i][0].cuda_event, kev[k][i][1].cuda_event)
            ev[i][0].record(stream)
            step(ev_mid[i])
            ev[i][1].record(stream)
        for k in (0, 1):
            _lib.call("lmce_set_timing_events", k, None, None)

    half = args.steps // 2
    # one sampling process per job: rank 0 samples every rank's GPU (one process per GPU of one
    # node, rank r on cuda:r), the other ranks none; it is set up before the last barrier, so
    # every rank enters the timed region together
    sampled = [device] if world == 1 else ([torch.device("cuda", r) for r in range(world)] if rank == 0 else [])
    with ClockSampler(sampled) as clk:
        torch.cuda.synchronize()
        barrier()
        clk.start()
        value_steps(0, half)
        barrier()
        launches = _lib.launch_count() - l0
        stage("end-to-end")
        e2e_a.record(stream)
        copy_stream.wait_stream(stream)
        run_e2e(e2e_steps)
        e2e_b.record(stream)
        barrier()
        l1 = _lib.launch_count()
        stage("timed steps (second half)")
        value_steps(half, args.steps)
        barrier()
        clk.stop()
        launches += _lib.launch_count() - l1
    step_ms = [a.elapsed_time(b) for a, b in ev]
    kern_ms = {k: statistics.mean(a.elapsed_time(b) for a, b in kev[k]) for k in (0, 1)}
    # forward phase (statistics kernel, record merge / exchange, finish, loss) and backward phase
    fwd_phase_ms = statistics.mean(a.elapsed_time(m) for (a, _), m in zip(ev, ev_mid))
    bwd_phase_ms = statistics.mean(m.elapsed_time(b) for (_, b), m in zip(ev, ev_mid))
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=device)
    e2e_ms = torch.tensor([e2e_a.elapsed_time(e2e_b)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    ms_per_step = total_ms.item() / args.steps
    value = n_tokens / (ms_per_step / 1e3)
    e2e_ms_step = e2e_ms.item() / e2e_steps
    e2e_value = n_tokens / (e2e_ms_step / 1e3)
    h2d = Xh.numel() * Xh.element_size() + yh.numel() * yh.element_size()

    stage("report")
    dx_exchange = "none (single GPU)"
    if world > 1:
        from rus_b200.sharded import nvls_dx_exchange
        dx_exchange = ("in-kernel NVLink SHARP exchange (multimem.ld_reduce + multimem.st)"
                       if nvls_dx_exchange(n_tokens, H, dt, device, group) is not None else "NCCL all-reduce (fp32)")
    # ---- roofline of the dominant kernel (largest share of the step)
    peaks, peak_src = load_peaks()
    clocks = clk.summary()
    if world > 1 and rank == 0:
        clocks["per_gpu"] = [{k: clk.summary(r).get(k) for k in ("sm_mhz", "reasons", "power_capped_fraction")}
                             for r in range(world)]
    k_peak, peak_kind = choose_peak(peaks, clocks)
    burst = float(peaks["bf16_tflops"])
    sust = float(peaks.get("bf16_tflops_sustained", burst))
    v_local = v_hi - v_lo
    # the library's choice of backward kernel (include/lmce.h: CTA pairs unless H < 256)
    bwd_pair = H % 64 == 0 and H >= 256 and os.environ.get("LMCE_BWD_KERNEL") != "single"
    c2_default = args.config == "c2" and world == 1 and args.v_chunk == 0
    kernels = {
        "stats": {"name": "lmce_stats_kernel (fused logits GEMM + online softmax statistics)",
                  "ms": kern_ms[0], "alg_flops": 2.0 * n_tokens * H * v_local,
                  "exec_flops": 2.0 * n_tokens * H * v_local,
                  "traffic": FWD_STATS_TRAFFIC_C2 if c2_default else None},
        "backward": {"name": ("lmce_bwd_pair_kernel (persistent on CTA pairs" if bwd_pair else "lmce_bwd_kernel (persistent")
                             + ": recomputed logits -> G, dX and dW GEMMs)",
                     "ms": kern_ms[1], "alg_flops": 4.0 * n_lab * H * v_local,
                     "exec_flops": 6.0 * n_lab * H * v_local,
                     "traffic": BWD_TRAFFIC_C2 if c2_default else None},
    }
    for kk in kernels.values():
        kk["achieved_tflops"] = kk["alg_flops"] / (kk["ms"] / 1e3) / 1e12
        kk["executed_tflops"] = kk["exec_flops"] / (kk["ms"] / 1e3) / 1e12
        kk["frac_of_burst"] = kk["achieved_tflops"] / burst
        kk["share_of_step"] = kk["ms"] / ms_per_step
    dom = kernels[max(kernels, key=lambda k: kernels[k]["ms"])]
    # whole-step roofline: algorithmic flops 2*N*H*V + 4*N_lab*H*V (recompute not credited)
    step_flops = 2.0 * n_tokens * H * v_local + 4.0 * n_lab * H * v_local
    step_tflops = step_flops / (ms_per_step / 1e3) / 1e12

    # per-rank view (N > 1): every rank's mean step, kernel and phase times and its median SM
    # clock, so that rank-to-rank speed differences (which the max over ranks absorbs) show
    per_rank = None
    if world > 1:
        mine = torch.tensor([statistics.mean(step_ms), kern_ms[0], kern_ms[1], fwd_phase_ms, bwd_phase_ms,
                             1e3 * host_s[0] / args.steps, 1e3 * host_s[1] / args.steps],
                            dtype=torch.float64, device=device)
        allr = torch.empty((world, mine.numel()), dtype=torch.float64, device=device)
        dist.all_gather_into_tensor(allr, mine)
        cols = allr.t().tolist()
        per_rank = {k: [round(v, 4) for v in c] for k, c in
                    zip(("step_ms", "stats_ms", "backward_ms", "forward_phase_ms", "backward_phase_ms",
                         "host_forward_ms", "host_backward_ms"), cols)}
        if rank == 0:
            per_rank["sm_mhz"] = [clk.summary(r).get("sm_mhz") for r in range(world)]
        dist.barrier(device_ids=[local_rank])
    err = _lib.device_error(reset=True)
    if err:
        print(f"device error word {err} on rank {rank}", file=sys.stderr)

    cpu_base = None
    output_ok = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        iters = 3
        # the same inputs the GPU arm timed (copied to the host), so that the outputs compare
        tps, _, tokens, n_full, ref = cpu_reference(args.config, iters, 1, threads, budget_s=60.0,
                                                    inputs=(Xh, yh, W.detach().cpu()))
        sample = "the whole step" if tokens == n_full else f"the first {tokens} of the step's {n_full} tokens"
        cpu_base = {"value": statistics.median(tps), "unit": "tokens/s", "cores": threads, "kind": "port",
                    "sample": f"{sample}, fwd+bwd, eager reference formula on the host CPU "
                              f"(median of {iters} after 1 warm-up)"}
        if tokens == n_full:
            # one more forward through the head on the timed inputs (after the timed region)
            with torch.no_grad():
                outs = head(Xg.detach(), y)
            output_ok = output_check(*outs, ref)
            if not output_ok["ok"]:
                print(f"output check failed: {output_ok}", file=sys.stderr)

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
                "workload": workload,
                "tokens_per_step": n_tokens,
                "labelled_tokens": n_lab,
                "H": H, "V": V,
                "parallelism": "single-gpu" if world == 1 else f"vocab-sharded tp{world} ({args.scaling})",
                "v_chunk": args.v_chunk,
                "dx_exchange": dx_exchange,
                "l2": "256 MiB flush written between timed steps",
            },
            "pct_tcgen05_peak": 100.0 * step_tflops / k_peak,
            "pct_tcgen05_burst_peak": 100.0 * step_tflops / burst,
            "pct_tcgen05_sustained_peak": 100.0 * step_tflops / sust,
            "step_tflops": step_tflops,
            "peak_activation_mib": peak_act_mib,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": e2e_ms_step,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": loss_h.numel() * 4,
                    "api": "rus_b200.chunked_lm_head (sharded_lm_head for N>1) + loss.backward()",
                    "copies": "each step's inputs copied from pinned host memory on a copy stream "
                              "(double-buffered) while the previous step computes; one timed region "
                              "over all steps, copies, L2 flushes and loss read-backs included; run between "
                              "the two halves of the device-timed steps"},
            "gpu_launches": int(launches),
            "roofline": {
                "bound": "tensor",
                "kernel": dom["name"],
                "achieved": dom["achieved_tflops"], "peak": k_peak, "unit": "TFLOP/s",
                "frac": dom["achieved_tflops"] / k_peak,
                "peak_kind": f"{peak_src} {peak_kind}",
                "traffic": dom["traffic"],
                "launch_ms": dom["ms"], "flops_per_launch": dom["alg_flops"],
                "executed_tflops": dom["executed_tflops"],
                "step_frac": step_tflops / k_peak,
            },
            "kernels": {k: {kk: v for kk, v in d.items() if kk != "name"} for k, d in kernels.items()},
            "host_issue_ms": {"forward": 1e3 * host_s[0] / args.steps, "backward": 1e3 * host_s[1] / args.steps},
            "phases_ms": {"forward": fwd_phase_ms, "backward": bwd_phase_ms,
                          "forward_outside_stats_kernel": fwd_phase_ms - kern_ms[0],
                          "backward_outside_backward_kernel": bwd_phase_ms - kern_ms[1]},
            "clocks": clocks,
            "device_error": err,
        }
        if per_rank is not None:
            line["per_rank"] = per_rank
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        if output_ok is not None:
            line["output_check"] = output_ok
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
