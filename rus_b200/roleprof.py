"""Role counters of the CTA-pair backward kernel (a diagnostic, not used by the head).

    python -m rus_b200.roleprof [--config c2] [--v-chunk N] [--steps K]

Builds ``rus_b200/liblmce_prof.so`` (the library compiled with ``-DLMCE_ROLE_PROFILE=1``,
whose kernels keep per-CTA cycle counters and a per-tile timeline; csrc/lmce_prof.cuh),
runs K forward + backward steps of a bench.py workload through it, and prints where each
role of the last backward's CTAs spent its cycles: the producer's waits for free stages and
dependencies, the UMMA issuer's waits for loaded stages and free accumulators, the
epilogue's work per tile kind, and the per-kind tile durations of the timeline; then the TMA
load rate and the stage-ring probe (``lmce_probe_tma_pipeline``). The counters perturb the
kernel slightly; use the normal build for timings.
"""
from __future__ import annotations

import argparse
import statistics
import subprocess
import sys
from pathlib import Path

import numpy as np
import torch

from . import _lib, build

PROF_LIB = Path(__file__).resolve().parent / "liblmce_prof.so"
SLOTS, NCTA, TILES = 32, 256, 1024
NAMES = {0: "total", 1: "producer: schedule ring", 2: "producer: G buffer release", 3: "producer: G complete",
         4: "producer: free stage", 6: "UMMA: next tile", 7: "UMMA: free accumulator", 8: "UMMA: stage (GT)",
         9: "UMMA: stage (DX)", 10: "UMMA: stage (DW)", 16: "epilogue: next tile", 17: "epilogue: dX chain",
         18: "epilogue: accumulator (GT)", 19: "epilogue: accumulator (DX)", 20: "epilogue: accumulator (DW)",
         21: "epilogue: work (GT)", 22: "epilogue: work (DX)", 23: "epilogue: work (DW)", 24: "epilogue: exchange"}


def build_profiling_library(force: bool = False) -> Path:
    if force or not PROF_LIB.exists() or any(d.stat().st_mtime > PROF_LIB.stat().st_mtime for d in build.DEPS):
        subprocess.run(build.compile_command(out=PROF_LIB, extra=["-DLMCE_ROLE_PROFILE=1"]), check=True)
    return PROF_LIB


def read_counters():
    ctr = np.zeros(NCTA * SLOTS, dtype=np.uint64)
    tl = np.zeros(NCTA * TILES * 8, dtype=np.uint64)
    _lib.call("lmce_profile_read", ctr.ctypes.data, ctr.nbytes, tl.ctypes.data, tl.nbytes, 1)
    return ctr.reshape(NCTA, SLOTS).astype(np.int64), tl.reshape(NCTA, TILES, 8).astype(np.int64)


def report(ctr, tl, bwd_ms):
    ncta = int((ctr[:, 0] > 0).sum())
    lead, peer = np.arange(0, ncta, 2), np.arange(1, ncta, 2)
    total = ctr[:ncta, 0].astype(float)
    ghz = total.mean() / (bwd_ms * 1e6)
    print(f"CTAs {ncta}; cycles per CTA {total.mean():.0f} (min {total.min():.0f}, max {total.max():.0f}); "
          f"backward {bwd_ms:.3f} ms, so ~{ghz:.3f} GHz")

    def pct(slot, rows):
        return 100.0 * ctr[rows, slot].astype(float).sum() / ctr[rows, 0].astype(float).sum()

    print("share of kernel cycles (pair leaders / peers):")
    for s in (1, 2, 3, 4):
        print(f"  {NAMES[s]:32s} {pct(s, lead):6.2f} / {pct(s, peer):6.2f}")
    for s in (6, 7, 8, 9, 10):
        print(f"  {NAMES[s]:32s} {pct(s, lead):6.2f}")
    for s in range(16, 25):
        print(f"  {NAMES[s]:32s} {pct(s, lead):6.2f} / {pct(s, peer):6.2f}")
    kb = {k: int(ctr[lead, s].sum()) for k, s in (("GT", 11), ("DX", 12), ("DW", 13))}
    print("  stages issued per kind:", kb)
    ntiles = ctr[:ncta, 25] + ctr[:ncta, 26] + ctr[:ncta, 27]
    dur = {0: [], 1: [], 2: []}
    for c in lead:
        prev = 0
        for e in tl[c, :int(min(ntiles[c], TILES))]:
            kind, t_m, t_f = int(e[0]), int(e[4]), int(e[6])
            if kind > 2 or t_m == 0 or t_f == 0:
                continue
            s0 = max(t_m, prev)
            dur[kind].append(t_f - s0)
            prev = t_f
    for k, name in ((0, "GT"), (1, "DX"), (2, "DW")):
        if dur[k]:
            a = np.array(dur[k]) / 1e3
            print(f"  {name} tiles {len(a)}: UMMA span per tile {a.mean():.2f} us mean, {np.median(a):.2f} median")


def _timed(dev, fn):
    """Run fn() on the current stream; (elapsed ns) from CUDA events around it."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e6


def tma_rates(dev) -> dict:
    """TMA delivery from an L2-resident 48 MB tensor for the two box shapes
    (lmce_probe_tma_rate): 2-D {64, 128} (128-byte row segments) and the kernels' 3-D
    {64, 128, 2} (256-byte row segments): (bytes per SM clock, bytes per ns per SM, SM GHz)."""
    t = torch.zeros(16384, 1536, dtype=torch.float16, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    cyc = torch.zeros(sms, dtype=torch.int64, device=dev)
    iters = 4000
    out = {}
    for kind, name in ((0, "2-D {64,128} x2"), (1, "3-D {64,128,2}")):
        ns = _timed(dev, lambda: _lib.call("lmce_probe_tma_rate", t.data_ptr(), 16384, 1536, kind, iters,
                                           cyc.data_ptr(), sms, torch.cuda.current_stream(dev).cuda_stream))
        c = cyc.double().mean().item()
        out[name] = ((iters - 9) * 32768 / c, iters * 32768 / ns, c / ns * iters / (iters - 9))
    return out


# (load kind, stage bytes, stages, hold cycles): the kernels' ring (three 64 KB stages of 3-D
# boxes, held 1024 cycles as a 256 x 256 pair UMMA with K = 128 holds them; 1536 cycles at the
# probe's full clock last as long as 1024 at the ~1.3 GHz the kernels run at under the power
# cap) and its neighbours
PIPELINES = ((1, 65536, 3, 0), (1, 65536, 3, 1024), (1, 65536, 3, 1536), (0, 65536, 3, 1024), (2, 65536, 3, 0),
             (2, 65536, 3, 1024),
             (1, 32768, 6, 512), (0, 32768, 6, 512), (2, 32768, 6, 512), (0, 49152, 4, 1024))
KIND_NAMES = {0: "2-D {64,128} boxes", 1: "3-D {64,128,2} boxes", 2: "bulk 32 KB copies"}


def pipeline_table(dev) -> list:
    """lmce_probe_tma_pipeline over PIPELINES, from an L2-resident 48 MB tensor and from a
    768 MB one (DRAM): (source, kind, stage KB, stages, hold, bytes/clk/SM, holder busy %,
    bytes/ns/SM, SM GHz). Bytes per SM clock depend on the SM clock (the memory system keeps
    its own), so the clock of each run is reported with it."""
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    cyc = torch.zeros(sms, dtype=torch.int64, device=dev)
    iters = 3000
    rows_out = []
    for src, rows in (("L2", 16384), ("DRAM", 262144)):
        t = torch.zeros(rows, 1536, dtype=torch.float16, device=dev)
        for kind, sb, st, hold in PIPELINES:
            ns = _timed(dev, lambda: _lib.call("lmce_probe_tma_pipeline", t.data_ptr(), rows, 1536, kind, sb, st,
                                               hold, iters, cyc.data_ptr(), sms,
                                               torch.cuda.current_stream(dev).cuda_stream))
            c = cyc.double().mean().item()
            rows_out.append((src, KIND_NAMES[kind], sb // 1024, st, hold, (iters - 9) * sb / c,
                             100.0 * (iters - 9) * hold / c, iters * sb / ns, c / ns * iters / (iters - 9)))
        del t
    return rows_out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2")
    ap.add_argument("--v-chunk", type=int, default=0)
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args(argv)
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    import bench

    _lib.LIB_PATH = build_profiling_library()
    from .ops import chunked_lm_head

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    X, y, W, _ = bench.make_config(args.config, dev)
    W = W.clone().requires_grad_(True)
    Xg = X.clone().requires_grad_(True)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)

    def step():
        Xg.grad = None
        W.grad = None
        loss, *_ = chunked_lm_head(Xg, y, W, None, args.v_chunk or None)
        loss.backward()

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    read_counters()  # clear
    ev = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        b.record()
        ev.append((a, b))
    for a, b in ev:
        flush.zero_()
        _lib.call("lmce_set_timing_events", 1, a.cuda_event, b.cuda_event)
        step()
    torch.cuda.synchronize()
    _lib.call("lmce_set_timing_events", 1, None, None)
    ctr, tl = read_counters()  # the last step's backward
    ms = [a.elapsed_time(b) for a, b in ev]
    print(f"{args.config}, v_chunk {args.v_chunk or 'default'}: backward median {statistics.median(ms):.3f} ms "
          f"over {args.steps} steps")
    report(ctr, tl, ms[-1])
    for name, (rate, per_ns, ghz) in tma_rates(dev).items():
        print(f"TMA load rate, {name} boxes: {rate:.1f} bytes/clk/SM = {per_ns:.1f} bytes/ns/SM at {ghz:.2f} GHz "
              f"(a 256 x 256 pair UMMA consumes 64 bytes/clk/SM)")
    print("TMA pipeline (ring of stages, each held `hold` cycles after it lands):")
    for src, kind, kb, st, hold, rate, busy, per_ns, ghz in pipeline_table(dev):
        print(f"  {src:4s} {kind:22s} {st} x {kb:2d} KB hold {hold:4d}: {rate:5.1f} bytes/clk/SM = "
              f"{per_ns:5.1f} bytes/ns/SM at {ghz:.2f} GHz, holder busy {busy:5.1f}%")


if __name__ == "__main__":
    main()
