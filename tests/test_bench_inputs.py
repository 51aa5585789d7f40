"""CPU: the benchmark's seeded config generators (bench.make_config) follow the configs of
shapes, dtypes, row-length laws, label masks and the planted argmax ties."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench


@pytest.mark.parametrize("cfg", ["c1", "c2", "c5"])
def test_config_shapes_and_masks(cfg):
    H, V, dt, _ = bench.CONFIGS[cfg]
    X, y, W, lens = bench.make_config(cfg, "cpu")
    n = sum(lens)
    assert X.shape == (n, H) and X.dtype == dt and W.shape == (V, H) and W.dtype == dt and y.shape == (n,)
    assert int(y[y != -100].min()) >= 0 and int(y.max()) < V
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    if cfg == "c1":
        assert len(lens) == 4 and all(16 <= L <= 512 for L in lens)
        for s0, L in zip(starts, lens):  # first 40% of each row ignored, the rest labelled
            k = int(0.4 * L)
            assert (y[s0:s0 + k] == -100).all() and (y[s0 + k:s0 + L] != -100).all()
    elif cfg == "c2":
        assert lens == [512] * 4
        frac = float((y == -100).float().mean())
        assert 0.07 < frac < 0.13
    else:  # c5: Zipf(1.2) lengths truncated to 1..512, three rows all ignored, planted ties
        assert len(lens) == 64 and all(1 <= L <= 512 for L in lens) and 1500 <= n <= 4500
        full = sum(bool((y[s0:s0 + L] == -100).all()) for s0, L in zip(starts, lens))
        assert full >= 3
        assert len(torch.unique(W, dim=0)) < V


def test_weak_scaling_replicas_stack_independent_batches():
    X1, y1, W1, l1 = bench.make_config("c2", "cpu", replicas=1)
    X2, y2, W2, l2 = bench.make_config("c2", "cpu", replicas=2)
    assert X2.shape[0] == 2 * X1.shape[0] and torch.equal(W1, W2)
    assert torch.equal(X2[: X1.shape[0]], X1) and not torch.equal(X2[X1.shape[0]:], X1)


def test_peak_choice_follows_the_clock_record():
    peaks = {"bf16_tflops": 1635.7, "bf16_tflops_sustained": 1396.7}
    burst = bench.choose_peak(peaks, {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "power_capped_fraction": 0.0})
    capped = bench.choose_peak(peaks, {"sm_mhz": 1350.0, "sm_max_mhz": 1965.0, "power_capped_fraction": 0.9})
    assert burst[0] == 1635.7 and "burst" in burst[1]
    assert capped[0] == 1396.7 and "sustained" in capped[1]


def test_clock_sampler_child_process(tmp_path, monkeypatch):
    """The clock sampler runs NVML in a child process (no interpreter lock shared with the
    thread that issues the GPU work) and returns per-GPU samples with their clock-event
    reasons; checked here against a stand-in NVML module on the host."""
    (tmp_path / "pynvml.py").write_text(
        "NVML_CLOCK_SM = 1\n"
        "class _P:\n"
        "    def __init__(self, i): self.domain, self.bus, self.device = 0, 10 + i, 0\n"
        "def nvmlInit(): pass\n"
        "def nvmlDeviceGetCount(): return 2\n"
        "def nvmlDeviceGetHandleByIndex(i): return i\n"
        "def nvmlDeviceGetPciInfo(h): return _P(h)\n"
        "def nvmlDeviceGetMaxClockInfo(h, c): return 1965\n"
        "def nvmlDeviceGetClockInfo(h, c): return 1800 + 100 * h\n"
        "def nvmlDeviceGetCurrentClocksEventReasons(h): return 4 * h\n")
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    monkeypatch.setattr(bench, "pci_ids", lambda devs: ["0:11:0", "0:10:0"][:len(devs)])
    import time

    with bench.ClockSampler([0, 1]) as clk:
        time.sleep(0.05)
        assert clk.summary(0)["samples"] == 0  # set up, not sampling before start()
        clk.start()
        time.sleep(0.05)
        clk.stop()
    a, b = clk.summary(0), clk.summary(1)
    assert a["samples"] > 3 and b["samples"] > 3
    assert a["sm_mhz"] == 1900.0 and a["reasons"] == ["sw_power_cap"] and a["power_capped_fraction"] == 1.0
    assert b["sm_mhz"] == 1800.0 and b["reasons"] == [] and b["sm_max_mhz"] == 1965.0
    assert bench.ClockSampler([]).summary()["samples"] == 0


def test_output_check_gates_loss_and_nll():
    """The bench compares its head's outputs on the timed inputs with the eager reference formula
    (host CPU): loss and per-token nll gate `ok` at the parity tests' 1e-3; entropy and argmax
    are reported only."""
    from oracle import lmce_oracle as orc

    g = torch.Generator().manual_seed(0)
    X = torch.randn(64, 128, generator=g).half()
    W = (torch.randn(500, 128, generator=g) * 0.02).half()
    y = torch.randint(0, 500, (64,), generator=g)
    y[:5] = -100
    ref = orc.eager_head(X, y, W, grads=False)
    same = bench.output_check(ref["loss"], ref["nll"], ref["entropy"], ref["argmax"], ref)
    assert same["ok"] and same["loss_rel_diff"] == 0.0 and same["argmax_agreement"] == 1.0
    assert not bench.output_check(ref["loss"] * 1.01, ref["nll"], ref["entropy"], ref["argmax"], ref)["ok"]
    nll = ref["nll"].clone()
    nll[7] += 0.01 * max(float(nll[7]), 1.0)
    assert not bench.output_check(ref["loss"], nll, ref["entropy"], ref["argmax"], ref)["ok"]
    ent = ref["entropy"] + 0.5  # reported, not gated
    out = bench.output_check(ref["loss"], ref["nll"], ent, ref["argmax"], ref)
    assert out["ok"] and out["entropy_max_rel_diff"] > 0.05
