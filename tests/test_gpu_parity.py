"""Parity of the sm_100a head (rus_b200.chunked_lm_head -> liblmce.so) against the oracle.

Tolerances:
  loss, lse, nll      1e-3 relative per token (absolute floor 1e-3 for values near 0)
  entropy             |d| <= 1e-3 * max(|ref|, 1)
  dX, dW              1e-2 relative L2
  argmax              bit-exact except where the two candidates' logits lie within
                      max(1e-3, one ulp of the input dtype) (oracle.argmax_mismatch_ok)
The reference's own known-answer test (solution/test_kernels.py:189-226) is also
run with its own tolerances (loss 2e-3, dX 5e-3, entropy 2e-3, argmax exact).
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import lmce_oracle as orc

pytestmark = pytest.mark.gpu


def _run_ours(hidden, labels, weight, num_items=None, v_chunk=None, want_dw=True):
    from rus_b200 import chunked_lm_head

    h = hidden.detach().clone().requires_grad_(True)
    w = weight.detach().clone().requires_grad_(want_dw)
    loss, nll, ent, arg = chunked_lm_head(h, labels, w, num_items, v_chunk)
    loss.backward()
    torch.cuda.synchronize()
    from rus_b200 import _lib

    assert _lib.device_error(reset=True) == 0
    return dict(loss=loss.detach(), nll=nll, entropy=ent, argmax=arg, dX=h.grad, dW=w.grad if want_dw else None)


def _close_per_token(ours, ref, rtol=1e-3, floor=1e-3):
    ours = ours.double().cpu()
    ref = ref.double().cpu()
    bad = (ours - ref).abs() > rtol * torch.maximum(ref.abs(), torch.full_like(ref, floor / rtol))
    return int(bad.sum())


def _check_contract(ours, ref, logits32, dtype, check_dw=True, label=""):
    """The north-star bars; returns the argmax report (printed with the case label)."""
    assert torch.isfinite(ours["loss"]).item()
    assert _close_per_token(ours["loss"].reshape(1), ref["loss"].reshape(1)) == 0, (ours["loss"], ref["loss"])
    assert _close_per_token(ours["nll"], ref["nll"]) == 0
    ent_o, ent_r = ours["entropy"].double().cpu(), ref["entropy"].double().cpu()
    assert ((ent_o - ent_r).abs() <= 1e-3 * torch.clamp(ent_r.abs(), min=1.0)).all()
    rep = orc.argmax_tie_report(ours["argmax"], ref["argmax"], logits32, dtype)
    print(f"argmax {label}: " + ", ".join(f"{k} {v}" for k, v in rep.items() if k != "ok"))
    # every mismatch is accepted by the tie rule, and every accepted one is a near-tie at the top
    assert rep["rejected"] == 0, f"{rep['rejected']} argmax mismatches beyond the tie rule"
    assert rep["not_top"] == 0, f"{rep['not_top']} accepted argmax mismatches away from the row maximum"
    dx_err = orc.rel_l2(ours["dX"].float(), ref["dX"].float())
    assert dx_err < 1e-2, dx_err
    if check_dw:
        dw_err = orc.rel_l2(ours["dW"].float(), ref["dW"].float())
        assert dw_err < 1e-2, dw_err
    return rep


def test_reference_known_answer(cuda_device):
    """solution/test_kernels.py:189-226 with its own inputs and tolerances."""
    torch.manual_seed(3)
    B, S, D, V = 2, 32, 256, 4099
    hidden = torch.randn((B, S, D), dtype=torch.float16)
    weight = torch.randn((V, D), dtype=torch.float16) * 0.02
    labels = torch.randint(0, V, (B, S), dtype=torch.long)
    labels[:, :8] = -100
    shift = torch.full((B, S), -100, dtype=torch.long)
    shift[:, :-1] = labels[:, 1:]

    ref = orc.eager_head(hidden, shift, weight)  # CPU oracle
    ours = _run_ours(hidden.to(cuda_device), shift.to(cuda_device), weight.to(cuda_device), v_chunk=1024)

    torch.testing.assert_close(ours["loss"].cpu(), ref["loss"], rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(ours["dX"].float().cpu().view(B * S, D), ref["dX"].float(), rtol=5e-3, atol=5e-3)
    torch.testing.assert_close(ours["entropy"].cpu(), ref["entropy"], rtol=2e-3, atol=2e-3)
    assert torch.equal(ours["argmax"].cpu(), ref["argmax"])
    torch.testing.assert_close(ours["dW"].float().cpu(), ref["dW"].float(), rtol=5e-3, atol=5e-3)


EDGE_CASES = [
    # (N, H, V, dtype, label pattern)
    (1, 64, 300, torch.float16, "all_valid"),
    (130, 128, 1000, torch.bfloat16, "half_masked"),
    (257, 192, 5000, torch.float16, "half_masked"),
    (64, 64, 100, torch.float16, "all_valid"),  # V smaller than one vocab tile
    (200, 256, 4099, torch.float16, "all_masked"),
    (384, 320, 2560, torch.bfloat16, "random"),
    # H >= 256 runs the CTA-pair backward: one labelled token, V below one vocab tile, H = 256
    (1, 256, 1000, torch.float16, "all_valid"),
    (70, 384, 100, torch.bfloat16, "all_valid"),
    (300, 256, 2000, torch.float16, "random"),
]


@pytest.mark.parametrize("n,h,v,dtype,pattern", EDGE_CASES)
def test_edge_cases(cuda_device, n, h, v, dtype, pattern):
    g = torch.Generator().manual_seed(n * 7 + h + v)
    hidden = torch.randn(n, h, generator=g).to(dtype)
    weight = (torch.randn(v, h, generator=g) * (2.0 / h ** 0.5)).to(dtype)
    labels = torch.randint(0, v, (n,), generator=g)
    if pattern == "half_masked":
        labels[: n // 2] = -100
    elif pattern == "all_masked":
        labels[:] = -100
    elif pattern == "random":
        labels[torch.rand(n, generator=g) < 0.3] = -100
    ref = orc.eager_head(hidden, labels, weight, grad_mode="fp32")
    ours = _run_ours(hidden.to(cuda_device), labels.to(cuda_device), weight.to(cuda_device), v_chunk=512)
    logits32 = hidden.float() @ weight.float().t()
    if pattern == "all_masked":
        assert ours["loss"].item() == 0.0
        assert float(ours["nll"].abs().max()) == 0.0
        assert float(ours["dX"].float().abs().max()) == 0.0
        assert float(ours["dW"].float().abs().max()) == 0.0
        ent_o, ent_r = ours["entropy"].double().cpu(), ref["entropy"].double()
        assert ((ent_o - ent_r).abs() <= 1e-3 * torch.clamp(ent_r.abs(), min=1.0)).all()
        return
    _check_contract(ours, ref, logits32, dtype)


@pytest.mark.parametrize("kind", ["int", "tensor", "zero", "negative"])
def test_num_items_in_batch(cuda_device, kind):
    """denom = num_items_in_batch clamped to >= 1 (ops.py:268-277: max(float(n), 1.0)), so a zero
    or negative count divides by 1, not by the number of labelled tokens."""
    g = torch.Generator().manual_seed(11)
    n, h, v = 96, 128, 3000
    hidden = torch.randn(n, h, generator=g).half()
    weight = (torch.randn(v, h, generator=g) * 0.05).half()
    labels = torch.randint(0, v, (n,), generator=g)
    labels[::3] = -100
    host = {"int": 500, "tensor": 500, "zero": 0, "negative": -7}[kind]
    num_items = torch.tensor(host, device=cuda_device) if kind == "tensor" else host
    ref = orc.eager_head(hidden, labels, weight, num_items_in_batch=host, grad_mode="fp32")
    if kind in ("zero", "negative"):
        assert ref["denom"] == 1.0
    ours = _run_ours(hidden.to(cuda_device), labels.to(cuda_device), weight.to(cuda_device), num_items=num_items)
    _check_contract(ours, ref, hidden.float() @ weight.float().t(), torch.float16)


@pytest.mark.parametrize("v_chunk", [256, 1024, 8192])
def test_v_chunk_invariance(cuda_device, v_chunk):
    """The backward's vocab chunking must not change the result beyond rounding."""
    g = torch.Generator().manual_seed(5)
    n, h, v = 300, 256, 9000
    hidden = torch.randn(n, h, generator=g).half().to(cuda_device)
    weight = (torch.randn(v, h, generator=g) * 0.05).half().to(cuda_device)
    labels = torch.randint(0, v, (n,), generator=g).to(cuda_device)
    a = _run_ours(hidden, labels, weight, v_chunk=v_chunk)
    b = _run_ours(hidden, labels, weight, v_chunk=v)
    assert orc.rel_l2(a["dX"].float(), b["dX"].float()) < 2e-3
    assert orc.rel_l2(a["dW"].float(), b["dW"].float()) < 2e-3
    assert torch.equal(a["argmax"], b["argmax"])


@pytest.mark.parametrize("cfg,n_override", [("c1", None), ("c5", 600), ("c5", None), ("c4", 256), ("c3", 256)])
def test_config_parity(cuda_device, cfg, n_override):
    """BASELINE.json configs (full H and V), against the reference eager path run on the GPU.
    ("c5", None) is the numerics-stress config at its full size (~2.7k tokens, three rows all
    ignored, logit std ~12, exact top-2 ties on 1% of the tokens)."""
    X, y, W, meta = orc.make_config_inputs(cfg, seed=0, device="cpu", n_override=n_override)
    Xd, yd, Wd = X.to(cuda_device), y.to(cuda_device), W.to(cuda_device)
    ref = orc.eager_head(Xd, yd, Wd, grad_mode="fp32")
    ours = _run_ours(Xd, yd, Wd)
    logits32 = (Xd.float() @ Wd.float().t())
    rep = _check_contract(ours, ref, logits32, X.dtype, label=f"{cfg} N={meta['N']}")
    if cfg == "c5":
        # the planted exact ties (two identical W rows, so identical fp32 logits in any
        # accumulation order) resolve to the lower index, as in the reference's argmax
        top = logits32.max(dim=1).values
        at_top = logits32 == top[:, None]
        tied = at_top.sum(1) > 1
        assert int(tied.sum()) >= max(1, meta["N"] // 200)
        first = torch.argmax(at_top.to(torch.int8), dim=1)
        assert torch.equal(ours["argmax"][tied].cpu(), first[tied].cpu())
    del logits32


@pytest.mark.parametrize("cfg", ["c1", "c2", "c5"])
def test_bench_workload_parity(cuda_device, cfg):
    """The exact inputs bench.py times (bench.make_config on the GPU, single GPU, the library's
    default vocab chunk), against the reference eager path on the GPU; c2 is the benchmark's
    headline workload (N=2048, H=1536, V=151936, fp16)."""
    import bench

    X, y, W, lens = bench.make_config(cfg, cuda_device)
    ref = orc.eager_head(X, y, W, grad_mode="fp32")
    ours = _run_ours(X, y, W)  # v_chunk None: the library's default, as in the benchmark
    logits32 = X.float() @ W.float().t()
    _check_contract(ours, ref, logits32, X.dtype, label=f"bench {cfg} N={X.shape[0]}")
    del logits32


def test_c1_against_cpu_oracle(cuda_device):
    """Config 1 at full size against the CPU oracle (eager formula, fp32 gradients)."""
    X, y, W, meta = orc.make_config_inputs("c1", seed=0)
    ref = orc.eager_head(X, y, W, grad_mode="fp32")
    ours = _run_ours(X.to(cuda_device), y.to(cuda_device), W.to(cuda_device))
    _check_contract(ours, ref, X.float() @ W.float().t(), X.dtype, label="c1 vs CPU oracle")


def test_forward_only_and_no_grad(cuda_device):
    from rus_b200 import chunked_lm_head

    g = torch.Generator().manual_seed(9)
    hidden = torch.randn(50, 128, generator=g).half().to(cuda_device)
    weight = (torch.randn(700, 128, generator=g) * 0.05).half().to(cuda_device)
    labels = torch.randint(0, 700, (50,), generator=g).to(cuda_device)
    with torch.no_grad():
        loss, nll, ent, arg = chunked_lm_head(hidden, labels, weight)
    ref = orc.eager_head(hidden.cpu(), labels.cpu(), weight.cpu(), grads=False)
    assert abs(loss.item() - ref["loss"].item()) <= 1e-3 * abs(ref["loss"].item())
    assert nll.shape == (50,) and ent.dtype == torch.float32 and arg.dtype == torch.int64
    assert not nll.requires_grad and not arg.requires_grad


def test_empty_batch(cuda_device):
    """N = 0 tokens (a packed batch with nothing kept): zero loss, empty per-token outputs,
    gradients of the right shapes and all zero."""
    from rus_b200 import chunked_lm_head

    h = torch.zeros(0, 128, dtype=torch.float16, device=cuda_device, requires_grad=True)
    w = (torch.randn(700, 128) * 0.05).half().to(cuda_device).requires_grad_(True)
    y = torch.zeros(0, dtype=torch.long, device=cuda_device)
    loss, nll, ent, arg = chunked_lm_head(h, y, w)
    loss.backward()
    assert loss.item() == 0.0
    assert nll.shape == (0,) and ent.shape == (0,) and arg.shape == (0,) and arg.dtype == torch.int64
    assert h.grad.shape == (0, 128)
    assert w.grad.shape == w.shape and float(w.grad.abs().max()) == 0.0


def test_label_out_of_range_is_reported(cuda_device):
    """A label that is neither -100 nor in [0, V) gives its token a NaN nll and leaves
    LMCE_ERR_LABEL_RANGE in the device error word; the kernels only compare labels (no memory is
    addressed by one), so the other tokens are unaffected and the backward stays finite. (The
    reference's eager F.cross_entropy stops on a device-side assert instead.)"""
    from rus_b200 import _lib, chunked_lm_head

    g = torch.Generator().manual_seed(21)
    n, hd, v = 96, 128, 700
    hidden = torch.randn(n, hd, generator=g).half()
    weight = (torch.randn(v, hd, generator=g) * 0.05).half()
    labels = torch.randint(0, v, (n,), generator=g)
    bad = labels.clone()
    bad[5] = v + 3
    bad[17] = -7
    _lib.device_error(reset=True)
    h = hidden.to(cuda_device).requires_grad_(True)
    loss, nll, ent, arg = chunked_lm_head(h, bad.to(cuda_device), weight.to(cuda_device))
    loss.backward()
    torch.cuda.synchronize()
    code = _lib.device_error(reset=True)
    assert _lib.device_error(reset=True) == 0
    assert code == _lib.LMCE_ERR_LABEL_RANGE
    nll = nll.cpu()
    assert bool(torch.isnan(nll[5])) and bool(torch.isnan(nll[17]))
    keep = torch.ones(n, dtype=torch.bool)
    keep[[5, 17]] = False
    ref = orc.eager_head(hidden, labels, weight, grads=False)
    assert _close_per_token(nll[keep], ref["nll"][keep]) == 0
    ent_o, ent_r = ent.double().cpu(), ref["entropy"].double()
    assert ((ent_o - ent_r).abs() <= 1e-3 * torch.clamp(ent_r.abs(), min=1.0)).all()
    assert bool(torch.isfinite(h.grad).all())


def test_timeout_path_reports_error(cuda_device):
    """A bounded wait that nothing satisfies returns LMCE_ERR_TIMEOUT instead of hanging."""
    from rus_b200 import _lib

    _lib.device_error(reset=True)
    _lib.call("lmce_selftest_wait_timeout", 50_000_000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == _lib.LMCE_ERR_TIMEOUT
    assert _lib.device_error(reset=True) == 0


def test_packed_batch_with_proxy(cuda_device):
    """Padding -> pack -> head -> scatter -> proxy (ops.py:1107-1184) against eager logits."""
    from rus_b200.packing import lm_head_with_proxy, shift_and_pack

    g = torch.Generator().manual_seed(17)
    B, S, H, V = 3, 40, 256, 5000
    hidden = torch.randn(B, S, H, generator=g).half()
    weight = (torch.randn(V, H, generator=g) * 0.05).half()
    labels = torch.randint(0, V, (B, S), generator=g)
    mask = torch.ones(B, S, dtype=torch.long)
    mask[0, 30:] = 0
    labels[0, 30:] = -100
    labels[1, :10] = -100
    packed = shift_and_pack(labels.to(cuda_device), mask.to(cuda_device))
    hp = hidden.reshape(-1, H).to(cuda_device).index_select(0, packed.valid_idx)
    loss, proxy = lm_head_with_proxy(hp, packed, weight.to(cuda_device))
    z = F.linear(hidden, weight).float()
    ref_loss = F.cross_entropy(z[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1), ignore_index=-100)
    assert abs(loss.item() - ref_loss.item()) <= 1e-3 * abs(ref_loss.item())
    assert proxy.shape == (B, S, V)
    kept = torch.zeros(B * S, dtype=torch.bool)
    kept[packed.valid_idx.cpu()] = True
    kept = kept.view(B, S)
    ent_ref = torch.logsumexp(z, -1) - torch.sum(F.softmax(z, -1) * z, -1)
    ent = (torch.logsumexp(proxy, -1) - torch.sum(F.softmax(proxy, -1) * proxy, -1)).cpu()
    assert ((ent[kept] - ent_ref[kept]).abs() <= 1e-3 * ent_ref[kept].abs().clamp(min=1)).all()
    ok = orc.argmax_mismatch_ok(proxy.argmax(-1).cpu()[kept], z.argmax(-1)[kept], z[kept], torch.float16)
    assert bool(ok.all())
    for row in range(B):
        r_ref = F.cross_entropy(z[row, :-1], labels[row, 1:], ignore_index=-100)
        r = F.cross_entropy(proxy[row, :-1].float(), labels[row, 1:].to(cuda_device), ignore_index=-100)
        assert abs(r.item() - r_ref.item()) <= 1e-3 * abs(r_ref.item())


@pytest.mark.parametrize("cfg", ["c3", "c4"])
def test_full_size_configs(cuda_device, cfg):
    """Configs 3 and 4 at their full token counts (N ~ 11.6k and 32768), against the reference eager
    path on the GPU, plus size-independent properties: ignored rows get exactly zero dX, the dW
    column sums vanish (sum_v G[t, v] = 0 for every labelled token), and the gradients are linear
    in grad_loss (doubling it doubles dX and dW exactly, up to one step of fp16's subnormal grid:
    doubling does not commute with rounding below 2^-14)."""
    from rus_b200 import chunked_lm_head

    X, y, W, meta = orc.make_config_inputs(cfg, seed=0, device="cpu")
    Xd, yd, Wd = X.to(cuda_device), y.to(cuda_device), W.to(cuda_device)
    del X, W
    ours = _run_ours(Xd, yd, Wd)
    ref = orc.eager_head(Xd, yd, Wd, grad_mode="fp32")
    logits32 = Xd.float() @ Wd.float().t()
    _check_contract(ours, ref, logits32, Xd.dtype, label=f"{cfg} full")
    del logits32, ref
    ignored = (yd == -100)
    if bool(ignored.any()):
        assert float(ours["dX"][ignored].abs().max()) == 0.0
    col = ours["dW"].float().sum(0)
    assert float(col.norm()) <= 1e-2 * float(ours["dW"].float().norm()) + 1e-6
    # linearity in grad_loss
    h = Xd.clone().requires_grad_(True)
    w = Wd.clone().requires_grad_(True)
    loss, *_ = chunked_lm_head(h, yd, w)
    (2.0 * loss).backward()
    assert ((h.grad.float() - 2 * ours["dX"].float()).abs() <= 2.0 ** -24).all()
    assert ((w.grad.float() - 2 * ours["dW"].float()).abs() <= 2.0 ** -24).all()
