"""CPU: the tolerance study that decides against an fp8 weight stream for the head.

Question: can the head read W in fp8 (tcgen05 kind::f8f6f4) and still meet the parity bar
(loss, nll, lse and entropy 1e-3 relative per token; dX and dW 1e-2 relative L2; argmax exact
except within 1e-3 of a tie)? W of the config-1/2 head (V=151936, H=1536, ~N(0, 0.02)) is
quantised per row to fp8 with an absmax scale; the eager formula (fp16-rounded logits, fp32
softmax statistics, exact fp32 gradients) runs on 256 tokens with both weights.

The reference has no fp8 path; this test pins the decision not to build one: with e4m3 the
whole-distribution statistics (lse, entropy) and dW stay inside the bar, but the single-logit
quantities (nll, argmax) and dX fall outside it, and e5m2 is worse on every measure.
"""
from __future__ import annotations

import pytest
import torch


def _head(W: torch.Tensor, X: torch.Tensor, y: torch.Tensor):
    z = (X.float() @ W.float().T).half().float()
    lse = torch.logsumexp(z, -1)
    p = torch.softmax(z, -1)
    ent = lse - (p * z).sum(-1)
    valid = y != -100
    nll = torch.where(valid, lse - z.gather(1, y.clamp(min=0)[:, None])[:, 0], torch.zeros(()))
    g = p.clone()
    g[valid, y[valid]] -= 1
    g[~valid] = 0
    return dict(lse=lse, entropy=ent, nll=nll, argmax=z.argmax(-1), dX=g @ W.float(), dW=g.T @ X.float())


def _quantised(W: torch.Tensor, fmt) -> torch.Tensor:
    scale = W.float().abs().amax(1, keepdim=True) / torch.finfo(fmt).max
    return ((W.float() / scale).to(fmt).float() * scale).half()


@pytest.fixture(scope="module")
def study():
    torch.manual_seed(0)
    n, h, v = 256, 1536, 151936
    X = (torch.randn(n, h) * (1 + 0.1 * torch.randn(h))).half()
    W = (torch.randn(v, h) * 0.02).half()
    y = torch.randint(0, v, (n,))
    y[torch.rand(n) < 0.1] = -100
    ref = _head(W, X, y)
    out = {}
    for name, fmt in (("e4m3", torch.float8_e4m3fn), ("e5m2", torch.float8_e5m2)):
        q = _head(_quantised(W, fmt), X, y)
        rel = lambda a, b: float(((a - b).abs() / b.abs().clamp(min=1)).max())  # noqa: E731
        l2 = lambda a, b: float((a - b).norm() / b.norm())  # noqa: E731
        out[name] = dict(lse=rel(q["lse"], ref["lse"]), entropy=rel(q["entropy"], ref["entropy"]),
                         nll=rel(q["nll"], ref["nll"]), argmax=float((q["argmax"] == ref["argmax"]).float().mean()),
                         dX=l2(q["dX"], ref["dX"]), dW=l2(q["dW"], ref["dW"]))
    return out


def test_e4m3_weight_misses_the_parity_bar(study):
    r = study["e4m3"]
    print("e4m3:", {k: f"{v:.2e}" for k, v in r.items()})
    # inside the bar: whole-distribution statistics and dW
    assert r["lse"] < 1e-3 and r["entropy"] < 1e-3 and r["dW"] < 1e-2
    # outside it: the per-token target logit, the argmax and dX
    assert r["nll"] > 1e-3
    assert r["argmax"] < 0.99
    assert r["dX"] > 1e-2


def test_e5m2_is_worse_than_e4m3(study):
    a, b = study["e4m3"], study["e5m2"]
    print("e5m2:", {k: f"{v:.2e}" for k, v in b.items()})
    assert b["nll"] > a["nll"] and b["dX"] > a["dX"] and b["argmax"] < a["argmax"]
