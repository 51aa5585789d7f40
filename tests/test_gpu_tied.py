"""GPU: the tied input embedding's gradient added into the head's dW (rus_b200.tied) against
plain autograd, where F.embedding's gradient and the head's dW are two tensors that the engine
adds; plus determinism and the time of the two ways."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import lmce_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(dev, n, h, v, dtype, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    W = (torch.randn(v, h, device=dev, generator=g) * 0.05).to(dtype)
    # Zipf-like ids: a few very frequent tokens, many rare ones
    ids = (torch.rand(n, device=dev, generator=g) ** 3 * v).long().clamp_(max=v - 1)
    labels = torch.randint(0, v, (n,), device=dev, generator=g)
    labels[torch.rand(n, device=dev, generator=g) < 0.1] = -100
    return W, ids, labels


def _step(W0, ids, labels, tied):
    from rus_b200 import chunked_lm_head
    from rus_b200.tied import TiedGradSlot, tied_embedding

    W = W0.clone().requires_grad_(True)
    if tied:
        slot = TiedGradSlot()
        x = tied_embedding(ids, W, slot)
        loss = chunked_lm_head(x * 1.5, labels, W, None, None, slot)[0]
    else:
        x = F.embedding(ids, W)
        loss = chunked_lm_head(x * 1.5, labels, W)[0]
    loss.backward()
    return W.grad


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tied_gradient_matches_autograd(cuda_device, dtype):
    W, ids, labels = _inputs(cuda_device, 1500, 256, 5000, dtype)
    ours = _step(W, ids, labels, tied=True)
    ref = _step(W, ids, labels, tied=False)
    # one rounding (ours) against two (embedding gradient, then the sum): within a dtype ulp
    assert orc.rel_l2(ours.float(), ref.float()) < (2e-3 if dtype == torch.float16 else 8e-3)
    # rows of ids that never occur carry the head's dW alone, identical in both
    unused = torch.ones(W.shape[0], dtype=torch.bool, device=cuda_device)
    unused[ids] = False
    assert torch.equal(ours[unused], ref[unused])
    again = _step(W, ids, labels, tied=True)
    assert torch.equal(ours, again), "tied gradient is not deterministic"


def test_tied_gradient_time(cuda_device):
    """Config-2 head (H=1536, V=151936, fp16, 2048 tokens): one backward with the shared dW
    buffer against plain autograd's two [V, H] gradients. Reported, not asserted."""
    W, ids, labels = _inputs(cuda_device, 2048, 1536, 151936, torch.float16)
    times = {}
    for tied in (False, True) * 3:
        for _ in range(2):
            _step(W, ids, labels, tied)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            _step(W, ids, labels, tied)
        b.record()
        torch.cuda.synchronize()
        times.setdefault("tied" if tied else "autograd", []).append(a.elapsed_time(b) / 10)
    print("fwd+bwd ms per step:", {k: [round(x, 3) for x in v] for k, v in times.items()})
