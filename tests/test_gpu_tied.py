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


def test_packed_norm_tied_flow_matches_autograd(cuda_device):
    """The flow around the head as the integration guide wires it (tied embedding -> layer
    stand-in -> pack -> fused final RMSNorm -> head with the tied slot -> scatter), against
    plain autograd through F.embedding, the oracle's RMSNorm and F.cross_entropy."""
    from rus_b200 import chunked_lm_head
    from rus_b200.packing import rms_norm_pack, scatter_head_outputs, shift_and_pack
    from rus_b200.tied import TiedGradSlot, tied_embedding

    B, S, H, V = 2, 96, 256, 5000
    g = torch.Generator(device=cuda_device).manual_seed(11)
    W0 = (torch.randn(V, H, device=cuda_device, generator=g) * 0.05).half()
    ids = torch.randint(0, V, (B, S), device=cuda_device, generator=g)
    labels = ids.clone()
    labels[:, :10] = -100
    mask = torch.ones(B, S, dtype=torch.long, device=cuda_device)
    mask[1, 70:] = 0
    labels[1, 70:] = -100
    norm_w = (1 + 0.1 * torch.randn(H, device=cuda_device, generator=g)).half()

    W = W0.clone().requires_grad_(True)
    slot = TiedGradSlot()
    h = tied_embedding(ids, W, slot) * 1.5 + 0.25  # stand-in for the model's layers
    packed = shift_and_pack(labels, mask)
    x = rms_norm_pack(h, norm_w, packed)
    loss, nll, ent, arg = chunked_lm_head(x, packed.shift_labels, W, None, None, slot)
    full_nll, full_ent, full_arg = scatter_head_outputs(packed, nll, ent, arg)
    loss.backward()

    Wr = W0.float().clone().requires_grad_(True)
    hr = F.embedding(ids, Wr) * 1.5 + 0.25
    xr, _ = orc.rms_norm_ref(hr, norm_w)
    xk = xr.reshape(-1, H)[packed.valid_idx]
    z = xk.half().float() @ Wr.half().float().T
    loss_r = F.cross_entropy(z, packed.shift_labels, ignore_index=-100, reduction="sum")
    loss_r = loss_r / (packed.shift_labels != -100).sum()
    loss_r.backward()
    assert abs(loss.item() - loss_r.item()) <= 2e-3 * abs(loss_r.item())
    assert orc.rel_l2(W.grad.float(), Wr.grad) < 2e-2
    assert full_nll.shape == (B, S) and full_arg.shape == (B, S)


def test_two_heads_share_one_slot(cuda_device):
    """Two micro-batches on one slot, their losses summed before one backward: the parked dW
    values add, and the weight gradient matches plain autograd."""
    from rus_b200 import chunked_lm_head
    from rus_b200.tied import TiedGradSlot, tied_embedding

    W0, ids, labels = _inputs(cuda_device, 1200, 256, 5000, torch.float16, seed=4)
    halves = (slice(0, 600), slice(600, 1200))

    W = W0.clone().requires_grad_(True)
    slot = TiedGradSlot()
    losses = [chunked_lm_head(tied_embedding(ids[s], W, slot) * k, labels[s], W, None, None, slot)[0]
              for s, k in zip(halves, (1.5, 0.5))]
    (losses[0] + losses[1]).backward()
    assert slot.dw is None

    Wr = W0.clone().requires_grad_(True)
    refs = [chunked_lm_head(F.embedding(ids[s], Wr) * k, labels[s], Wr)[0] for s, k in zip(halves, (1.5, 0.5))]
    (refs[0] + refs[1]).backward()
    assert abs(losses[0].item() - refs[0].item()) <= 1e-6 * abs(refs[0].item())
    # fp16 sums in a different order: a few ulps
    assert orc.rel_l2(W.grad.float(), Wr.grad.float()) < 4e-3
