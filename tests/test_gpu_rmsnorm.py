"""GPU: the final RMSNorm fused with the packing gather (lmce_rmsnorm_pack) and its backward
fused with the scatter (lmce_rmsnorm_backward), against the oracle's restatement of the
reference's rms_norm_fwd / rms_norm_bwd (solution/kernels.py:124-190), end to end through the
head, and timed against normalising every row and then gathering."""
from __future__ import annotations

import pytest
import torch

from oracle import lmce_oracle as orc

pytestmark = pytest.mark.gpu


def _batch(dev, dtype, B=4, S=300, H=1536, V=151936, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    h = (torch.randn(B, S, H, device=dev, generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(dtype)
    labels = torch.randint(0, V, (B, S), device=dev, generator=g)
    mask = torch.ones(B, S, dtype=torch.long, device=dev)
    mask[1, 200:] = 0
    labels[1, 200:] = -100
    labels[:, :20] = -100
    return h, w, labels, mask


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rmsnorm_pack_matches_reference(cuda_device, dtype):
    from rus_b200.packing import rms_norm_pack, shift_and_pack

    h, w, labels, mask = _batch(cuda_device, dtype)
    packed = shift_and_pack(labels, mask)
    hh = h.clone().requires_grad_(True)
    x = rms_norm_pack(hh, w, packed)
    ref, rstd = orc.rms_norm_ref(h.reshape(-1, h.shape[-1])[packed.valid_idx], w)
    # rsqrt and the summation order may move a value across a rounding boundary: one ulp
    ulp = 2 ** -10 if dtype == torch.float16 else 2 ** -7
    torch.testing.assert_close(x.float(), ref.float(), rtol=ulp, atol=ulp)
    dy = torch.randn_like(x)
    x.backward(dy)
    dref = torch.zeros_like(h).reshape(-1, h.shape[-1])
    dref[packed.valid_idx] = orc.rms_norm_bwd_ref(dy, h.reshape(-1, h.shape[-1])[packed.valid_idx], w, rstd)
    assert orc.rel_l2(hh.grad.reshape(-1, h.shape[-1]).float(), dref.float()) < 1e-2
    dropped = torch.ones(h.shape[0] * h.shape[1], dtype=torch.bool, device=cuda_device)
    dropped[packed.valid_idx] = False
    assert (hh.grad.reshape(-1, h.shape[-1])[dropped] == 0).all()


def test_rmsnorm_pack_head_end_to_end(cuda_device):
    """hidden [B, S, H] -> pack + final RMSNorm -> head -> loss.backward(): loss and d_hidden
    against the eager formula through autograd (fp32 gradients)."""
    from rus_b200 import chunked_lm_head
    from rus_b200.packing import rms_norm_pack, shift_and_pack

    h, w, labels, mask = _batch(cuda_device, torch.float16, B=2, S=256, H=512, V=20000, seed=3)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    W = (torch.randn(20000, 512, device=cuda_device, generator=g) * 0.05).half()
    packed = shift_and_pack(labels, mask)
    hh = h.clone().requires_grad_(True)
    loss = chunked_lm_head(rms_norm_pack(hh, w, packed), packed.shift_labels, W)[0]
    loss.backward()
    hr = h.float().clone().requires_grad_(True)
    x_ref, _ = orc.rms_norm_ref(hr, w)
    xk = x_ref.reshape(-1, 512)[packed.valid_idx]
    z = xk.half().float() @ W.float().T
    loss_ref = torch.nn.functional.cross_entropy(z, packed.shift_labels, ignore_index=-100, reduction="sum")
    loss_ref = loss_ref / (packed.shift_labels != -100).sum()
    loss_ref.backward()
    assert abs(loss.item() - loss_ref.item()) <= 2e-3 * abs(loss_ref.item())
    assert orc.rel_l2(hh.grad.float(), hr.grad) < 2e-2


def test_rmsnorm_pack_time(cuda_device):
    """Config-2 hidden size, 4 x 512 tokens, 10% dropped: fused pack + norm against norm over
    all rows then gather (the reference's order). Reported, not asserted."""
    from rus_b200 import _lib
    from rus_b200.ops import _stream
    from rus_b200.packing import shift_and_pack

    h, w, labels, mask = _batch(cuda_device, torch.float16, B=4, S=512)
    mask[:, 460:] = 0
    labels[:, 460:] = -100
    packed = shift_and_pack(labels, mask)
    n, H = packed.valid_idx.numel(), h.shape[-1]
    h2 = h.reshape(-1, H)
    x = torch.empty((n, H), dtype=h.dtype, device=cuda_device)
    full = torch.empty_like(h2)
    rstd = torch.empty(h2.shape[0], device=cuda_device)
    st = _stream(cuda_device)

    def fused():
        _lib.call("lmce_rmsnorm_pack", h2.data_ptr(), w.data_ptr(), 1e-6, packed.valid_idx.data_ptr(), None, n, H, 0,
                  x.data_ptr(), rstd.data_ptr(), st)

    def separate():
        _lib.call("lmce_rmsnorm_pack", h2.data_ptr(), w.data_ptr(), 1e-6, None, None, h2.shape[0], H, 0,
                  full.data_ptr(), rstd.data_ptr(), st)
        torch.index_select(full, 0, packed.valid_idx, out=x)

    res = {}
    for name, fn in (("fused", fused), ("norm_all_then_gather", separate)) * 2:
        for _ in range(3):
            fn()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(50):
            fn()
        b.record()
        torch.cuda.synchronize()
        res.setdefault(name, []).append(round(a.elapsed_time(b) / 50 * 1e3, 1))
    print("microseconds per call:", res)
