"""GPU: the packing around the head (lmce_pack_tokens, lmce_scatter_token_outputs) against the
oracle's loop restatement of solution/ops.py:1107-1127 and 1151-1164."""
from __future__ import annotations

import pytest
import torch

from oracle import lmce_oracle as orc

pytestmark = pytest.mark.gpu


def _case(pattern, seed=4):
    g = torch.Generator().manual_seed(seed)
    if pattern == "config5":  # 64 rows x 512 (the config-5 shape), Zipf-like lengths, 3 rows unlabelled
        B, S, V = 64, 512, 151936
        lengths = torch.clamp((torch.rand(B, generator=g) ** -1.2).long(), 1, S)
        mask = (torch.arange(S)[None, :] < lengths[:, None]).long()
        labels = torch.randint(0, V, (B, S), generator=g)
        labels[mask == 0] = -100
        labels[:3] = -100
        return labels, mask
    B, S, V = 3, 17, 50
    labels = torch.randint(0, V, (B, S), generator=g)
    mask = torch.ones(B, S, dtype=torch.long)
    if pattern == "padded":
        mask[0, 12:] = 0
        labels[0, 12:] = -100
        mask[2, 5:] = 0
        labels[2, 3:] = -100
    elif pattern == "all_padded_no_labels":
        mask[:] = 0
        labels[:] = -100
    elif pattern == "no_mask":
        labels[1, 4:] = -100
        mask = None
    elif pattern == "seq1":
        labels = labels[:, :1]
        mask = torch.tensor([[1], [0], [1]])
    return labels, mask


@pytest.mark.parametrize("pattern", ["padded", "all_padded_no_labels", "full", "no_mask", "seq1", "config5"])
def test_pack_matches_reference_logic(cuda_device, pattern):
    from rus_b200.packing import shift_and_pack

    labels, mask = _case(pattern)
    B, S = labels.shape
    H = 64
    hidden = torch.randn(B, S, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    packed = shift_and_pack(labels.to(cuda_device), None if mask is None else mask.to(cuda_device),
                            hidden=hidden.to(cuda_device))
    lab, idx, lens = orc.pack_restatement(labels, mask)
    assert packed.shift_labels.tolist() == lab
    assert packed.valid_idx.tolist() == idx
    assert packed.row_lengths.tolist() == lens
    assert int(packed.count.item()) == len(idx)
    assert torch.equal(packed.hidden_packed.cpu(), hidden.reshape(B * S, H)[idx])


def test_scatter_matches_reference_logic(cuda_device):
    from rus_b200.packing import scatter_head_outputs, shift_and_pack

    labels, mask = _case("config5", seed=9)
    B, S = labels.shape
    packed = shift_and_pack(labels.to(cuda_device), mask.to(cuda_device))
    n = packed.valid_idx.numel()
    g = torch.Generator().manual_seed(2)
    nll = torch.rand(n, generator=g) * 10
    ent = torch.rand(n, generator=g) * 5
    arg = torch.randint(0, 151936, (n,), generator=g)
    full_nll, full_ent, full_arg = scatter_head_outputs(packed, nll.to(cuda_device), ent.to(cuda_device),
                                                        arg.to(cuda_device))
    ref_nll, ref_ent, ref_arg = orc.scatter_restatement(B * S, packed.valid_idx.tolist(), nll.tolist(),
                                                        ent.tolist(), arg.tolist())
    assert full_nll.shape == (B, S) and full_arg.dtype == torch.int64
    assert full_nll.cpu().view(-1).tolist() == pytest.approx(ref_nll, rel=0, abs=0)
    assert full_arg.cpu().view(-1).tolist() == ref_arg
    torch.testing.assert_close(full_ent.cpu().view(-1), torch.tensor(ref_ent, dtype=torch.float32), rtol=1e-6,
                               atol=1e-6)
