"""CPU: ChunkedLogitsProxy and the packing around the head (host logic).

The proxy is fed the oracle's per-token statistics of the reference's known-answer
case (solution/test_kernels.py:189-241) and must answer the expressions TRL and
Soup evaluate on logits exactly as real logits would, including the three asserts
of the reference test that its own proxy fails (shape :235, shifted argmax :238,
per-row cross-entropy :240).
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import lmce_oracle as orc
from rus_b200.packing import scatter_head_outputs, shift_and_pack
from rus_b200.proxy import ChunkedLogitsProxy, fast_entropy_from_logits


@pytest.fixture(scope="module")
def ref_case():
    torch.manual_seed(3)
    B, S, D, V = 2, 32, 256, 4099
    hidden = torch.randn((B, S, D), dtype=torch.float16)
    weight = torch.randn((V, D), dtype=torch.float16) * 0.02
    labels = torch.randint(0, V, (B, S), dtype=torch.long)
    labels[:, :8] = -100
    shift = torch.full((B, S), -100, dtype=torch.long)
    shift[:, :-1] = labels[:, 1:]
    out = orc.eager_head(hidden, shift, weight, grads=False)
    logits = F.linear(hidden, weight).float()
    return dict(B=B, S=S, V=V, labels=labels, shift=shift, logits=logits,
                nll=out["nll"].view(B, S), ent=out["entropy"].view(B, S), arg=out["argmax"].view(B, S))


def _proxy(c):
    return ChunkedLogitsProxy(c["nll"], c["ent"], c["arg"], vocab_size=c["V"])


def test_metadata(ref_case):
    p = _proxy(ref_case)
    assert p.shape == (ref_case["B"], ref_case["S"], ref_case["V"])
    assert p.dim() == 3 and p.size(-1) == ref_case["V"] and p.dtype == torch.float16
    assert p.float().dtype == torch.float32 and p.to(torch.float32).dtype == torch.float32


def test_trl_entropy_expression(ref_case):
    p = _proxy(ref_case)
    ent = torch.logsumexp(p, dim=-1) - torch.sum(F.softmax(p, dim=-1) * p, dim=-1)
    z = ref_case["logits"]
    ref = torch.logsumexp(z, -1) - torch.sum(F.softmax(z, -1) * z, -1)
    torch.testing.assert_close(ent, ref, rtol=2e-3, atol=2e-3)
    assert fast_entropy_from_logits(p) is p.per_token_entropy
    with pytest.raises(TypeError):
        fast_entropy_from_logits(z)


def test_argmax_and_shift(ref_case):
    p = _proxy(ref_case)
    ref = ref_case["logits"].argmax(-1)
    assert torch.equal(p.argmax(dim=-1), ref)
    assert torch.equal(p[:, :-1].argmax(dim=-1), ref[:, :-1])
    assert torch.equal(p.argmax(dim=-1)[:, :-1], ref[:, :-1])
    assert p[:, :-1].shape == (ref_case["B"], ref_case["S"] - 1, ref_case["V"])
    assert torch.equal(p[..., :-1, :].argmax(-1), ref[:, :-1])


def test_rewind_row_cross_entropy(ref_case):
    p = _proxy(ref_case)
    z, labels = ref_case["logits"], ref_case["labels"]
    for row in range(ref_case["B"]):
        ref = F.cross_entropy(z[row, :-1], labels[row, 1:], ignore_index=-100)
        got = F.cross_entropy(p[row, :-1].float(), labels[row, 1:], ignore_index=-100)
        torch.testing.assert_close(got, ref, rtol=2e-3, atol=2e-3)
    V = ref_case["V"]
    shift = ref_case["shift"]
    ref_sum = F.cross_entropy(z.view(-1, V), shift.view(-1), ignore_index=-100, reduction="sum")
    got_sum = F.cross_entropy(p.view(-1, V), shift.view(-1), ignore_index=-100, reduction="sum")
    torch.testing.assert_close(got_sum, ref_sum, rtol=2e-3, atol=2e-3)
    got_none = F.cross_entropy(p.reshape(-1, V), shift.view(-1), reduction="none")
    assert got_none.shape == shift.view(-1).shape


def test_log_softmax_gather(ref_case):
    p = _proxy(ref_case)
    shift = ref_case["shift"].clamp(min=0)
    got = F.log_softmax(p, dim=-1).gather(-1, shift.unsqueeze(-1)).squeeze(-1)
    ref = F.log_softmax(ref_case["logits"], -1).gather(-1, shift.unsqueeze(-1)).squeeze(-1)
    valid = ref_case["shift"] != -100
    torch.testing.assert_close(got[valid], ref[valid], rtol=2e-3, atol=2e-3)


def test_layout_noops_keep_identity(ref_case):
    p = _proxy(ref_case)
    assert p.contiguous() is p and p.detach() is p and p.clone() is p


def _pack_loop(labels, mask):
    """Plain-Python restatement of ops.py:1107-1127 for checking."""
    B, S = labels.shape
    shift = [[-100] * S for _ in range(B)]
    for b in range(B):
        for s in range(S - 1):
            shift[b][s] = int(labels[b, s + 1])
    keep = [[bool(mask[b, s]) or shift[b][s] != -100 for s in range(S)] for b in range(B)]
    if not any(any(r) for r in keep):
        for b in range(B):
            keep[b][0] = True
    idx = [b * S + s for b in range(B) for s in range(S) if keep[b][s]]
    return [shift[i // S][i % S] for i in idx], idx, [sum(r) for r in keep]


@pytest.mark.parametrize("pattern", ["padded", "all_padded_no_labels", "full"])
def test_shift_and_pack_matches_reference_logic(pattern):
    g = torch.Generator().manual_seed(4)
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
    packed = shift_and_pack(labels, mask)
    lab, idx, lens = _pack_loop(labels, mask)
    assert packed.shift_labels.tolist() == lab
    assert packed.valid_idx.tolist() == idx
    assert packed.row_lengths.tolist() == lens


def test_scatter_fills_dropped_positions_with_mean_entropy():
    labels = torch.tensor([[5, 6, 7, -100], [1, 2, -100, -100]])
    mask = torch.tensor([[1, 1, 1, 0], [1, 1, 0, 0]])
    packed = shift_and_pack(labels, mask)
    n = packed.valid_idx.numel()
    nll = torch.arange(1, n + 1, dtype=torch.float32)
    ent = torch.linspace(0.5, 2.0, n)
    arg = torch.arange(10, 10 + n)
    full_nll, full_ent, full_arg = scatter_head_outputs(packed, nll, ent, arg)
    kept = torch.zeros(8, dtype=torch.bool)
    kept[packed.valid_idx] = True
    assert torch.equal(full_nll.view(-1)[kept], nll) and (full_nll.view(-1)[~kept] == 0).all()
    assert torch.allclose(full_ent.view(-1)[~kept], ent.mean().expand(int((~kept).sum())))
    assert torch.equal(full_arg.view(-1)[kept], arg)
