"""CPU: ChunkedLogitsProxy, and the oracle's restatement of the packing around the head.

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
from rus_b200.packing import shift_and_pack
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


def test_pack_restatement_known_case():
    """The oracle's loop restatement of ops.py:1107-1127 on a hand-checked case."""
    labels = torch.tensor([[5, 6, 7, -100], [1, 2, -100, -100]])
    mask = torch.tensor([[1, 1, 1, 0], [1, 1, 0, 0]])
    lab, idx, lens = orc.pack_restatement(labels, mask)
    # row 0: shifted 6, 7, -100, -100; attended 0..2 -> keep 0, 1, 2
    # row 1: shifted 2, -100, -100, -100; attended 0, 1 -> keep 4, 5
    assert idx == [0, 1, 2, 4, 5] and lab == [6, 7, -100, 2, -100] and lens == [3, 2]
    lab, idx, lens = orc.pack_restatement(torch.full((2, 3), -100), torch.zeros(2, 3, dtype=torch.long))
    assert idx == [0, 3] and lab == [-100, -100] and lens == [1, 1]
    full = orc.scatter_restatement(6, [1, 4], [1.0, 2.0], [0.5, 1.5], [7, 8])
    assert full == ([0.0, 1.0, 0.0, 0.0, 2.0, 0.0], [1.0, 0.5, 1.0, 1.0, 1.5, 1.0], [0, 7, 0, 0, 8, 0])


def test_packing_refuses_cpu_tensors():
    """The product path has no CPU fallback."""
    labels = torch.tensor([[5, 6, 7, -100]])
    with pytest.raises(RuntimeError, match="CUDA"):
        shift_and_pack(labels)
