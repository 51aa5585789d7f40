"""CPU: the oracle pinned against golden vectors made by the reference itself.

tests/golden/*.npz hold outputs of fokyso82002-rgb/rus ``chunked_lm_head`` run on
CPU through Triton's interpreter (tests/golden/make_golden.py). The reference's
own known-answer test (solution/test_kernels.py:189-226) compares that op with
the eager formula at loss 2e-3, dX 5e-3, entropy 2e-3, argmax exact; the same
tolerances pin the oracle's eager formula here, and the oracle's numpy
restatement of the chunked algorithm must match the reference much more tightly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import lmce_oracle as orc
from tests.golden import make_golden as mg

CASES = list(mg.CASES)


@pytest.fixture(scope="module", params=CASES)
def case(request):
    name = request.param
    gold = mg.load_case(name)
    hidden, shift, weight, num_items, v_chunk = mg.make_case_inputs(name)
    return name, gold, hidden, shift, weight, num_items, v_chunk


def test_inputs_regenerate_bit_exactly(case):
    name, gold, hidden, shift, weight, *_ = case
    assert mg.input_digest(hidden, shift, weight) == gold["meta"]["digest"], f"{name}: generator drift"


def test_eager_oracle_matches_reference(case):
    name, gold, hidden, shift, weight, num_items, _ = case
    ref = orc.eager_head(hidden, shift, weight, num_items_in_batch=num_items)
    np.testing.assert_allclose(ref["loss"].item(), gold["loss"], rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(ref["nll"].numpy(), gold["nll"], rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(ref["entropy"].numpy(), gold["entropy"], rtol=2e-3, atol=2e-3)
    assert np.array_equal(ref["argmax"].numpy(), gold["argmax"])
    np.testing.assert_allclose(ref["dX"].float().numpy(), gold["dX"], rtol=5e-3, atol=5e-3)


def test_chunked_restatement_matches_reference(case):
    name, gold, hidden, shift, weight, num_items, v_chunk = case
    r = orc.chunked_restatement(hidden, shift, weight, num_items_in_batch=num_items, v_chunk=v_chunk)
    np.testing.assert_allclose(r["loss"], gold["loss"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r["nll"], gold["nll"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r["entropy"], gold["entropy"], rtol=1e-5, atol=1e-5)
    assert np.array_equal(r["argmax"], gold["argmax"])
    # fp16/bf16 dX accumulator: allow a couple of ulps of rounding-order difference
    denom = np.linalg.norm(gold["dX"]) or 1.0
    assert np.linalg.norm(r["dX"] - gold["dX"]) / denom < 2e-3


def test_reference_proxy_identities(case):
    """What works of the reference proxy (test_kernels.py:236-239): the TRL entropy
    expression returns per_token_entropy and argmax returns per_token_argmax."""
    name, gold, *_ = case
    np.testing.assert_array_equal(gold["proxy_entropy"], gold["entropy"])
    np.testing.assert_array_equal(gold["proxy_argmax"], gold["argmax"])


def test_ties_resolve_to_lowest_index():
    gold = mg.load_case("ties")
    hidden, shift, weight, *_ = mg.make_case_inputs("ties")
    z = (hidden.reshape(-1, hidden.shape[-1]).float() @ weight.float().t())
    z16 = z.half().float()
    top = z16.max(dim=1).values
    tied = (z16[:, 37] == top) & (z16[:, 100] == top)
    assert int(tied.sum()) > 32
    assert (gold["argmax"][tied.numpy()] == 37).all()


def test_all_masked_loss_is_zero():
    gold = mg.load_case("all_masked")
    assert float(gold["loss"]) == 0.0
    assert float(np.abs(gold["dX"]).max()) == 0.0


@pytest.mark.parametrize("world", [2, 3, 8])
def test_shard_merge_protocol(world):
    """Merging per-shard partial records reproduces the unsharded statistics."""
    hidden, shift, weight, num_items, _ = mg.make_case_inputs("bf16_ragged")
    h = hidden.reshape(-1, hidden.shape[-1])
    y = shift.reshape(-1)
    V = weight.shape[0]
    bounds = [V * r // world for r in range(world + 1)]
    recs = [orc.parts_of_shard(h, y, weight[bounds[r]:bounds[r + 1]], bounds[r]) for r in range(world)]
    fin = orc.finish_np(orc.part_merge_np(recs), y)
    full = orc.finish_np(orc.parts_of_shard(h, y, weight, 0), y)
    for k in ("lse", "entropy", "nll"):
        np.testing.assert_allclose(fin[k], full[k], rtol=1e-9, atol=1e-9)
    assert np.array_equal(fin["argmax"], full["argmax"])
    gold = mg.load_case("bf16_ragged")
    np.testing.assert_allclose(fin["loss"], gold["loss"], rtol=2e-3)


def test_config_generators():
    X, y, W, meta = orc.make_config_inputs("c1", seed=0)
    assert X.shape == (meta["N"], 1536) and W.shape == (151936, 1536) and X.dtype == torch.float16
    start = 0
    for L in meta["lens"]:  # first 40% of each row ignored
        k = int(0.4 * L)
        assert (y[start:start + k] == -100).all() and (y[start + k:start + L] != -100).all()
        start += L
    X, y, W, meta = orc.make_config_inputs("c5", seed=0, n_override=400)
    assert W.shape == (151936, 896)
    assert (y == -100).sum() > 0
    # config 5 at full size: Zipf(1.2) lengths truncated to 1..512 (E[N] ~ 2.8k), three rows all
    # ignored, and the exact top-2 ties (duplicated W rows) present
    X, y, W, meta = orc.make_config_inputs("c5", seed=0)
    assert 1500 <= meta["N"] <= 4500 and max(meta["lens"]) <= 512 and min(meta["lens"]) >= 1
    starts = [0]
    for L in meta["lens"][:-1]:
        starts.append(starts[-1] + L)
    full_rows = sum(bool((y[s0:s0 + L] == -100).all()) for s0, L in zip(starts, meta["lens"]))
    assert full_rows >= 3
    assert len(torch.unique(W, dim=0)) < W.shape[0]


def test_argmax_tie_report_classifies_mismatches():
    """The argmax report sorts mismatches by the rule that accepts them and flags any accepted
    mismatch whose candidates are not at the top of the row (planted here on the CPU)."""
    z = torch.tensor([[5.0, 5.0004, 1.0, 0.0],     # strict tie (gap 4e-4 < 1e-3)
                      [40.0, 40.02, 3.0, 0.0],     # within one fp16 ulp at 40 (0.03125), > 1e-3
                      [2.0, 9.0, 1.0, 0.0],        # real disagreement: rejected
                      [1.0, 0.5, 0.2, 0.0]])       # exact match
    ref = torch.tensor([1, 1, 1, 0])
    ours = torch.tensor([0, 0, 0, 0])
    rep = orc.argmax_tie_report(ours, ref, z, torch.float16)
    assert (rep["exact"], rep["strict"], rep["widened"], rep["rejected"]) == (1, 1, 1, 1)
    assert rep["not_top"] == 0
    assert rep["ok"].tolist() == [True, True, False, True]
    # a near-tie between two candidates far below the row maximum is accepted by the gap
    # alone but is not a tie at the top: not_top counts it
    z2 = torch.tensor([[10.0, 3.0, 3.0004, 0.0]])
    rep2 = orc.argmax_tie_report(torch.tensor([1]), torch.tensor([2]), z2, torch.float16)
    assert rep2["strict"] == 1 and rep2["not_top"] == 1
