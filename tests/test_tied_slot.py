"""CPU: the tied-gradient slot's guard (host logic only; the kernels are covered by the GPU tests).

When a head parks its dW in a slot and no embedding backward collects it (here: the head's
input was detached from the embedding, so autograd never reaches the embedding), the next
forward through that slot must refuse to run rather than add the stale gradient into the
next step's weight gradient.
"""
from __future__ import annotations

import pytest
import torch

from rus_b200.tied import TiedGradSlot, tied_embedding


def test_stale_parked_gradient_is_refused_before_any_device_work():
    slot = TiedGradSlot()
    # what a head's backward leaves when its input was detached: a parked dW nobody took
    slot.dw = torch.zeros(16, 8)
    ids = torch.tensor([[1, 2, 3]])
    w = torch.zeros(16, 8)
    with pytest.raises(RuntimeError, match="still holds a head gradient"):
        tied_embedding(ids, w, slot)
    assert slot.dw is not None  # left in place for the caller to inspect or clear


def test_empty_slot_reaches_the_device_check():
    slot = TiedGradSlot()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        tied_embedding(torch.tensor([[1, 2]]), torch.zeros(16, 8), slot)
