"""Tied input embedding whose weight gradient shares the head's dW buffer.

With a tied embedding/lm_head weight (Qwen2.5-0.5B/1.5B), autograd would build two
[V, H] gradients, the head's dW and the embedding's scatter-add, and add them. Here
the head's backward (``chunked_lm_head(..., tied_slot=slot)``) parks its dW in the
slot and returns no weight gradient; the embedding's backward, which runs later in
the same backward pass, adds its rows into that buffer with
``lmce_embedding_grad_add`` (per token id, summed in fp64, one rounding) and returns
it as the weight's only gradient. The forward lookup is ``lmce_embedding_lookup``
(the reference's is HostHead.embed, solution/hostload.py:381-386).

Several heads and embeddings may share one slot within a backward pass (micro-batches
summed into one loss): a head adds its dW to whatever is parked, and the first
embedding backward that runs afterwards takes the sum; the others return their own
gradient alone, so the weight's total gradient is the same in every execution order.
A slot passed to a head must also reach an embedding on that head's input path: if a
backward pass parks a dW that no embedding backward collects (the head's input was
detached, or the embedding sits in another graph), the next forward through the slot
raises instead of adding that stale gradient into the next step's. A slot serves one
forward/backward at a time; micro-batches whose backward passes overlap need a slot each.
"""
from __future__ import annotations

import torch

from . import _lib
from .ops import _DTYPES, _stream


class TiedGradSlot:
    """Holds the head's dW between the head's backward and the embedding's backward."""

    def __init__(self):
        self.dw: torch.Tensor | None = None


class TiedEmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input_ids, weight, slot):
        if slot is not None and slot.dw is not None:
            raise RuntimeError(
                "tied_embedding: the slot still holds a head gradient from an earlier backward pass that "
                "no embedding backward collected (was the head's input detached from this embedding?); "
                "it would be added into this step's gradient. Clear it (slot.dw = None) or use one slot "
                "per forward/backward.")
        if weight.device.type != "cuda":
            raise RuntimeError("tied_embedding runs on CUDA tensors only (no CPU path)")
        ids = input_ids.contiguous().view(-1).to(torch.int64)
        w = weight.contiguous()
        v, h = w.shape
        out = torch.empty((ids.numel(), h), dtype=w.dtype, device=w.device)
        if ids.numel() > 0:
            with torch.cuda.device(w.device):
                _lib.call("lmce_embedding_lookup", w.data_ptr(), ids.data_ptr(), ids.numel(), h, v, 0,
                          out.data_ptr(), _stream(w.device))
        ctx.save_for_backward(ids)
        ctx.slot = slot
        ctx.wshape = (v, h)
        ctx.wdtype = w.dtype
        return out.view(*input_ids.shape, h)

    @staticmethod
    def backward(ctx, grad_out):
        (ids,) = ctx.saved_tensors
        if not ctx.needs_input_grad[1]:
            return None, None, None
        v, h = ctx.wshape
        dev = grad_out.device
        slot = ctx.slot
        dw = slot.dw if slot is not None else None
        if slot is not None:
            slot.dw = None
        if dw is None:  # no head gradient parked (untied use): the embedding gradient alone
            dw = torch.zeros((v, h), dtype=ctx.wdtype, device=dev)
        g = grad_out.contiguous().view(-1, h).to(ctx.wdtype)
        n = ids.numel()
        if n > 0:
            lib = _lib.load()
            ws_bytes = int(lib.lmce_embedding_grad_workspace_bytes(n, v))
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            with torch.cuda.device(dev):
                _lib.call("lmce_embedding_grad_add", g.data_ptr(), ids.data_ptr(), n, h, v, 0, _DTYPES[ctx.wdtype],
                          dw.data_ptr(), ws.data_ptr(), ws_bytes, _stream(dev))
        return None, dw, None


def tied_embedding(input_ids: torch.Tensor, weight: torch.Tensor, slot: TiedGradSlot | None = None) -> torch.Tensor:
    """Embedding lookup ``weight[input_ids]`` whose weight gradient is added into the head's dW
    parked in ``slot`` (pass the same slot to ``chunked_lm_head``). Ids outside [0, V) give
    zero rows and no gradient (the library's lookup serves vocab shards that way); unlike
    ``F.embedding`` they are not reported, since checking would need a host read."""
    return TiedEmbeddingFn.apply(input_ids, weight, slot)
