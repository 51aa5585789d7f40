"""Packing around the head: causal label shift, padding-free token packing, and
scattering the head's per-token outputs back to [B, S] for the logits proxy.

Mirrors the patched ``Qwen2ForCausalLM.forward`` of the reference
(``solution/ops.py:1107-1127`` before the head, ``ops.py:1151-1184`` after it)
without its host synchronisations: row lengths stay on the device (the
reference's ``.tolist()`` at ops.py:1117 feeds its layer engine, which is not
part of this path) and the entropy filler for dropped positions is the mean
entropy computed on the device (the reference's ``.item()`` at ops.py:1161).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .ops import chunked_lm_head
from .proxy import ChunkedLogitsProxy

IGNORE = -100


@dataclass
class PackedBatch:
    shift_labels: torch.Tensor   # [N] int64 labels of the kept positions (-100 = ignored)
    valid_idx: torch.Tensor      # [N] flat indices (into B*S) of the kept positions
    row_lengths: torch.Tensor    # [B] int32 kept positions per row (device)
    batch: int
    seq: int


def shift_and_pack(labels: torch.Tensor, attention_mask: torch.Tensor | None = None) -> PackedBatch:
    """ops.py:1107-1127: shift labels left by one (last position -100), keep positions that are
    attended or carry a label (at least one token per batch), and pack them."""
    B, S = labels.shape
    dev = labels.device
    if attention_mask is None:
        attention_mask = torch.ones((B, S), dtype=torch.long, device=dev)
    shift = torch.full((B, S), IGNORE, dtype=torch.int64, device=dev)
    if S > 1:
        shift[:, :-1] = labels[:, 1:].to(torch.int64)
    keep = attention_mask.bool() | (shift != IGNORE)
    # at least one token per batch (ops.py:1113-1115), without a host round trip
    none_kept = ~keep.any()
    keep[:, 0] |= none_kept
    valid_idx = torch.nonzero(keep.reshape(-1), as_tuple=False).squeeze(-1)
    return PackedBatch(shift_labels=shift.reshape(-1).index_select(0, valid_idx), valid_idx=valid_idx,
                       row_lengths=keep.sum(dim=-1, dtype=torch.int32), batch=B, seq=S)


def scatter_head_outputs(packed: PackedBatch, nll: torch.Tensor, entropy: torch.Tensor, argmax: torch.Tensor):
    """ops.py:1151-1164: per-token outputs back to [B, S]; dropped positions get nll 0,
    argmax 0 and the mean entropy of the kept tokens."""
    B, S = packed.batch, packed.seq
    dev = nll.device
    full_nll = torch.zeros(B * S, dtype=torch.float32, device=dev).index_copy_(0, packed.valid_idx, nll)
    full_arg = torch.zeros(B * S, dtype=torch.int64, device=dev).index_copy_(0, packed.valid_idx, argmax)
    mean_ent = entropy.mean() if entropy.numel() > 0 else torch.zeros((), dtype=torch.float32, device=dev)
    full_ent = mean_ent.expand(B * S).clone().index_copy_(0, packed.valid_idx, entropy)
    return full_nll.view(B, S), full_ent.view(B, S), full_arg.view(B, S)


def lm_head_with_proxy(hidden_packed: torch.Tensor, packed: PackedBatch, weight: torch.Tensor,
                       num_items_in_batch=None, v_chunk: int | None = None, proxy_dtype=torch.float16):
    """Steps 3-4 of the reference's fused forward (ops.py:1143-1184): the head on packed
    hidden states, then a zero-storage [B, S, V] logits proxy. Returns (loss, proxy)."""
    loss, nll, ent, arg = chunked_lm_head(hidden_packed, packed.shift_labels, weight, num_items_in_batch, v_chunk)
    full_nll, full_ent, full_arg = scatter_head_outputs(packed, nll, ent, arg)
    V = weight.shape[0]
    proxy = ChunkedLogitsProxy(full_nll, full_ent, full_arg, V, virtual_shape=(packed.batch, packed.seq, V),
                               dtype=proxy_dtype)
    return loss, proxy
