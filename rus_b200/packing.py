"""Packing around the head: causal label shift, padding-free token packing, and
scattering the head's per-token outputs back to [B, S] for the logits proxy.

Mirrors the patched ``Qwen2ForCausalLM.forward`` of the reference
(``solution/ops.py:1107-1127`` before the head, ``ops.py:1151-1184`` after it) with
the library's own kernels (``lmce_pack_tokens``, ``lmce_scatter_token_outputs``): two
launches each way, the kept count and the mean-entropy filler stay on the device, and
the only host read is the kept count that sizes the packed tensors (the reference
reads the row lengths with ``.tolist()`` at ops.py:1117, the mean entropy with
``.item()`` at ops.py:1161, and ``torch.nonzero`` reads its count as well). CUDA
tensors only: there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .ops import _DTYPES, _stream, chunked_lm_head
from .proxy import ChunkedLogitsProxy

IGNORE = -100


@dataclass
class PackedBatch:
    shift_labels: torch.Tensor   # [N] int64 labels of the kept positions (-100 = ignored)
    valid_idx: torch.Tensor      # [N] flat indices (into B*S) of the kept positions
    row_lengths: torch.Tensor    # [B] int32 kept positions per row (device)
    batch: int
    seq: int
    count: torch.Tensor | None = None          # [1] int32 N on the device
    hidden_packed: torch.Tensor | None = None  # [N, H] kept rows of the hidden states, when asked for


def _ptr(t):
    return None if t is None else t.data_ptr()


def shift_and_pack(labels: torch.Tensor, attention_mask: torch.Tensor | None = None,
                   hidden: torch.Tensor | None = None) -> PackedBatch:
    """ops.py:1107-1127: shift labels left by one (last position -100), keep positions that are
    attended or carry a label (position 0 of every row when none is kept), and pack them; with
    ``hidden`` ([B, S, H] fp16/bf16) the kept rows are gathered as well."""
    if labels.device.type != "cuda":
        raise RuntimeError("shift_and_pack runs on CUDA tensors only (no CPU path)")
    B, S = labels.shape
    dev = labels.device
    total = B * S
    lab = labels.to(torch.int64).contiguous()
    mask = None if attention_mask is None else attention_mask.to(device=dev, dtype=torch.int64).contiguous()
    shift = torch.empty(total, dtype=torch.int64, device=dev)
    idx = torch.empty(total, dtype=torch.int64, device=dev)
    row_lengths = torch.empty(B, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    h2d, hp, hdim, dt = None, None, 0, 0
    if hidden is not None:
        hdim = hidden.shape[-1]
        h2d = hidden.reshape(total, hdim).contiguous()
        hp = torch.empty_like(h2d)
        dt = _DTYPES[h2d.dtype]
    with torch.cuda.device(dev):
        _lib.call("lmce_pack_tokens", lab.data_ptr(), _ptr(mask), B, S, shift.data_ptr(), idx.data_ptr(),
                  row_lengths.data_ptr(), count.data_ptr(), _ptr(h2d), hdim, dt, _ptr(hp), _stream(dev))
    n = int(count.item())  # the one host read: sizes the packed tensors
    return PackedBatch(shift_labels=shift[:n], valid_idx=idx[:n], row_lengths=row_lengths, batch=B, seq=S,
                       count=count, hidden_packed=hp[:n] if hp is not None else None)


def scatter_head_outputs(packed: PackedBatch, nll: torch.Tensor, entropy: torch.Tensor, argmax: torch.Tensor):
    """ops.py:1151-1164: per-token outputs back to [B, S]; dropped positions get nll 0,
    argmax 0 and the mean entropy of the kept tokens (computed on the device)."""
    B, S = packed.batch, packed.seq
    dev = nll.device
    if dev.type != "cuda":
        raise RuntimeError("scatter_head_outputs runs on CUDA tensors only (no CPU path)")
    count = packed.count
    if count is None:
        count = torch.tensor([packed.valid_idx.numel()], dtype=torch.int32, device=dev)
    full_nll = torch.empty(B * S, dtype=torch.float32, device=dev)
    full_ent = torch.empty(B * S, dtype=torch.float32, device=dev)
    full_arg = torch.empty(B * S, dtype=torch.int64, device=dev)
    nll_c = nll.to(torch.float32).contiguous()
    ent_c = entropy.to(torch.float32).contiguous()
    arg_c = argmax.to(torch.int64).contiguous()
    idx = packed.valid_idx.contiguous()
    with torch.cuda.device(dev):
        _lib.call("lmce_scatter_token_outputs", nll_c.data_ptr(), ent_c.data_ptr(), arg_c.data_ptr(), idx.data_ptr(),
                  count.data_ptr(), B * S, full_nll.data_ptr(), full_ent.data_ptr(), full_arg.data_ptr(),
                  _stream(dev))
    return full_nll.view(B, S), full_ent.view(B, S), full_arg.view(B, S)


class RMSNormPackFn(torch.autograd.Function):
    """Final RMSNorm of the kept rows, written packed (lmce_rmsnorm_pack); backward scatters
    d_hidden to the unpacked rows, zero elsewhere (lmce_rmsnorm_backward)."""

    @staticmethod
    def forward(ctx, hidden, weight, eps, valid_idx):
        hdim = hidden.shape[-1]
        h2d = hidden.reshape(-1, hdim).contiguous()
        w = weight.contiguous()
        n = valid_idx.numel()
        dev = h2d.device
        x = torch.empty((n, hdim), dtype=h2d.dtype, device=dev)
        rstd = torch.empty(n, dtype=torch.float32, device=dev)
        if n > 0:
            with torch.cuda.device(dev):
                _lib.call("lmce_rmsnorm_pack", h2d.data_ptr(), w.data_ptr(), float(eps), valid_idx.data_ptr(), None,
                          n, hdim, _DTYPES[h2d.dtype], x.data_ptr(), rstd.data_ptr(), _stream(dev))
        ctx.save_for_backward(h2d, w, rstd, valid_idx)
        ctx.shape = hidden.shape
        return x

    @staticmethod
    def backward(ctx, dx):
        h2d, w, rstd, valid_idx = ctx.saved_tensors
        dh = torch.zeros_like(h2d)
        n = valid_idx.numel()
        if n > 0 and ctx.needs_input_grad[0]:
            g = dx.to(h2d.dtype).contiguous()
            with torch.cuda.device(h2d.device):
                _lib.call("lmce_rmsnorm_backward", g.data_ptr(), h2d.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                          valid_idx.data_ptr(), None, n, h2d.shape[1], _DTYPES[h2d.dtype], dh.data_ptr(),
                          _stream(h2d.device))
        return dh.view(ctx.shape), None, None, None


def rms_norm_pack(hidden: torch.Tensor, weight: torch.Tensor, packed: PackedBatch, eps: float = 1e-6):
    """The final RMSNorm in front of the head (ops.py:824) applied to the kept rows only and
    written packed, replacing normalise-all-then-gather; [N, H] for ``chunked_lm_head``. The
    norm weight is frozen, as in the reference (its gradient is not computed)."""
    if hidden.device.type != "cuda":
        raise RuntimeError("rms_norm_pack runs on CUDA tensors only (no CPU path)")
    if weight.requires_grad:
        raise RuntimeError("rms_norm_pack does not compute the norm weight's gradient; pass a frozen weight")
    return RMSNormPackFn.apply(hidden, weight, eps, packed.valid_idx)


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
