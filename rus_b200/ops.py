"""Fused lm_head cross-entropy head — host side of the reference's operator API.

``chunked_lm_head`` / ``FusedChunkedLMHeadFn`` keep the signature and output
contract of fokyso82002-rgb/rus ``solution/ops.py:174-349``:

    loss, per_token_nll, per_token_entropy, per_token_argmax = chunked_lm_head(
        hidden_states, shift_labels, weight, num_items_in_batch=None, v_chunk=8192)

* ``hidden_states`` [..., H] fp16/bf16 on a B200, ``shift_labels`` [...] int
  (-100 = ignored), ``weight`` [V, H] in the same dtype (a device tensor; the
  reference's host-pinned ``HostHead`` streamer is a 16 GB-GPU workaround and is
  not accepted here).
* ``loss`` is a differentiable fp32 scalar ``sum(nll) / denom`` with
  ``denom = num_items_in_batch`` if given, else the number of labels != -100,
  clamped to >= 1 (ops.py:268-277). ``per_token_nll``, ``per_token_entropy``
  (fp32) and ``per_token_argmax`` (int64) are flat [N] and non-differentiable
  (ops.py:326-330).
* ``v_chunk`` is the vocab chunk of the gradient pass (default: chosen by the library).
* ``backward`` returns dX in the dtype and shape of ``hidden_states`` and, when
  ``weight.requires_grad``, dW in the dtype of ``weight``. (The reference
  returns ``None`` for the weight, ops.py:339; its gradient pass is also never
  reached because ``torch.is_grad_enabled()`` is False inside
  ``Function.forward``, ops.py:280.)

All arithmetic runs in the sm_100a kernels of ``liblmce.so`` (include/lmce.h);
there is no CPU or PyTorch fallback. No [N, V] logits tensor is allocated:
the forward keeps N x slabs x 24 bytes of partial statistics, the backward a
vocab-chunk gradient tile of N x v_chunk elements.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

V_CHUNK_DEFAULT = 8192  # the reference's default chunk; pass it explicitly to force that chunk width

_DTYPES = {torch.float16: _lib.LMCE_DTYPE_F16, torch.bfloat16: _lib.LMCE_DTYPE_BF16}


def _debug_sync() -> bool:
    return os.environ.get("LMCE_DEBUG", "0") not in ("", "0")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_inputs(hidden: torch.Tensor, labels: torch.Tensor, weight: torch.Tensor) -> None:
    if not isinstance(weight, torch.Tensor):
        raise TypeError(
            "weight_or_host_head must be a device tensor [V, H]; host-streamed heads are not supported on B200"
        )
    if not hidden.is_cuda or not weight.is_cuda or not labels.is_cuda:
        raise _lib.LmceError(_lib.LMCE_ERR_UNSUPPORTED, "lmce runs on CUDA tensors only (no CPU fallback)")
    if hidden.dtype not in _DTYPES:
        raise _lib.LmceError(_lib.LMCE_ERR_UNSUPPORTED, f"hidden dtype {hidden.dtype} (need fp16 or bf16)")
    if weight.dtype != hidden.dtype:
        raise _lib.LmceError(_lib.LMCE_ERR_UNSUPPORTED, "hidden and weight must have the same dtype")
    if weight.dim() != 2 or weight.shape[1] != hidden.shape[-1]:
        raise _lib.LmceError(_lib.LMCE_ERR_INVALID_ARGUMENT, "weight must be [V, H] with H = hidden.shape[-1]")
    if hidden.device != weight.device or labels.device != hidden.device:
        raise _lib.LmceError(_lib.LMCE_ERR_INVALID_ARGUMENT, "all tensors must be on the same device")


def _denom_args(num_items_in_batch, device: torch.device):
    """(device pointer or None, host value or NaN for "not given", keep-alive tensor)."""
    if num_items_in_batch is None:
        return None, float("nan"), None
    if isinstance(num_items_in_batch, torch.Tensor):
        t = num_items_in_batch.detach().to(device=device, dtype=torch.float32).reshape(1).contiguous()
        return t.data_ptr(), float("nan"), t
    return None, float(num_items_in_batch), None


def head_forward_stats(h2d: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, vocab_offset: int = 0):
    """Run the fused logits GEMM + online statistics over one vocab shard.

    Returns the per-token partial records as a uint8 tensor [N, n_parts * 24]
    and ``n_parts``."""
    n, h = h2d.shape
    v = weight.shape[0]
    lib = _lib.load()
    n_parts = int(lib.lmce_fwd_num_parts(n, v))
    parts = torch.empty((n, n_parts * _lib.PART_BYTES), dtype=torch.uint8, device=h2d.device)
    _lib.call(
        "lmce_fwd_stats",
        h2d.data_ptr(),
        weight.data_ptr(),
        labels.data_ptr(),
        n,
        h,
        v,
        vocab_offset,
        _DTYPES[h2d.dtype],
        parts.data_ptr(),
        n_parts,
        _stream(h2d.device),
    )
    return parts, n_parts


def head_finish(parts: torch.Tensor, n_parts: int, tok_stride: int, part_stride: int, labels: torch.Tensor,
                num_items_in_batch=None):
    """Merge partial records and produce (loss, nll, entropy, argmax, lse, denom)."""
    n = labels.numel()
    dev = labels.device
    lse = torch.empty(n, dtype=torch.float32, device=dev)
    nll = torch.empty(n, dtype=torch.float32, device=dev)
    ent = torch.empty(n, dtype=torch.float32, device=dev)
    arg = torch.empty(n, dtype=torch.int64, device=dev)
    scalars = torch.empty(2, dtype=torch.float32, device=dev)
    ni_ptr, ni_val, _keep = _denom_args(num_items_in_batch, dev)
    _lib.call(
        "lmce_stats_finish",
        parts.data_ptr(),
        n_parts,
        tok_stride,
        part_stride,
        labels.data_ptr(),
        n,
        ni_ptr,
        ni_val,
        lse.data_ptr(),
        nll.data_ptr(),
        ent.data_ptr(),
        arg.data_ptr(),
        scalars[0:1].data_ptr(),
        scalars[1:2].data_ptr(),
        _stream(dev),
    )
    if _debug_sync():
        _raise_device_error()
    return scalars[0], nll, ent, arg, lse, scalars[1:2]


def head_backward(h2d, weight, labels, lse, grad_loss, denom, want_dx: bool, want_dw: bool,
                  v_chunk: int | None = None, vocab_offset: int = 0, dx_f32: torch.Tensor | None = None):
    """Recompute logits per vocab chunk and contract G into dX / dW (no [N, V] buffer)."""
    n, h = h2d.shape
    v = weight.shape[0]
    dev = h2d.device
    lib = _lib.load()
    v_chunk = int(v_chunk or 0)
    ws_bytes = int(lib.lmce_bwd_workspace_bytes(n, h, v, v_chunk))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    dx = torch.empty_like(h2d) if (want_dx and dx_f32 is None) else None
    dw = torch.empty_like(weight) if want_dw else None
    gl = grad_loss.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    _lib.call(
        "lmce_backward",
        h2d.data_ptr(),
        weight.data_ptr(),
        labels.data_ptr(),
        lse.data_ptr(),
        n,
        h,
        v,
        vocab_offset,
        _DTYPES[h2d.dtype],
        gl.data_ptr(),
        denom.data_ptr(),
        _ptr(dx),
        _ptr(dx_f32),
        _ptr(dw),
        v_chunk,
        ws.data_ptr(),
        ws_bytes,
        _stream(dev),
    )
    if _debug_sync():
        _raise_device_error()
    return dx, dw


def head_backward_nvls(h2d, weight, labels, lse, grad_loss, denom, xch, want_dw: bool,
                       v_chunk: int | None = None, vocab_offset: int = 0):
    """Backward of one vocab shard with the cross-GPU dX sum fused into the kernel
    (lmce_backward_nvls); ``xch`` is the ``_lib.DxExchange`` of the group's symmetric
    buffers. Returns this shard's dW (or None); the summed dX lands in every rank's
    copy of ``xch.out_mc``."""
    n, h = h2d.shape
    v = weight.shape[0]
    dev = h2d.device
    lib = _lib.load()
    v_chunk = int(v_chunk or 0)
    ws_bytes = int(lib.lmce_bwd_workspace_bytes(n, h, v, v_chunk))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    dw = torch.empty_like(weight) if want_dw else None
    gl = grad_loss.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    _lib.call("lmce_backward_nvls", h2d.data_ptr(), weight.data_ptr(), labels.data_ptr(), lse.data_ptr(), n, h, v,
              vocab_offset, _DTYPES[h2d.dtype], gl.data_ptr(), denom.data_ptr(), ctypes.byref(xch), _ptr(dw),
              v_chunk, ws.data_ptr(), ws_bytes, _stream(dev))
    if _debug_sync():
        _raise_device_error()
    return dw


def _raise_device_error() -> None:
    code = _lib.device_error(reset=True)
    if code != _lib.LMCE_OK:
        raise _lib.LmceError(code, "reported by a kernel")


class FusedChunkedLMHeadFn(torch.autograd.Function):
    """Exact cross-entropy loss, per-token NLL, Shannon entropy and argmax of
    ``hidden_states @ weight.T`` without materialising the [N, V] logits."""

    @staticmethod
    def forward(ctx, hidden_states, shift_labels, weight_or_host_head, num_items_in_batch=None, v_chunk=None,
                tied_slot=None):
        weight = weight_or_host_head
        _check_inputs(hidden_states, shift_labels, weight)
        h2d = hidden_states.contiguous().view(-1, hidden_states.shape[-1])
        labels = shift_labels.contiguous().view(-1).to(torch.int64)
        if labels.numel() != h2d.shape[0]:
            raise _lib.LmceError(_lib.LMCE_ERR_INVALID_ARGUMENT, "shift_labels must have one label per token")
        w = weight.contiguous()
        n = h2d.shape[0]
        dev = h2d.device
        with torch.cuda.device(dev):
            if n == 0:
                loss = torch.zeros((), dtype=torch.float32, device=dev)
                nll = torch.zeros(0, dtype=torch.float32, device=dev)
                ent = torch.zeros(0, dtype=torch.float32, device=dev)
                arg = torch.zeros(0, dtype=torch.int64, device=dev)
                lse = nll
                denom = torch.ones(1, dtype=torch.float32, device=dev)
            else:
                parts, n_parts = head_forward_stats(h2d, w, labels)
                loss, nll, ent, arg, lse, denom = head_finish(parts, n_parts, n_parts, 1, labels,
                                                              num_items_in_batch)
        ctx.save_for_backward(h2d, w, labels, lse, denom)
        ctx.orig_shape = hidden_states.shape
        ctx.v_chunk = int(v_chunk) if v_chunk else 0  # 0: the library's default chunk
        ctx.tied_slot = tied_slot
        ctx.mark_non_differentiable(nll, ent, arg)
        return loss, nll, ent, arg

    @staticmethod
    def backward(ctx, grad_loss, _grad_nll=None, _grad_ent=None, _grad_arg=None):
        h2d, w, labels, lse, denom = ctx.saved_tensors
        want_dx = ctx.needs_input_grad[0]
        want_dw = ctx.needs_input_grad[2]
        if not (want_dx or want_dw):
            return None, None, None, None, None, None
        if h2d.shape[0] == 0:
            dx = torch.zeros(ctx.orig_shape, dtype=h2d.dtype, device=h2d.device) if want_dx else None
            dw = torch.zeros_like(w) if want_dw else None
        else:
            with torch.cuda.device(h2d.device):
                dx, dw = head_backward(h2d, w, labels, lse, grad_loss, denom, want_dx, want_dw, ctx.v_chunk)
            if dx is not None:
                dx = dx.view(ctx.orig_shape)
        if dw is not None and ctx.tied_slot is not None:
            # tied input embedding: its backward adds into this buffer and returns the sum; a
            # second head on the same slot in one backward pass adds to what is parked
            if ctx.tied_slot.dw is None:
                ctx.tied_slot.dw = dw
            else:
                ctx.tied_slot.dw.add_(dw)
            dw = None
        return dx, None, dw, None, None, None


def chunked_lm_head(hidden_states, shift_labels, weight_or_host_head, num_items_in_batch=None,
                    v_chunk: int | None = None, tied_slot=None):
    """Drop-in for ``solution.ops.chunked_lm_head`` (ops.py:342-349).

    ``v_chunk`` is the vocab chunk of the gradient pass; ``None`` (the default) lets the
    library size it (for the CTA-pair kernel gradient buffers of ~90 MiB, 4096..20480
    vocab rows); an explicit value is used as given. ``tied_slot`` (a
    ``rus_b200.tied.TiedGradSlot`` shared with ``tied_embedding``) hands dW to the tied
    input embedding's backward, which adds its own gradient into the same buffer."""
    return FusedChunkedLMHeadFn.apply(hidden_states, shift_labels, weight_or_host_head, num_items_in_batch,
                                      v_chunk, tied_slot)
