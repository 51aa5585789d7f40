"""Vocab-sharded lm_head CE head over the GPUs of one box (tensor parallel over V).

Rank r of a world of R owns rows ``shard_range(V, r, R)`` of the [V, H] head;
hidden states and labels are replicated. The two exchange steps:

* forward: each rank folds its shard into one 24-byte partial record per token
  (``lmce_fwd_stats`` + ``lmce_stats_reduce``); the records are all-gathered
  (NCCL over NVLink, R x N x 24 bytes) and every rank merges them with
  ``lmce_stats_finish`` into identical lse / nll / entropy / argmax / loss.
* backward: each rank contracts its shard's gradient tile into its local dW
  shard and an fp32 dX contribution, which is summed over the ranks and cast to
  the input dtype (``lmce_dx_finalize``). By default one NCCL all-reduce sums
  the fp32 contributions. With ``LMCE_NVLS=1``, on GPUs that share an NVLink
  switch with multicast (NVLS) support, the sum is fused into the backward
  kernel instead: the last vocab chunk's dX tiles are added into a symmetric
  multicast buffer with ``multimem.red`` as they finish (``lmce_backward_nvls``).
  dX rows are final only once the last vocab chunk is done, so that sum runs at
  the end of the kernel with little compute left to hide it; at the config-2
  shape on 8 GPUs NCCL's all-reduce is faster (4.03 vs 4.66 ms per step), which
  is why the fused path is opt-in.

The reference has no multi-GPU path (it pins one T4); this is the B200 build's
addition for the same operator interface.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import _lib
from .ops import _check_inputs, _stream, head_backward, head_backward_nvls, head_finish, head_forward_stats


def shard_range(vocab_size: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the vocab rows rank ``rank`` owns; shards differ by at most one row."""
    if not (0 <= rank < world) or vocab_size < world:
        raise ValueError(f"cannot split V={vocab_size} over {world} ranks (rank {rank})")
    return vocab_size * rank // world, vocab_size * (rank + 1) // world


def exchange_records(record: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-token records [N, 24] (uint8) into [R, N, 24]; the merge reads
    record (token t, rank p) at t * 1 + p * N (in 24-byte units)."""
    world = dist.get_world_size(group)
    out = torch.empty((world * record.shape[0],) + tuple(record.shape[1:]), dtype=record.dtype,
                      device=record.device)
    dist.all_gather_into_tensor(out, record.contiguous(), group=group)
    return out.view((world,) + tuple(record.shape))


def reduce_dx(dx_f32: torch.Tensor, group=None) -> torch.Tensor:
    dist.all_reduce(dx_f32, op=dist.ReduceOp.SUM, group=group)
    return dx_f32


_NVLS_CACHE: dict = {}


def _group_name(group) -> str:
    return (group if group is not None else dist.group.WORLD).group_name


def nvls_dx_buffer(n: int, h: int, device: torch.device, group=None):
    """(fp32 [n, h] symmetric tensor, handle) with a multicast mapping on every rank of
    the group, or None when the group cannot use NVLink SHARP (the decision is made
    jointly, so every rank takes the same path). Cached per shape. Enabled by LMCE_NVLS=1."""
    if os.environ.get("LMCE_NVLS", "0") != "1" or device.type != "cuda":
        return None
    key = (device.index, _group_name(group), n, h)
    if key in _NVLS_CACHE:
        return _NVLS_CACHE[key]
    buf = None
    ok = 1
    try:
        import torch.distributed._symmetric_memory as symm_mem

        t = symm_mem.empty((n, h), dtype=torch.float32, device=device)
        hdl = symm_mem.rendezvous(t, _group_name(group))
        if int(getattr(hdl, "multicast_ptr", 0)) == 0 or int(getattr(hdl, "offset", 0)) != 0:
            ok = 0
        else:
            buf = (t, hdl)
    except Exception:
        ok = 0
    flag = torch.tensor([ok], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) == 0:
        buf = None
    _NVLS_CACHE[key] = buf
    return buf


class VocabShardedLMHeadFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden_states, shift_labels, weight_shard, vocab_offset, vocab_size, group,
                num_items_in_batch=None, v_chunk=None):
        _check_inputs(hidden_states, shift_labels, weight_shard)
        h2d = hidden_states.contiguous().view(-1, hidden_states.shape[-1])
        labels = shift_labels.contiguous().view(-1).to(torch.int64)
        w = weight_shard.contiguous()
        n = h2d.shape[0]
        world = dist.get_world_size(group)
        with torch.cuda.device(h2d.device):
            parts, n_parts = head_forward_stats(h2d, w, labels, vocab_offset)
            record = torch.empty((n, _lib.PART_BYTES), dtype=torch.uint8, device=h2d.device)
            _lib.call("lmce_stats_reduce", parts.data_ptr(), n_parts, n_parts, 1, n, record.data_ptr(),
                      _stream(h2d.device))
            gathered = exchange_records(record, group)
            loss, nll, ent, arg, lse, denom = head_finish(gathered, world, 1, n, labels, num_items_in_batch)
        ctx.save_for_backward(h2d, w, labels, lse, denom)
        ctx.vocab_offset = int(vocab_offset)
        ctx.group = group
        ctx.orig_shape = hidden_states.shape
        ctx.v_chunk = int(v_chunk) if v_chunk else 0
        ctx.mark_non_differentiable(nll, ent, arg)
        return loss, nll, ent, arg

    @staticmethod
    def backward(ctx, grad_loss, *_):
        h2d, w, labels, lse, denom = ctx.saved_tensors
        want_dx = ctx.needs_input_grad[0]
        want_dw = ctx.needs_input_grad[2]
        dx_f32 = None
        dev = h2d.device
        n, h = h2d.shape
        with torch.cuda.device(dev):
            nvls = nvls_dx_buffer(n, h, dev, ctx.group) if want_dx else None
            if nvls is not None:
                # fused: the kernel adds this rank's dX rows into every rank's copy through the switch
                dx_f32, hdl = nvls
                dx_f32.zero_()
                hdl.barrier(channel=0)  # every rank zeroed before any rank adds
                dw = head_backward_nvls(h2d, w, labels, lse, grad_loss, denom, int(hdl.multicast_ptr), want_dw,
                                        ctx.v_chunk, ctx.vocab_offset)
                hdl.barrier(channel=0)  # every rank's additions have landed
            else:
                if want_dx:
                    dx_f32 = torch.zeros(h2d.shape, dtype=torch.float32, device=dev)
                # every rank takes the same collective steps, whatever it needs locally
                _, dw = head_backward(h2d, w, labels, lse, grad_loss, denom, want_dx, want_dw, ctx.v_chunk,
                                      vocab_offset=ctx.vocab_offset, dx_f32=dx_f32)
                if want_dx:
                    reduce_dx(dx_f32, ctx.group)
            dx = None
            if want_dx:
                dx = torch.empty_like(h2d)
                _lib.call("lmce_dx_finalize", dx_f32.data_ptr(), n, h, 0 if h2d.dtype == torch.float16 else 1,
                          dx.data_ptr(), _stream(dev))
                dx = dx.view(ctx.orig_shape)
        return dx, None, dw, None, None, None, None, None


def sharded_lm_head(hidden_states, shift_labels, weight_shard, vocab_offset: int, vocab_size: int, group=None,
                    num_items_in_batch=None, v_chunk: int | None = None):
    """Vocab-parallel ``chunked_lm_head``: same outputs on every rank; dW is the local shard's."""
    return VocabShardedLMHeadFn.apply(hidden_states, shift_labels, weight_shard, vocab_offset, vocab_size, group,
                                      num_items_in_batch, v_chunk)
