"""Vocab-sharded lm_head CE head over the GPUs of one box (tensor parallel over V).

Rank r of a world of R owns rows ``shard_range(V, r, R)`` of the [V, H] head;
hidden states and labels are replicated. The two exchange steps:

* forward: each rank folds its shard into one 24-byte partial record per token
  (``lmce_fwd_stats`` + ``lmce_stats_reduce``); the records are all-gathered
  (NCCL over NVLink, R x N x 24 bytes) and every rank merges them with
  ``lmce_stats_finish`` into identical lse / nll / entropy / argmax / loss.
* backward: each rank contracts its shard's gradient tile into its local dW
  shard and an fp32 dX contribution; the dX contributions are summed with one
  all-reduce and cast to the input dtype (``lmce_dx_finalize``).

The reference has no multi-GPU path (it pins one T4); this is the B200 build's
addition for the same operator interface.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .ops import V_CHUNK_DEFAULT, _check_inputs, _stream, head_backward, head_finish, head_forward_stats


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


class VocabShardedLMHeadFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden_states, shift_labels, weight_shard, vocab_offset, vocab_size, group,
                num_items_in_batch=None, v_chunk=V_CHUNK_DEFAULT):
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
        ctx.v_chunk = int(v_chunk) if v_chunk else V_CHUNK_DEFAULT
        ctx.mark_non_differentiable(nll, ent, arg)
        return loss, nll, ent, arg

    @staticmethod
    def backward(ctx, grad_loss, *_):
        h2d, w, labels, lse, denom = ctx.saved_tensors
        want_dx = ctx.needs_input_grad[0]
        want_dw = ctx.needs_input_grad[2]
        dx_f32 = None
        with torch.cuda.device(h2d.device):
            if want_dx:
                dx_f32 = torch.zeros(h2d.shape, dtype=torch.float32, device=h2d.device)
            # every rank takes the same collective steps, whatever it needs locally
            _, dw = head_backward(h2d, w, labels, lse, grad_loss, denom, want_dx, want_dw, ctx.v_chunk,
                                  vocab_offset=ctx.vocab_offset, dx_f32=dx_f32)
            dx = None
            if want_dx:
                reduce_dx(dx_f32, ctx.group)
                dx = torch.empty_like(h2d)
                _lib.call("lmce_dx_finalize", dx_f32.data_ptr(), h2d.shape[0], h2d.shape[1],
                          0 if h2d.dtype == torch.float16 else 1, dx.data_ptr(), _stream(h2d.device))
                dx = dx.view(ctx.orig_shape)
        return dx, None, dw, None, None, None, None, None


def sharded_lm_head(hidden_states, shift_labels, weight_shard, vocab_offset: int, vocab_size: int, group=None,
                    num_items_in_batch=None, v_chunk: int = V_CHUNK_DEFAULT):
    """Vocab-parallel ``chunked_lm_head``: same outputs on every rank; dW is the local shard's."""
    return VocabShardedLMHeadFn.apply(hidden_states, shift_labels, weight_shard, vocab_offset, vocab_size, group,
                                      num_items_in_batch, v_chunk)
