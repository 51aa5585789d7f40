"""Vocab-sharded lm_head CE head over the GPUs of one box (tensor parallel over V).

Rank r of a world of R owns rows ``shard_range(V, r, R)`` of the [V, H] head;
hidden states and labels are replicated. The two exchange steps:

* forward: each rank folds its shard into one 24-byte partial record per token
  (``lmce_fwd_stats`` + ``lmce_stats_reduce``); the records are all-gathered
  (NCCL over NVLink, R x N x 24 bytes) and every rank merges them with
  ``lmce_stats_finish`` into identical lse / nll / entropy / argmax / loss.
* backward: each rank contracts its shard's gradient tile into its local dW
  shard and an fp32 dX contribution, which is summed over the ranks. On GPUs
  that share an NVLink switch with multicast (NVLS) support, for dX of at least
  32 MiB in fp32 or groups of at least 8 GPUs (``LMCE_NVLS=1`` forces it, ``0``
  disables it), the sum is fused into the backward kernel (``lmce_backward_nvls``):
  as a row block's last-chunk dX tiles finish on every rank, each rank sums its
  slice of the block's columns over the GPUs through the switch
  (``multimem.ld_reduce``) and stores the result to every GPU's output copy
  (``multimem.st``), while the last two chunks' dW tiles still compute. The
  buffers are torch symmetric memory, kept per hidden size and dtype and grown
  when a call has more tokens than they hold. Otherwise one
  NCCL all-reduce sums the fp32 contributions after the kernel and
  ``lmce_dx_finalize`` casts them to the input dtype. Measured at the config-2 shape
  (backward phase, fused / NCCL, ms per step, one box of B200s): 2048 tokens (dX 12.6 MB)
  on 2, 4 and 8 GPUs 1.098 / 1.086, 0.630 / 0.606 and 0.383 / 0.510; earlier kernels gave,
  per step, 16384 tokens (100 MB) on 8 GPUs 3.58 / 3.90 and 8192 tokens (50 MB) on 4 GPUs
  3.24 / 3.58; hence the rule.

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


class NvlsDxExchange:
    """Symmetric buffers of the fused dX exchange for one (device, group, h, dtype) and up to
    ``capacity`` tokens: the per-row-block flags, this rank's fp32 contribution and the dtype
    output, in one allocation mapped into an NVLink multicast object on every rank of the
    group. Calls with fewer tokens use the leading rows."""

    def __init__(self, buf: torch.Tensor, hdl, n: int, h: int, dtype: torch.dtype, rank: int, world: int):
        self.buf, self.hdl = buf, hdl
        self.capacity = n
        part_off = self.flag_bytes(n, h, world)
        out_off = part_off + _round_up(4 * n * h, 256)
        base, mc = buf.data_ptr(), int(hdl.multicast_ptr)
        self.out_local = buf[out_off:out_off + 2 * n * h].view(dtype).view(n, h)
        self.xch = _lib.DxExchange(partial=base + part_off, partial_mc=mc + part_off, out_mc=mc + out_off,
                                   flags=base, flags_mc=mc, epoch=0, rank=rank, world=world)

    @staticmethod
    def flag_bytes(n: int, h: int, world: int) -> int:
        # one done stamp per rank, then per 256-row block, rank and 256-column dX tile two
        # stamps (the two 128-row blocks of the one-CTA kernel, or the pair kernel's halves)
        return _round_up(4 * (world + 2 * ((n + 255) // 256) * world * ((h + 255) // 256)), 256)

    @classmethod
    def nbytes(cls, n: int, h: int, world: int) -> int:
        return cls.flag_bytes(n, h, world) + _round_up(4 * n * h, 256) + _round_up(2 * n * h, 256)

    def next_epoch(self) -> None:
        self.xch.epoch = self.xch.epoch % 0xFFFFFFFF + 1


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def exchange_capacity(n: int, current: int = 0) -> int:
    """Token capacity of the exchange buffers for a call with n tokens when the group's current
    buffers hold ``current`` (0: none): unchanged while n fits, else the larger of n and 1.5x the
    current capacity, in multiples of 1024 tokens."""
    if 0 < n <= current:
        return current
    return max(_round_up(max(n, 1), 1024), _round_up(current * 3 // 2, 1024))


NVLS_MIN_DX_BYTES = 32 << 20  # fp32 dX size from which the fused exchange beats NCCL's all-reduce
NVLS_MIN_WORLD = 8  # group size from which it wins at any size


def wants_fused_exchange(n: int, h: int, world: int, mode: str = "auto") -> bool:
    """Whether the dX sum of n tokens x h columns over `world` ranks should be fused into the
    backward (before checking that the GPUs support it): LMCE_NVLS mode "0" never, "1" always,
    otherwise from NVLS_MIN_DX_BYTES of fp32 dX or from NVLS_MIN_WORLD ranks."""
    if mode == "0":
        return False
    if mode == "1":
        return True
    return 4 * n * h >= NVLS_MIN_DX_BYTES or world >= NVLS_MIN_WORLD


def nvls_dx_exchange(n: int, h: int, dtype: torch.dtype, device: torch.device, group=None):
    """The group's ``NvlsDxExchange`` for n tokens, or None when the fused exchange is not
    used: LMCE_NVLS=0, or (default) fp32 dX below NVLS_MIN_DX_BYTES in a group of fewer than
    NVLS_MIN_WORLD ranks, or the group cannot use NVLink SHARP (decided jointly, so every rank
    takes the same path). LMCE_NVLS=1 uses it
    whenever the GPUs support it. One buffer per (device, group, h, dtype), reused for any n
    up to its capacity and replaced by one 1.5x larger when n outgrows it (every rank sees
    the same n, so all ranks reallocate together)."""
    if device.type != "cuda" or not wants_fused_exchange(n, h, dist.get_world_size(group),
                                                          os.environ.get("LMCE_NVLS", "auto")):
        return None
    key = (device.index, _group_name(group), h, dtype)
    cached = _NVLS_CACHE.get(key, False)
    if cached is None:
        return None  # the group cannot use NVLink SHARP
    if cached is not False and cached.capacity >= n:
        return cached
    cap = exchange_capacity(n, 0 if cached is False else cached.capacity)
    if cached is not False:
        # every rank's last kernel on the old buffer has finished before any rank frees it
        torch.cuda.synchronize(device)
        dist.barrier(group=group, device_ids=[device.index])
        del _NVLS_CACHE[key]
        cached = None
    state = None
    ok = 1
    try:
        import torch.distributed._symmetric_memory as symm_mem

        world = dist.get_world_size(group)
        buf = symm_mem.empty(NvlsDxExchange.nbytes(cap, h, world), dtype=torch.uint8, device=device)
        hdl = symm_mem.rendezvous(buf, _group_name(group))
        if int(getattr(hdl, "multicast_ptr", 0)) == 0 or int(getattr(hdl, "offset", 0)) != 0:
            ok = 0
        else:
            state = NvlsDxExchange(buf, hdl, cap, h, dtype, dist.get_rank(group), world)
    except Exception:
        ok = 0
    flag = torch.tensor([ok], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) == 0:
        state = None
    else:
        state.buf.zero_()  # flags start at zero on every rank before any rank's first call stamps them
        torch.cuda.synchronize(device)
        dist.barrier(group=group, device_ids=[device.index])
    _NVLS_CACHE[key] = state
    return state


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
            nvls = nvls_dx_exchange(n, h, h2d.dtype, dev, ctx.group) if want_dx else None
            if nvls is not None:
                # fused: the kernel sums dX over the group through the switch into every rank's copy
                # (the kernel returns only once every rank's sums have landed in this rank's copy)
                nvls.next_epoch()
                dw = head_backward_nvls(h2d, w, labels, lse, grad_loss, denom, nvls.xch, want_dw, ctx.v_chunk,
                                        ctx.vocab_offset)
                dx = torch.empty_like(h2d)
                _lib.call("lmce_dx_copy_labelled", nvls.out_local.data_ptr(), labels.data_ptr(), n, h,
                          0 if h2d.dtype == torch.float16 else 1, dx.data_ptr(), _stream(dev))
                return dx.view(ctx.orig_shape), None, dw, None, None, None, None, None
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
