"""CPU, world size 2 over gloo: the vocab-sharded head's exchange steps.

The per-shard compute is the oracle's (this runs without a GPU); what is under
test is rus_b200.sharded's shard partition, the record all-gather layout that
``lmce_stats_finish`` consumes (token stride 1, rank stride N, 24-byte records),
the dX all-reduce, and that a rank failing before a collective makes the other
rank's collective end with an error instead of waiting forever.
"""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REC_DTYPE = np.dtype([("m", "<f4"), ("s", "<f4"), ("w", "<f4"), ("best", "<f4"), ("idx", "<i4"), ("zy", "<f4")])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pack(rec: dict) -> torch.Tensor:
    n = len(rec["m"])
    a = np.zeros(n, dtype=REC_DTYPE)
    for k in REC_DTYPE.names:
        a[k] = rec[k]
    return torch.from_numpy(a.view(np.uint8).reshape(n, 24).copy())


def _unpack(buf: np.ndarray) -> dict:
    a = np.ascontiguousarray(buf).view(REC_DTYPE).reshape(-1)
    return {k: a[k].astype(np.float64) if k != "idx" else a[k].astype(np.int64) for k in REC_DTYPE.names}


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        from oracle import lmce_oracle as orc
        from rus_b200.sharded import exchange_records, reduce_dx, shard_range
        from tests.golden import make_golden as mg

        hidden, shift, weight, _, _ = mg.make_case_inputs("bf16_ragged")
        h = hidden.reshape(-1, hidden.shape[-1])
        y = shift.reshape(-1)
        V = weight.shape[0]
        lo, hi = shard_range(V, rank, world)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange (injected)")
        rec = orc.parts_of_shard(h, y, weight[lo:hi], lo)
        gathered = exchange_records(_pack(rec))  # [R, N, 24]
        n = h.shape[0]
        flat = gathered.numpy().reshape(-1, 24)
        # the layout lmce_stats_finish reads: record (t, p) at t*1 + p*N
        recs = [_unpack(flat[p * n:(p + 1) * n]) for p in range(world)]
        fin = orc.finish_np(orc.part_merge_np(recs), y)
        full = orc.finish_np(orc.parts_of_shard(h, y, weight, 0), y)
        ok_stats = all(np.allclose(fin[k], full[k], rtol=1e-5, atol=1e-5) for k in ("lse", "entropy", "nll"))
        ok_arg = bool(np.array_equal(fin["argmax"], full["argmax"]))
        # dX: each rank's fp32 contribution from its shard, summed by the all-reduce
        ref = orc.eager_head(hidden, shift, weight, grad_mode="fp32")
        z = torch.nn.functional.linear(h, weight).float()  # logits rounded to the input dtype, as the oracle
        p = torch.softmax(z, -1)
        valid = y != -100
        g = p.clone()
        g[valid.nonzero().squeeze(-1), y[valid]] -= 1.0
        g[~valid] = 0
        g /= ref["denom"]
        dx_part = (g[:, lo:hi] @ weight[lo:hi].float()).contiguous()
        reduce_dx(dx_part)
        ok_dx = orc.rel_l2(dx_part, ref["dX"]) < 1e-5
        q.put((rank, ok_stats and ok_arg and ok_dx, ""))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, ok, msg = q.get(timeout=120)
        results[rank] = (ok, msg)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_sharded_exchange_world2():
    res = _run(2, "ok")
    for rank, (ok, msg) in res.items():
        assert ok, f"rank {rank}: {msg}"


def test_rank_failure_surfaces_as_error():
    res = _run(2, "fail")
    assert not res[1][0] and "injected" in res[1][1]
    ok0, msg0 = res[0]
    assert not ok0, "rank 0 must not succeed when its peer never joins the exchange"
    assert msg0, "rank 0 must end with an error, not hang"


def test_shard_range_partitions_vocab():
    from rus_b200.sharded import shard_range

    for V in (151936, 152064, 128256, 4099):
        for world in (1, 2, 4, 8):
            spans = [shard_range(V, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == V
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 0, 8)


def test_exchange_capacity_grows_geometrically():
    """The fused exchange's buffers keep their capacity for calls that fit and grow to at least
    1.5x when outgrown, so a run whose token counts vary reallocates O(log) times."""
    from rus_b200.sharded import NvlsDxExchange, exchange_capacity

    assert exchange_capacity(700) == 1024
    assert exchange_capacity(300, 1024) == 1024
    assert exchange_capacity(1024, 1024) == 1024
    assert exchange_capacity(1025, 1024) == 2048
    assert exchange_capacity(1500, 2048) == 2048
    assert exchange_capacity(5000, 2048) == 5120
    cap, grows = 0, 0
    for n in list(range(100, 40000, 37)):
        new = exchange_capacity(n, cap)
        assert new >= n and new % 1024 == 0
        grows += new != cap
        cap = new
    assert grows <= 10
    # flag words of (row block m, rank, column tile) do not depend on N: a smaller call's flags
    # are the leading words of a larger allocation's
    assert NvlsDxExchange.flag_bytes(300, 1536, 8) <= NvlsDxExchange.flag_bytes(2048, 1536, 8)


def test_fused_exchange_rule():
    """When the vocab-sharded backward sums dX inside its kernel (NVLink SHARP) rather than with
    an NCCL all-reduce afterwards: from 32 MiB of fp32 dX, or in groups of 8 GPUs at any size
    (measured on B200: at 2048 tokens, H = 1536, the fused sum wins at 8 GPUs and ties at 2 and 4);
    LMCE_NVLS=0 / 1 override it."""
    from rus_b200.sharded import NVLS_MIN_DX_BYTES, wants_fused_exchange

    assert NVLS_MIN_DX_BYTES == 32 << 20
    small, large = (2048, 1536), (9434, 3584)  # 12.6 MB and 135 MB of fp32 dX
    assert not wants_fused_exchange(*small, world=2)
    assert not wants_fused_exchange(*small, world=4)
    assert wants_fused_exchange(*small, world=8)
    assert all(wants_fused_exchange(*large, world=w) for w in (2, 4, 8))
    assert wants_fused_exchange(8192, 1024, world=2)  # exactly 32 MiB
    assert not wants_fused_exchange(8191, 1024, world=2)
    assert wants_fused_exchange(*small, world=2, mode="1")
    assert not wants_fused_exchange(*large, world=8, mode="0")
