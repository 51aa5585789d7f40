"""GPU, 2 ranks over NCCL: the vocab-sharded head against the single-GPU head.

Runs as spawned child processes, one per GPU (skipped with fewer than 2 GPUs).
NVLS is switched off for the test (NCCL_NVLS_ENABLE=0); a short process-group
timeout bounds every collective.
"""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from oracle import lmce_oracle as orc
        from rus_b200 import chunked_lm_head
        from rus_b200.sharded import shard_range, sharded_lm_head

        g = torch.Generator().manual_seed(99)
        N, H, V = 700, 512, 30011
        X = torch.randn(N, H, generator=g).half().to(dev)
        W = (torch.randn(V, H, generator=g) * 0.05).half().to(dev)
        y = torch.randint(0, V, (N,), generator=g)
        y[torch.rand(N, generator=g) < 0.2] = -100
        y = y.to(dev)
        from rus_b200.sharded import nvls_dx_buffer

        lo, hi = shard_range(V, rank, world)
        xr = X.clone().requires_grad_(True)
        wr = W.clone().requires_grad_(True)
        loss_r, nll_r, ent_r, arg_r = chunked_lm_head(xr, y, wr, None, 4096)
        loss_r.backward()
        ok = True
        msg = ""
        for mode in ("auto", "nccl"):  # auto: NVLink SHARP in-kernel dX sum when the switch supports it
            os.environ["LMCE_NVLS"] = "0" if mode == "nccl" else "1"
            xs = X.clone().requires_grad_(True)
            ws = W[lo:hi].clone().requires_grad_(True)
            for _ in range(2):  # twice: the cached symmetric buffer is reused
                xs.grad = None
                ws.grad = None
                loss, nll, ent, arg = sharded_lm_head(xs, y, ws, lo, V, None, None, 4096)
                loss.backward()
            torch.cuda.synchronize()
            ok &= abs(loss.item() - loss_r.item()) <= 1e-4 * abs(loss_r.item())
            ok &= bool(((nll - nll_r).abs() <= 1e-4 * nll_r.abs().clamp(min=1)).all())
            ok &= bool(((ent - ent_r).abs() <= 1e-4 * ent_r.abs().clamp(min=1)).all())
            ok &= bool(torch.equal(arg, arg_r))
            ok &= orc.rel_l2(xs.grad.float(), xr.grad.float()) < 1e-3
            ok &= orc.rel_l2(ws.grad.float(), wr.grad[lo:hi].float()) < 1e-3
            if mode == "auto":
                msg = "nvls" if nvls_dx_buffer(N, H, dev) is not None else "nccl-fallback"
        q.put((rank, bool(ok), msg))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, False, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


def test_vocab_sharded_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, ok, msg = q.get(timeout=300)
        res[rank] = (ok, msg)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for rank, (ok, msg) in sorted(res.items()):
        assert ok, f"rank {rank}: {msg}"
    print("dX exchange used:", res[0][1])
