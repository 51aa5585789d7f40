"""GPU: the head never holds an [N, V] logits-sized buffer. Every allocation made during one
forward + backward (recorded by torch's caching allocator) is below N * V * 2 bytes, except dW,
the [V, H] output the caller asked for."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [64, 880, 2048])
def test_no_logits_sized_allocation(cuda_device, n):
    from rus_b200 import chunked_lm_head

    H, V = 1536, 151936  # the Qwen2.5-1.5B head of configs 1 and 2
    g = torch.Generator(device=cuda_device).manual_seed(n)
    X = torch.randn(n, H, device=cuda_device, generator=g).half().requires_grad_(True)
    W = (torch.randn(V, H, device=cuda_device, generator=g) * 0.02).half().requires_grad_(True)
    y = torch.randint(0, V, (n,), device=cuda_device, generator=g)
    y[torch.rand(n, device=cuda_device, generator=g) < 0.1] = -100
    chunked_lm_head(X, y, W)[0].backward()  # first call: library load and caches
    X.grad = None
    W.grad = None
    torch.cuda.synchronize()
    torch.cuda.memory._record_memory_history(max_entries=100000)
    try:
        loss, *_ = chunked_lm_head(X, y, W)
        loss.backward()
        torch.cuda.synchronize()
        snap = torch.cuda.memory._snapshot()
    finally:
        torch.cuda.memory._record_memory_history(enabled=None)
    sizes = [e["size"] for trace in snap["device_traces"] for e in trace if e["action"] == "alloc"]
    assert sizes, "no allocation recorded"
    limit = n * V * 2
    dw = V * H * 2
    big = [s for s in sizes if s >= limit and not (dw <= s < dw + (2 << 20))]
    assert not big, f"allocations of at least N*V*2 = {limit} bytes: {big}"
