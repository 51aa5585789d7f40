"""GPU: the no-allocation forward entry point (lmce_forward_noalloc).

Some callers cannot allocate device memory — a plugin inside a runtime that owns
every device allocation, a foreign-language binding that can only hand over
tensor pointers, a serving loop that forbids allocation after warm-up. For them
the library keeps its per-token partial records in a fixed 8 MiB device array of
its own. This test calls that entry point through the C ABI twice in a row, with
different inputs, and checks each result against the regular entry points
(lmce_fwd_stats into a caller buffer + lmce_stats_finish) at the tolerances the
other parity tests use; it also runs a token count large enough that the entry
point must use fewer vocab slabs than the regular path to fit the array, and
checks that a call after the first allocates no device memory. The file is named
so pytest collects it last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from rus_b200 import _lib

pytestmark = pytest.mark.gpu

NAN = float("nan")  # num_items not given
DT = {torch.float16: _lib.LMCE_DTYPE_F16, torch.bfloat16: _lib.LMCE_DTYPE_BF16}


def _outputs(n, dev):
    return dict(lse=torch.empty(n, device=dev), nll=torch.empty(n, device=dev), ent=torch.empty(n, device=dev),
                arg=torch.empty(n, dtype=torch.int64, device=dev), loss=torch.empty(1, device=dev),
                denom=torch.empty(1, device=dev))


def _regular(lib, X, W, y, stream):
    n, h = X.shape
    v = W.shape[0]
    parts_n = lib.lmce_fwd_num_parts(n, v)
    parts = torch.empty(n * parts_n * _lib.PART_BYTES, dtype=torch.uint8, device=X.device)
    o = _outputs(n, X.device)
    _lib.check(lib.lmce_fwd_stats(X.data_ptr(), W.data_ptr(), y.data_ptr(), n, h, v, 0, DT[X.dtype],
                                  parts.data_ptr(), parts_n, stream))
    _lib.check(lib.lmce_stats_finish(parts.data_ptr(), parts_n, parts_n, 1, y.data_ptr(), n, None, NAN,
                                     o["lse"].data_ptr(), o["nll"].data_ptr(), o["ent"].data_ptr(),
                                     o["arg"].data_ptr(), o["loss"].data_ptr(), o["denom"].data_ptr(), stream))
    return o


def _noalloc(lib, X, W, y, stream, o=None):
    n, h = X.shape
    v = W.shape[0]
    o = _outputs(n, X.device) if o is None else o
    _lib.check(lib.lmce_forward_noalloc(X.data_ptr(), W.data_ptr(), y.data_ptr(), n, h, v, DT[X.dtype], None, NAN,
                                        o["lse"].data_ptr(), o["nll"].data_ptr(), o["ent"].data_ptr(),
                                        o["arg"].data_ptr(), o["loss"].data_ptr(), o["denom"].data_ptr(), stream))
    return o


def _inputs(seed, n, h, v, dtype, dev):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(n, h, generator=g).to(dtype).to(dev)
    W = (torch.randn(v, h, generator=g) * (2.0 / h ** 0.5)).to(dtype).to(dev)
    y = torch.randint(0, v, (n,), generator=g)
    y[torch.rand(n, generator=g) < 0.2] = -100
    return X, W, y.to(dev)


def _assert_close(a, b):
    for k in ("lse", "nll", "loss", "denom"):
        ref = b[k].double()
        assert ((a[k].double() - ref).abs() <= 1e-3 * torch.clamp(ref.abs(), min=1.0)).all(), k
    ent_ref = b["ent"].double()
    assert ((a["ent"].double() - ent_ref).abs() <= 1e-3 * torch.clamp(ent_ref.abs(), min=1.0)).all()
    assert torch.equal(a["arg"], b["arg"])


def test_noalloc_forward_matches_regular_entry_points_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    cases = [(101, 2048, 1536, 151936, torch.float16), (202, 700, 256, 9000, torch.bfloat16)]
    for seed, n, h, v, dtype in cases:  # two calls in a row, different shapes and contents
        X, W, y = _inputs(seed, n, h, v, dtype, dev)
        got = _noalloc(lib, X, W, y, stream)
        ref = _regular(lib, X, W, y, stream)
        torch.cuda.synchronize()
        assert _lib.device_error(reset=True) == 0
        _assert_close(got, ref)


def test_noalloc_rejects_sizes_beyond_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    too_many = (8 << 20) // _lib.PART_BYTES + 1
    rc = lib.lmce_forward_noalloc(16, 16, 16, too_many, 64, 100, 0, None, NAN, 16, 16, 16, 16, 16, 16, None)
    assert rc == _lib.LMCE_ERR_INVALID_ARGUMENT
    assert b"no-allocation scratch" in ctypes.string_at(lib.lmce_last_error())


def test_noalloc_caps_vocab_slabs_to_fit_the_scratch():
    """Tens of thousands of tokens with a small head: the regular path would write more
    n_tokens x slabs records than the 8 MiB array holds, so the entry point merges fewer,
    longer vocab slabs per token; the results must not change."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    n, h, v = 60000, 64, 4096
    cap = (8 << 20) // _lib.PART_BYTES // n
    assert lib.lmce_fwd_num_parts(n, v) > cap, "this shape must take the slab-capping branch"
    X, W, y = _inputs(303, n, h, v, torch.float16, dev)
    got = _noalloc(lib, X, W, y, stream)
    ref = _regular(lib, X, W, y, stream)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == 0
    _assert_close(got, ref)


def test_noalloc_call_allocates_no_device_memory():
    """After a first call on the device (which looks up the array's address and loads the
    kernels), a call changes neither the caching allocator's counters nor the device's free
    memory: it runs without any allocation."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    X, W, y = _inputs(404, 1500, 512, 20000, torch.bfloat16, dev)
    o = _outputs(X.shape[0], dev)
    _noalloc(lib, X, W, y, stream, o)  # first call on this shape
    torch.cuda.synchronize()
    count0 = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
    free0 = torch.cuda.mem_get_info(dev)[0]
    _noalloc(lib, X, W, y, stream, o)
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0) == count0
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert _lib.device_error(reset=True) == 0
