"""CPU: the C-ABI library loads, exports exactly what include/lmce.h declares, validates
arguments before touching the GPU, and the product path refuses to run without CUDA."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from rus_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "lmce.h"


def header_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^LMCE_API\s+[\w\s\*]+?\b(lmce_\w+)\s*\(", text, flags=re.M))


def test_library_builds_and_loads():
    from rus_b200 import build

    build.build_library()
    lib = _lib.load()
    assert lib.lmce_abi_version() == 1


def test_exports_every_declared_symbol():
    declared = header_functions()
    assert len(declared) >= 10
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in lmce.h but not exported"
    assert declared == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/lmce.h"


def test_argument_validation_without_gpu():
    lib = _lib.load()
    rc = lib.lmce_fwd_stats(None, None, None, 10, 64, 100, 0, 0, None, 1, None)
    assert rc == _lib.LMCE_ERR_INVALID_ARGUMENT
    assert b"null" in lib.lmce_last_error()
    rc = lib.lmce_backward(1, 1, 1, 1, 10, 100, 100, 0, 0, None, 1, None, None, None, 8192, 16, 1 << 30, None)
    assert rc == _lib.LMCE_ERR_UNSUPPORTED  # hidden_dim not a multiple of 64
    rc = lib.lmce_backward(16, 16, 16, 16, 10, 128, 100, 0, 0, None, 16, None, None, None, 8192, 16, 16, None)
    assert rc == _lib.LMCE_ERR_WORKSPACE
    # the stage-ring probe rejects rings that do not fit shared memory and stages that are not
    # whole pieces of the load kind, before touching a device
    cyc = (ctypes.c_ulonglong * 256)()
    for kind, stage, stages in ((1, 65536, 4), (1, 49152, 4), (0, 8192, 3), (3, 32768, 3), (2, 32768, 9)):
        rc = lib.lmce_probe_tma_pipeline(256, 1024, 1536, kind, stage, stages, 0, 100, cyc, 256, None)
        assert rc == _lib.LMCE_ERR_INVALID_ARGUMENT, (kind, stage, stages)


def test_default_workspace_holds_no_logits_sized_buffer():
    """The backward workspace with the library's default chunk (the op's largest transient
    allocation) stays below an [N, V] buffer of the input dtype for every N >= 64 (below
    that the 256-row padding of the gathered rows and the dX accumulator dominates)."""
    lib = _lib.load()
    for h, v in ((1536, 151936), (896, 151936), (4096, 128256), (128, 5000)):
        for n in (64, 65, 100, 256, 880, 2048, 4096, 11600, 32768):
            ws = lib.lmce_bwd_workspace_bytes(n, h, v, 0)
            assert ws < n * v * 2, (n, h, v, ws)


def test_workspace_sizes_are_bounded():
    lib = _lib.load()
    n, h, v = 2048, 1536, 151936
    ws = lib.lmce_bwd_workspace_bytes(n, h, v, 8192)
    # compacted rows + one vocab-chunk gradient tile + fp32 dX accumulator: far below an [N, V] buffer
    assert ws < 2 * n * v * 2 / 4
    assert ws >= n * 8192 * 2
    assert lib.lmce_bwd_workspace_bytes(0, h, v, 8192) == 0


def test_no_cpu_fallback():
    from rus_b200 import chunked_lm_head

    hidden = torch.randn(4, 64).half()
    weight = torch.randn(100, 64).half()
    labels = torch.randint(0, 100, (4,))
    with pytest.raises(_lib.LmceError):
        chunked_lm_head(hidden, labels, weight)


def test_product_does_not_import_oracle():
    for py in (ROOT / "rus_b200").rglob("*.py"):
        src = py.read_text()
        assert "oracle" not in re.sub(r'""".*?"""', "", src, flags=re.S).replace("# ", ""), py
