"""
The scratch-free reduction entry point, kt_reduce_sum_f32_noalloc, through the
C ABI on a GPU.

It exists for callers that cannot allocate device memory (host callbacks and
real-time loops where cudaMalloc would block or synchronize, embedders with a
fixed memory budget, FFI callers holding only their input/output buffers):
its scratch is a fixed array inside the library. Two calls in a row, on
different inputs, must each give the same sum as kt_reduce_sum_f32 with a
caller-provided workspace (within the reduction budget of 1e-4 relative; the
kernel and grid are the same, so the results are in fact expected to be
identical). The second call also shows that the shared scratch left by the
first call does not leak into the next result.

This file is collected last, so a run that stops at the first failure has
already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import kt_ops  # noqa: E402
import workloads  # noqa: E402


def _noalloc_fn(lib):
    fn = lib.symbol("kt_reduce_sum_f32_noalloc")
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def test_noalloc_matches_workspace_entry_point_twice(dev, lib):
    """Two calls queued back to back on one stream (no synchronisation between
    them), with different lengths and different output buffers; each result is
    compared with kt_reduce_sum_f32 and with the oracle's fp64 sum."""
    from oracle import ref

    fn = _noalloc_fn(lib)
    stream = torch.cuda.current_stream().cuda_stream
    cases = [((1 << 22) + 3, 101), (1_000_001, 202)]
    xs, outs = [], []
    for n, seed in cases:
        x = workloads.make_inputs("reduction", d={"n": n}, seed=seed)["x"]
        xs.append((x, torch.from_numpy(x).to(dev)))
        outs.append((torch.full((1,), float("nan"), dtype=torch.float64, device=dev),
                     torch.full((1,), float("nan"), dtype=torch.float32, device=dev)))
    torch.cuda.synchronize()
    for call, ((n, _), (_, xd), (o64, o32)) in enumerate(zip(cases, xs, outs)):
        rc = fn(xd.data_ptr(), n, o64.data_ptr(), o32.data_ptr(), stream)
        assert rc == 0, f"call {call}: status {rc}: {lib.last_error()}"
    torch.cuda.synchronize()
    for call, ((x, xd), (o64, o32)) in enumerate(zip(xs, outs)):
        got64 = o64.item()
        want64 = kt_ops.reduce_sum(xd, lib=lib).item()
        oracle = ref.reduce_sum_ref(x)
        assert abs(got64 - want64) <= 1e-4 * abs(want64), (call, got64, want64)
        assert abs(got64 - oracle) <= 1e-4 * abs(oracle), (call, got64, oracle)
        assert float(o32.item()) == float(np.float32(got64))


def test_noalloc_rejects_bad_arguments(dev, lib):
    fn = _noalloc_fn(lib)
    xd = torch.zeros(16, device=dev)
    out64 = torch.zeros(1, dtype=torch.float64, device=dev)
    assert fn(xd.data_ptr(), 16, None, None, None) == 1  # KT_ERR_ARG: null output
    assert fn(xd.data_ptr(), -1, out64.data_ptr(), None, None) == 1  # negative length
    assert fn(xd.data_ptr() + 1, 8, out64.data_ptr(), None, None) == 1  # x not 4-byte aligned
    assert "aligned" in lib.last_error()
