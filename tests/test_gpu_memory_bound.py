"""
GPU parity of the memory-bound families (softmax, LayerNorm, reduction)
against the oracle and the reference's own golden outputs, through the C ABI.

Tolerances (written here, per family):
  softmax    normwise max|y-ref|/max|ref| <= 1e-5 and elementwise
             |y-ref| <= 1e-5*|ref| + 1e-12
  layernorm  normwise <= 1e-5 and elementwise |y-ref| <= 1e-5*|ref| + 2e-6
  reduction  |s-ref|/|ref| <= 1e-4 (ref = fp64 sum), bitwise deterministic
The reference's own max-abs budgets (softmax 1e-5, layernorm 1e-4,
reduction 1e-3; src/verifier.py:47-53) are checked on its known-answer inputs.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import kt_lib  # noqa: E402
import kt_ops  # noqa: E402
import workloads  # noqa: E402
from oracle import ref  # noqa: E402


def to_dev(a: np.ndarray, dev, offset: int = 0) -> torch.Tensor:
    """Copy to the device; offset > 0 places the data `offset` elements into a
    larger allocation so the tensor's address is not 16-byte aligned."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a)
    if offset == 0:
        return t.to(dev)
    base = torch.empty(a.size + offset, dtype=t.dtype, device=dev)
    view = base[offset:offset + a.size].view(a.shape)
    view.copy_(t)
    return view


def softmax_ok(y, x):
    want = ref.softmax_ref(x)
    assert ref.normwise_rel_err(y, want) <= 1e-5
    assert np.all(np.abs(y - want) <= 1e-5 * np.abs(want) + 1e-12)


def layernorm_ok(y, x, g, b, eps):
    want = ref.layernorm_ref(x, g, b, eps)
    assert ref.normwise_rel_err(y, want) <= 1e-5
    assert np.all(np.abs(y - want) <= 1e-5 * np.abs(want) + 2e-6)


# ---------------------------------------------------------------------------
# Known-answer inputs of the reference verifier, against its own outputs
# ---------------------------------------------------------------------------

def test_softmax_reference_kat(dev, lib, golden):
    x = ref.kat_pattern(64).reshape(4, 16)
    y = kt_ops.softmax(to_dev(x, dev), lib=lib).cpu().numpy()
    assert ref.max_abs_diff(y, golden["softmax_4x16"]) <= 1e-5
    softmax_ok(y, x)


def test_layernorm_reference_kat(dev, lib, golden):
    x = ref.kat_pattern(64).reshape(4, 16)
    g = np.ones(16, np.float32)
    b = np.zeros(16, np.float32)
    y = kt_ops.layernorm(to_dev(x, dev), to_dev(g, dev), to_dev(b, dev), 1e-5, lib=lib).cpu().numpy()
    assert ref.max_abs_diff(y, golden["layernorm_4x16"]) <= 1e-4
    layernorm_ok(y, x, g, b, 1e-5)


@pytest.mark.parametrize("blk", [64, 128, 192, 256])
def test_reduction_reference_kat(dev, lib, golden, blk):
    x = ref.kat_pattern(256)
    s = float(kt_ops.reduce_sum(to_dev(x, dev), lib=lib).item())
    # the reference checks per-block partials; their total is the full sum
    partials = golden[f"reduction_N256_blk{blk}"].astype(np.float64)
    assert abs(s - partials.sum()) <= 1e-3
    # float4 groups are summed in fp32 before the fp64 accumulation
    assert abs(s - ref.reduce_sum_ref(x)) <= 1e-6 * max(1.0, abs(s))


# ---------------------------------------------------------------------------
# Softmax
# ---------------------------------------------------------------------------

SOFTMAX_SHAPES = [(1, 1), (1, 5), (3, 17), (7, 33), (4, 512), (5, 513), (2, 1000), (6, 1028),
                  (257, 4096), (3, 4097), (2, 4099), (1, 20000), (2, 40000), (4096, 4096)]


@pytest.mark.parametrize("rows,cols", SOFTMAX_SHAPES)
def test_softmax_shapes(dev, lib, rows, cols):
    x = workloads.make_inputs("softmax", d={"rows": rows, "cols": cols}, seed=rows * 7919 + cols)["x"]
    y = kt_ops.softmax(to_dev(x, dev), lib=lib).cpu().numpy()
    softmax_ok(y, x)


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_softmax_unaligned(dev, lib, offset):
    x = workloads.make_inputs("softmax", d={"rows": 33, "cols": 4096}, seed=offset)["x"]
    xd = to_dev(x, dev, offset)
    y = kt_ops.softmax(xd, lib=lib).cpu().numpy()
    softmax_ok(y, x)


def test_softmax_large_magnitude(dev, lib):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 4096)) * 30.0 + 1e4).astype(np.float32)
    y = kt_ops.softmax(to_dev(x, dev), lib=lib).cpu().numpy()
    softmax_ok(y, x)
    assert np.allclose(y.sum(axis=1), 1.0, rtol=1e-5)


def test_softmax_empty_and_errors(dev, lib):
    for shape in ((0, 16), (16, 0)):
        x = torch.empty(shape, dtype=torch.float32, device=dev)
        kt_ops.softmax(x, lib=lib)
    with pytest.raises(kt_lib.KtError) as ei:
        lib.softmax_f32(0, 0, 4, 16)
    assert ei.value.status == kt_lib.KT_ERR_ARG
    with pytest.raises(kt_lib.KtError) as ei:
        lib.softmax_f32(0, 0, -1, 16)
    assert ei.value.status == kt_lib.KT_ERR_ARG


def test_softmax_config_size_deterministic(dev, lib):
    inp = workloads.make_inputs("softmax", "config")
    xd = to_dev(inp["x"], dev)
    y1 = kt_ops.softmax(xd, lib=lib)
    y2 = kt_ops.softmax(xd, lib=lib)
    assert torch.equal(y1, y2)
    softmax_ok(y1.cpu().numpy(), inp["x"])


# ---------------------------------------------------------------------------
# LayerNorm
# ---------------------------------------------------------------------------

LN_SHAPES = [(1, 1), (1, 7), (3, 17), (4, 512), (5, 513), (9, 1000), (513, 4096), (3, 4097),
             (1, 20000), (2, 40000), (16384, 4096)]


@pytest.mark.parametrize("rows,cols", LN_SHAPES)
def test_layernorm_shapes(dev, lib, rows, cols):
    inp = workloads.make_inputs("layernorm", d={"rows": rows, "cols": cols}, seed=rows * 31 + cols)
    y = kt_ops.layernorm(to_dev(inp["x"], dev), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev),
                         inp["eps"], lib=lib).cpu().numpy()
    layernorm_ok(y, inp["x"], inp["gamma"], inp["beta"], inp["eps"])


def test_layernorm_unaligned_and_offset_mean(dev, lib):
    inp = workloads.make_inputs("layernorm", d={"rows": 17, "cols": 4096}, seed=3)
    x = (inp["x"] * 0.01 + 100.0).astype(np.float32)  # large mean, small spread
    y = kt_ops.layernorm(to_dev(x, dev, 1), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev),
                         inp["eps"], lib=lib).cpu().numpy()
    want = ref.layernorm_ref(x, inp["gamma"], inp["beta"], inp["eps"])
    # the mean of 100 ± 0.01·N(0,1) cancels ~4 decimal digits of every x in fp32
    assert ref.normwise_rel_err(y, want) <= 2e-3


def test_layernorm_constant_rows(dev, lib):
    x = np.full((8, 4096), 3.25, np.float32)
    g = np.ones(4096, np.float32)
    b = np.full(4096, 0.5, np.float32)
    y = kt_ops.layernorm(to_dev(x, dev), to_dev(g, dev), to_dev(b, dev), 1e-5, lib=lib).cpu().numpy()
    assert np.array_equal(y, np.full_like(x, 0.5))


def test_layernorm_errors(dev, lib):
    with pytest.raises(kt_lib.KtError) as ei:
        lib.layernorm_f32(0, 0, 0, 0, 4, 16, 1e-5)
    assert ei.value.status == kt_lib.KT_ERR_ARG
    x = torch.empty((0, 16), dtype=torch.float32, device=dev)
    g = torch.ones(16, device=dev)
    kt_ops.layernorm(x, g, g, lib=lib)


# ---------------------------------------------------------------------------
# Reduction
# ---------------------------------------------------------------------------

RED_SIZES = [0, 1, 2, 3, 4, 5, 7, 255, 256, 257, 1023, 4097, 65537, (1 << 20) + 1, (1 << 22) + 3]


@pytest.mark.parametrize("n", RED_SIZES)
def test_reduction_sizes(dev, lib, n):
    x = workloads.make_inputs("reduction", d={"n": n}, seed=n + 11)["x"]
    out32 = torch.zeros(1, dtype=torch.float32, device=dev)
    s = float(kt_ops.reduce_sum(to_dev(x, dev), out32=out32, lib=lib).item())
    want = ref.reduce_sum_ref(x)
    assert abs(s - want) <= 1e-4 * abs(want) + 1e-9
    assert float(out32.item()) == np.float32(s)


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_reduction_unaligned(dev, lib, offset):
    x = workloads.make_inputs("reduction", d={"n": 100003}, seed=offset)["x"]
    s = float(kt_ops.reduce_sum(to_dev(x, dev, offset), lib=lib).item())
    want = ref.reduce_sum_ref(x)
    assert abs(s - want) <= 1e-4 * abs(want)


def test_reduction_exact_integers(dev, lib):
    # every partial is an exact integer in fp64: the sum must be exact
    x = np.tile(np.array([1.0, 2.0, -1.0, 3.0], np.float32), 1 << 20)
    s = float(kt_ops.reduce_sum(to_dev(x, dev), lib=lib).item())
    assert s == float(x.astype(np.float64).sum())


def test_reduction_config_size(dev, lib):
    x = workloads.make_inputs("reduction", "config")["x"]
    xd = to_dev(x, dev)
    ws = kt_ops.ReduceWorkspace(x.size, dev, lib)
    s1 = kt_ops.reduce_sum(xd, workspace=ws, lib=lib).item()
    s2 = kt_ops.reduce_sum(xd, workspace=ws, lib=lib).item()
    assert s1 == s2  # bitwise deterministic for a fixed grid
    want = ref.reduce_sum_ref(x)
    assert abs(s1 - want) <= 1e-4 * abs(want)


def test_reduction_linearity(dev, lib):
    # size-independent property: sum(a) + sum(b) == sum(concat(a, b)) within the budget
    a = workloads.make_inputs("reduction", d={"n": 3_000_001}, seed=1)["x"]
    b = workloads.make_inputs("reduction", d={"n": 2_000_003}, seed=2)["x"]
    sa = kt_ops.reduce_sum(to_dev(a, dev), lib=lib).item()
    sb = kt_ops.reduce_sum(to_dev(b, dev), lib=lib).item()
    sab = kt_ops.reduce_sum(to_dev(np.concatenate([a, b]), dev), lib=lib).item()
    l1 = np.abs(a).sum(dtype=np.float64) + np.abs(b).sum(dtype=np.float64)
    assert abs((sa + sb) - sab) <= 1e-9 * l1


def test_reduction_errors(dev, lib):
    x = torch.zeros(1024, device=dev)
    out = torch.zeros(1, dtype=torch.float64, device=dev)
    ws_small = torch.empty(8, dtype=torch.uint8, device=dev)
    with pytest.raises(kt_lib.KtError) as ei:
        lib.reduce_sum_f32(x.data_ptr(), 1024, out.data_ptr(), None, ws_small.data_ptr(), 8)
    assert ei.value.status == kt_lib.KT_ERR_ARG
    with pytest.raises(kt_lib.KtError) as ei:
        lib.reduce_sum_f32(x.data_ptr(), 1024, 0, None, ws_small.data_ptr(), 8)
    assert ei.value.status == kt_lib.KT_ERR_ARG


# ---------------------------------------------------------------------------
# Naive baselines and in-process timing
# ---------------------------------------------------------------------------

def test_naive_baselines_match(dev, lib):
    inp = workloads.make_inputs("softmax", d={"rows": 64, "cols": 1024}, seed=9)
    xd = to_dev(inp["x"], dev)
    y = torch.empty_like(xd)
    lib.run("naive_softmax", kt_lib.make_args(in0=xd.data_ptr(), out0=y.data_ptr(), d0=64, d1=1024))
    torch.cuda.synchronize()
    assert ref.normwise_rel_err(y.cpu().numpy(), ref.softmax_ref(inp["x"])) <= 1e-5
    x = workloads.make_inputs("reduction", d={"n": 100000}, seed=3)["x"]
    xd = to_dev(x, dev)
    out = torch.zeros(1, dtype=torch.float64, device=dev)
    ws = torch.empty(1 << 16, dtype=torch.uint8, device=dev)
    args = kt_lib.make_args(in0=xd.data_ptr(), out0=out.data_ptr(), workspace=ws.data_ptr(), ws_bytes=1 << 16,
                            d0=100000)
    lib.run("naive_reduction", args)
    torch.cuda.synchronize()
    assert abs(out.item() - ref.reduce_sum_ref(x)) <= 1e-3 * abs(ref.reduce_sum_ref(x)) + 1e-3


def test_naive_layernorm_matches(dev, lib, golden):
    """The naive LayerNorm baseline (one thread per row, serial fp32 mean and
    variance, as src/kernels/baseline_kernels.cu:110-142) against the oracle,
    on seeded rows with gamma/beta and on the reference's known-answer rows."""
    inp = workloads.make_inputs("layernorm", d={"rows": 96, "cols": 1024}, seed=21)
    xd, gd, bd = to_dev(inp["x"], dev), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev)
    y = torch.empty_like(xd)
    lib.run("naive_layernorm", kt_lib.make_args(in0=xd.data_ptr(), in1=gd.data_ptr(), in2=bd.data_ptr(),
                                                out0=y.data_ptr(), d0=96, d1=1024, f0=inp["eps"]))
    torch.cuda.synchronize()
    want = ref.layernorm_ref(inp["x"], inp["gamma"], inp["beta"], inp["eps"])
    assert ref.normwise_rel_err(y.cpu().numpy(), want) <= 1e-5
    x = ref.kat_pattern(64).reshape(4, 16)
    ones, zeros = np.ones(16, np.float32), np.zeros(16, np.float32)
    xd, gd, bd = to_dev(x, dev), to_dev(ones, dev), to_dev(zeros, dev)
    y = torch.empty_like(xd)
    lib.run("naive_layernorm", kt_lib.make_args(in0=xd.data_ptr(), in1=gd.data_ptr(), in2=bd.data_ptr(),
                                                out0=y.data_ptr(), d0=4, d1=16, f0=1e-5))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert ref.max_abs_diff(got, golden["layernorm_4x16"]) <= golden["tolerances"][3]
    assert ref.normwise_rel_err(got, ref.layernorm_ref(x, ones, zeros, 1e-5)) <= 1e-5
    assert lib.device_error() == 0


def test_kt_time_samples(dev, lib):
    x = workloads.make_inputs("softmax", "config")["x"]
    xd = to_dev(x, dev)
    y = torch.empty_like(xd)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    args = kt_lib.make_args(in0=xd.data_ptr(), out0=y.data_ptr(), d0=4096, d1=4096)
    samples = lib.time("softmax", args, warmup=3, iters=10, flush=flush.data_ptr(), flush_bytes=flush.numel() * 4)
    assert len(samples) == 10 and all(0.0 < s < 50.0 for s in samples)
    softmax_ok(y.cpu().numpy(), x)
    assert lib.device_error() == 0


@pytest.mark.parametrize("fam", ["softmax", "layernorm"])
def test_register_kernel_variant(dev, lib, tmp_path, monkeypatch, fam):
    """The one-row-per-CTA register kernels (stages=0), built as a tuning variant;
    the default library runs the TMA bulk-copy ring for these shapes."""
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    ok, log, so = generator.ensure_variant(fam, {"block_size": 256, "vec_per_thread": 4, "min_blocks": 1,
                                                 "stages": 0})
    assert ok, log
    v = kt_lib.KtLibrary(so)
    for rows, cols in ((257, 4096), (33, 1028), (4096, 4096)):
        inp = workloads.make_inputs(fam, d={"rows": rows, "cols": cols}, seed=rows + cols)
        if fam == "softmax":
            y = kt_ops.softmax(to_dev(inp["x"], dev), lib=v).cpu().numpy()
            softmax_ok(y, inp["x"])
        else:
            y = kt_ops.layernorm(to_dev(inp["x"], dev), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev),
                                 inp["eps"], lib=v).cpu().numpy()
            layernorm_ok(y, inp["x"], inp["gamma"], inp["beta"], inp["eps"])


# ---------------------------------------------------------------------------
# Rows split across a thread-block cluster (DSMEM exchange of partials)
# ---------------------------------------------------------------------------

# wider than one CTA's 4096-float capacity: the default library splits each row
# across a cluster of 2 (8192), 4 (12288, 16384) or 8 (32768) CTAs; 8196 and
# 40000 have no such split and take the two-pass streaming kernel
WIDE = [(37, 8192), (300, 8192), (5, 12288), (19, 16384), (3, 32768), (2, 8196), (2, 40000)]


@pytest.mark.parametrize("rows,cols", WIDE)
def test_wide_rows(dev, lib, rows, cols):
    inp = workloads.make_inputs("layernorm", d={"rows": rows, "cols": cols}, seed=rows * 13 + cols)
    y = kt_ops.softmax(to_dev(inp["x"], dev), lib=lib).cpu().numpy()
    softmax_ok(y, inp["x"])
    y = kt_ops.layernorm(to_dev(inp["x"], dev), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev), inp["eps"],
                         lib=lib).cpu().numpy()
    layernorm_ok(y, inp["x"], inp["gamma"], inp["beta"], inp["eps"])
    assert lib.device_error() == 0


@pytest.mark.parametrize("fam", ["softmax", "layernorm"])
@pytest.mark.parametrize("params", [{"cluster_size": 2}, {"cluster_size": 4, "tma_box": 4096},
                                    {"stages": 3, "tma_box": 4096}])
def test_cluster_and_box_variants(dev, lib, tmp_path, monkeypatch, fam, params):
    """Tuner points of the Blackwell axes, built as variant libraries: rows that
    one CTA could hold split across a cluster of 2 or 4 CTAs, and bulk copies
    cut into 4 KB pieces (the staged ring and the cluster kernel)."""
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    full = {"block_size": 256, "vec_per_thread": 4, "min_blocks": 1, "stages": 3, **params}
    ok, log, so = generator.ensure_variant(fam, full)
    assert ok, log
    v = kt_lib.KtLibrary(so)
    assert v.variant_params().get("cluster_size", 1) == params.get("cluster_size", 1)
    for rows, cols in ((257, 4096), (4, 1024), (3, 2056), (4096, 4096)):
        inp = workloads.make_inputs(fam, d={"rows": rows, "cols": cols}, seed=rows + 3 * cols)
        if fam == "softmax":
            y = kt_ops.softmax(to_dev(inp["x"], dev), lib=v).cpu().numpy()
            softmax_ok(y, inp["x"])
        else:
            y = kt_ops.layernorm(to_dev(inp["x"], dev), to_dev(inp["gamma"], dev), to_dev(inp["beta"], dev),
                                 inp["eps"], lib=v).cpu().numpy()
            layernorm_ok(y, inp["x"], inp["gamma"], inp["beta"], inp["eps"])
    assert v.device_error() == 0
