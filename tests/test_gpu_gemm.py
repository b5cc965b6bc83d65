"""
GPU parity of the matmul family through the C ABI: the exact fp32 FFMA
kernel and the TF32 tcgen05 kernel, with and without transpose_b, against
the fp64 oracle.

Tolerances: FFMA normwise max|C-ref|/max|ref| <= 1e-5; TF32 normwise <= 1e-3
(the budget for tf32 operands); for TF32 with K < 32 the error is measured
against max(|A|·|B|) instead (oracle.ref.product_scaled_err), since a short
dot product may cancel. On the reference's known-answer inputs
(N=64) the FFMA path also meets the reference's max-abs budget 1e-3
(src/verifier.py:47-53).
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

FFMA, TF32 = kt_lib.KT_GEMM_FFMA, kt_lib.KT_GEMM_TF32
TOL = {FFMA: 1e-5, TF32: 1e-3}


def run(lib, dev, A, B, tb, variant):
    Bd = np.ascontiguousarray(B.T) if tb else B
    C = kt_ops.gemm(torch.from_numpy(A).to(dev), torch.from_numpy(np.ascontiguousarray(Bd)).to(dev),
                    transpose_b=tb, variant=variant, lib=lib)
    torch.cuda.synchronize()
    return C.cpu().numpy()


@pytest.mark.parametrize("variant", [FFMA, TF32])
@pytest.mark.parametrize("tb", [False, True])
def test_gemm_reference_kat(dev, lib, golden, variant, tb):
    A, B = ref.kat_matmul_inputs(64)
    C = run(lib, dev, A, B, tb, variant)
    want = ref.matmul_ref(A, B)
    assert ref.normwise_rel_err(C, want) <= TOL[variant]
    if variant == FFMA:
        assert ref.max_abs_diff(C, golden["matmul_N64"]) <= 1e-3


SHAPES = [(1, 1, 4), (128, 256, 32), (128, 256, 8192), (256, 512, 64), (300, 200, 100), (1000, 1000, 1000),
          (512, 384, 1024), (129, 257, 33), (64, 4, 4), (7, 260, 12)]


@pytest.mark.parametrize("variant", [FFMA, TF32])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_shapes(dev, lib, variant, tb, M, N, K):
    inp = workloads.make_inputs("matmul", d={"M": M, "N": N, "K": K}, seed=M * 7 + N * 3 + K)
    C = run(lib, dev, inp["A"], inp["B"], tb, variant)
    assert C.shape == (M, N)
    if variant == TF32 and K < 32:
        # a dot product of a few terms can cancel to a value far below its
        # products; tf32 rounding is bounded relative to the products
        assert ref.product_scaled_err(C, inp["A"], inp["B"]) <= TOL[variant]
    else:
        assert ref.normwise_rel_err(C, ref.matmul_ref(inp["A"], inp["B"])) <= TOL[variant]
    assert lib.device_error() == 0


def test_gemm_k_zero_gives_zero(dev, lib):
    A = torch.zeros((16, 0), device=dev)
    B = torch.zeros((0, 8), device=dev)
    for v in (FFMA, TF32):
        C = torch.full((16, 8), 7.0, device=dev)
        kt_ops.gemm(A, B, variant=v, out=C, lib=lib)
        torch.cuda.synchronize()
        assert torch.count_nonzero(C).item() == 0


@pytest.mark.parametrize("tb", [False, True])
def test_gemm_tf32_config_size(dev, lib, tb):
    inp = workloads.make_inputs("matmul", "config")
    A, B = inp["A"], inp["B"]
    Ad = torch.from_numpy(A).to(dev)
    Bd = torch.from_numpy(np.ascontiguousarray(B.T) if tb else B).to(dev)
    C1 = kt_ops.gemm(Ad, Bd, transpose_b=tb, variant=TF32, lib=lib)
    C2 = kt_ops.gemm(Ad, Bd, transpose_b=tb, variant=TF32, lib=lib)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)  # deterministic
    rows = np.r_[0:64, 4096:4160, 8128:8192]
    got = C1[torch.from_numpy(rows).to(dev)].cpu().numpy()
    want = ref.matmul_ref(A[rows], B)
    assert ref.normwise_rel_err(got, want) <= 1e-3
    assert lib.device_error() == 0


@pytest.mark.parametrize("tb", [False, True])
def test_gemm_ffma_config_rows(dev, lib, tb):
    inp = workloads.make_inputs("matmul", "config")
    Bh = np.ascontiguousarray(inp["B"].T) if tb else inp["B"]
    C = kt_ops.gemm(torch.from_numpy(inp["A"]).to(dev), torch.from_numpy(Bh).to(dev), transpose_b=tb, variant=FFMA,
                    lib=lib)
    torch.cuda.synchronize()
    rows = np.r_[0:32, 4000:4032, 8160:8192]
    got = C[torch.from_numpy(rows).to(dev)].cpu().numpy()
    assert ref.normwise_rel_err(got, ref.matmul_ref(inp["A"][rows], inp["B"])) <= 1e-5
    assert lib.device_error() == 0


def test_naive_gemm_matches(dev, lib):
    inp = workloads.make_inputs("matmul", d={"M": 100, "N": 70, "K": 50}, seed=4)
    Ad = torch.from_numpy(inp["A"]).to(dev)
    Bd = torch.from_numpy(inp["B"]).to(dev)
    C = torch.empty((100, 70), device=dev)
    lib.run("naive_matmul", kt_lib.make_args(in0=Ad.data_ptr(), in1=Bd.data_ptr(), out0=C.data_ptr(),
                                             d0=100, d1=70, d2=50))
    torch.cuda.synchronize()
    assert ref.normwise_rel_err(C.cpu().numpy(), ref.matmul_ref(inp["A"], inp["B"])) <= 1e-5


def test_two_variant_libraries_in_one_process(dev, lib, tmp_path, monkeypatch):
    """Two different builds loaded side by side keep their own kernel set-up
    (a BN=128, 6-stage TF32 variant next to the default BN=256 library)."""
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    ok, log, so = generator.ensure_variant("matmul", {"bk": 16, "cta_tile": "128x128", "stages": 6})
    assert ok, log
    other = kt_lib.KtLibrary(so)
    inp = workloads.make_inputs("matmul", d={"M": 384, "N": 640, "K": 512}, seed=12)
    want = ref.matmul_ref(inp["A"], inp["B"])
    for L in (lib, other, lib):
        for tb in (False, True):
            C = run(L, dev, inp["A"], inp["B"], tb, TF32)
            assert ref.normwise_rel_err(C, want) <= 1e-3


@pytest.mark.parametrize("tile,stages", [("128x224", 5), ("128x192", 5)])
def test_gemm_tf32_narrower_tiles(dev, lib, tmp_path, monkeypatch, tile, stages):
    """TF32 accumulator tiles of 224 and 192 columns with five pipeline stages
    (tuner axis cta_tile), built as variant libraries: N not a multiple of the
    tile (a partial last tile), ragged and aligned shapes, both B layouts."""
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    ok, log, so = generator.ensure_variant("matmul", {"bk": 16, "cta_tile": tile, "stages": stages})
    assert ok, log
    v = kt_lib.KtLibrary(so)
    for (M, N, K) in ((384, 640, 512), (200, 1000, 96), (1024, 2048, 1024)):
        inp = workloads.make_inputs("matmul", d={"M": M, "N": N, "K": K}, seed=M + N + K)
        want = ref.matmul_ref(inp["A"], inp["B"])
        for tb in (False, True):
            assert ref.normwise_rel_err(run(v, dev, inp["A"], inp["B"], tb, TF32), want) <= 1e-3
    assert v.device_error() == 0


def test_gemm_ffma_packed_variant(dev, lib, tmp_path, monkeypatch):
    """The packed fma.rn.f32x2 FFMA kernel (tuner axis ffma_x2), built as a
    variant library: exact fp32 like the default, on ragged and aligned shapes."""
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    ok, log, so = generator.ensure_variant("matmul", {"variant": "ffma", "bk": 16, "ffma_x2": 1, "min_blocks": 1})
    assert ok, log
    v = kt_lib.KtLibrary(so)
    for (M, N, K) in ((129, 257, 33), (512, 384, 1024), (7, 260, 12)):
        inp = workloads.make_inputs("matmul", d={"M": M, "N": N, "K": K}, seed=M + N + K)
        for tb in (False, True):
            C = run(v, dev, inp["A"], inp["B"], tb, FFMA)
            assert ref.normwise_rel_err(C, ref.matmul_ref(inp["A"], inp["B"])) <= 1e-5
    assert v.device_error() == 0
