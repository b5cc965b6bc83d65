"""
The oracle against the reference's own outputs (tests/golden/reference_kat.npz,
made by tests/golden/make_golden.py from src/verifier.py of the reference),
plus planted-mistake checks that the comparison metrics catch errors.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ref


def test_golden_tolerances_are_the_references(golden):
    # matmul, softmax, reduction, layernorm, attention (src/verifier.py:47-53)
    assert list(golden["tolerances"]) == [1e-3, 1e-5, 1e-3, 1e-4, 1e-3]


def test_softmax_oracle_matches_reference(golden):
    x = ref.kat_pattern(64).reshape(4, 16)
    y = ref.softmax_ref(x)
    assert ref.max_abs_diff(y, golden["softmax_4x16"]) <= 1e-7
    assert np.allclose(y.sum(axis=1), 1.0, rtol=1e-12)


def test_layernorm_oracle_matches_reference(golden):
    x = ref.kat_pattern(64).reshape(4, 16)
    y = ref.layernorm_ref(x, np.ones(16), np.zeros(16), 1e-5)
    assert ref.max_abs_diff(y, golden["layernorm_4x16"]) <= 1e-6


def test_matmul_oracle_matches_reference(golden):
    A, B = ref.kat_matmul_inputs(64)
    C = ref.matmul_ref(A, B)
    assert ref.max_abs_diff(C, golden["matmul_N64"]) <= 1e-5
    # transpose_b: B holds Bt
    assert np.array_equal(ref.matmul_ref(A, np.ascontiguousarray(B.T), transpose_b=True), C)


def test_attention_oracle_matches_reference(golden):
    Q, K, V = ref.kat_attention_inputs(512, 64)
    O = ref.attention_ref(Q, K, V)
    assert ref.max_abs_diff(O, golden["attention_S512_D64"]) <= 1e-5


@pytest.mark.parametrize("blk", [64, 128, 192, 256])
def test_reduction_partials_match_reference_bitwise(golden, blk):
    x = ref.kat_pattern(256)
    parts = ref.reduction_partials_ref(x, blk)
    assert np.array_equal(parts, golden[f"reduction_N256_blk{blk}"])
    assert abs(parts.astype(np.float64).sum() - ref.reduce_sum_ref(x)) <= 1e-5


def test_reference_compare_probe(golden):
    d, ok = golden["compare_probe"]
    assert d == pytest.approx(ref.max_abs_diff(np.array([1.0, 2.0]), np.array([1.0, 2.5])))
    assert ok == 0.0


def test_causal_attention_first_row_is_v0():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 3, 16, 8)) for _ in range(3))
    o = ref.attention_ref(q, k, v, causal=True)
    assert np.allclose(o[..., 0, :], v[..., 0, :])
    # last row sees every key: equals the non-causal last row
    assert np.allclose(o[..., -1, :], ref.attention_ref(q, k, v)[..., -1, :])


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0, -0.0], np.float32)
    b = ref.bf16_bits_from_f32(x)
    back = ref.f32_from_bf16_bits(b)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -8)
    # exactly representable values round-trip
    assert np.array_equal(ref.f32_from_bf16_bits(ref.bf16_bits_from_f32(back)), back)
    # ties round to even: 1 + 2^-8 lies halfway between bf16 1.0 and 1.0078125
    assert ref.f32_from_bf16_bits(ref.bf16_bits_from_f32(np.array([1.0 + 2.0 ** -8], np.float32)))[0] == 1.0


# --- planted mistakes: a wrong oracle output must fail the stated budgets ----------

def test_planted_softmax_error_is_caught(golden):
    y = ref.softmax_ref(ref.kat_pattern(64).reshape(4, 16))
    bad = y.copy()
    bad[2, 5] *= 1.0 + 5e-5
    assert ref.normwise_rel_err(bad, y) > 1e-6
    assert ref.max_abs_diff(bad, golden["softmax_4x16"]) <= 1e-5  # the reference's max-abs budget misses it
    assert not np.all(np.abs(bad - y) <= 1e-5 * np.abs(y) + 1e-12)  # the elementwise budget catches it


def test_planted_reduction_error_is_caught():
    x = ref.kat_pattern(100000)
    s = ref.reduce_sum_ref(x)
    assert abs((s + 2e-4 * abs(s)) - s) / abs(s) > 1e-4


def test_normwise_metric_shape_mismatch():
    assert ref.normwise_rel_err(np.zeros(3), np.ones(3)) == 1.0
    assert ref.normwise_rel_err(np.zeros(0), np.zeros(0)) == 0.0


@pytest.mark.parametrize("causal", [False, True])
def test_attention_rows_ref_matches_full(causal):
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((300, 64)) for _ in range(3))
    full = ref.attention_ref(q, k, v, 0.125, causal)
    rows = np.array([0, 1, 5, 100, 255, 256, 299])
    assert np.allclose(ref.attention_rows_ref(q, k, v, rows, 0.125, causal), full[rows], rtol=1e-12, atol=1e-14)
