"""
The C ABI without a GPU: the library loads, exports every function that
include/kt_abi.h declares, and rejects bad arguments with KT_ERR_ARG before
touching the device. A generated tuning variant exports the same symbols.
"""

from __future__ import annotations

import ctypes
import json
import re
from pathlib import Path

import pytest

import kt_lib

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_functions() -> set[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(kt_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_the_binding_surface():
    names = declared_functions()
    assert set(kt_lib.EXPORTED_SYMBOLS) <= names, set(kt_lib.EXPORTED_SYMBOLS) - names


def test_library_exports_every_declared_function(lib):
    missing = kt_lib.missing_symbols(lib.path, sorted(declared_functions()))
    assert missing == []


def test_version_and_params(lib):
    assert lib.version() == 1
    assert isinstance(lib.variant_params(), dict)


def test_null_and_negative_arguments_are_rejected(lib):
    checks = [
        lambda: lib.softmax_f32(0, 0, 4, 16),
        lambda: lib.softmax_f32(0, 0, -1, 16),
        lambda: lib.layernorm_f32(0, 0, 0, 0, 4, 16, 1e-5),
        lambda: lib.layernorm_f32(1 << 20, 1 << 20, 1 << 20, 1 << 20, 4, 16, -1.0),
        lambda: lib.reduce_sum_f32(0, 16, 0, None, 0, 0),
        lambda: lib.reduce_sum_f32(0, -5, 1 << 20, None, 1 << 20, 1 << 20),
        lambda: lib.gemm_f32(0, 0, 0, 8, 8, 8, False, kt_lib.KT_GEMM_FFMA),
        lambda: lib.gemm_f32(0, 0, 0, -8, 8, 8, False, kt_lib.KT_GEMM_FFMA),
        lambda: lib.gemm_f32(1 << 20, 1 << 20, 1 << 20, 8, 8, 8, False, 7),
        lambda: lib.fa_fwd_bf16(0, 0, 0, 0, 1, 1, 128, 128, 0.1, False),
        # cross-GPU sum: bad world / rank / epoch / exchange table, all refused before any CUDA call
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [], 0, 0, 1),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [1 << 20] * 9, 0, 9, 1),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [1 << 20] * 2, 2, 2, 1),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [1 << 20] * 2, 0, 2, 0),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [1 << 20, 0], 0, 2, 1),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 1 << 20, None, 1 << 20, 1 << 16, [1 << 20, 8], 0, 2, 1),
        lambda: lib.reduce_sum_f32_xrank(1 << 20, 16, 0, None, 1 << 20, 1 << 16, [], 0, 1, 1),
    ]
    for fn in checks:
        with pytest.raises(kt_lib.KtError) as ei:
            fn()
        assert ei.value.status in (kt_lib.KT_ERR_ARG, kt_lib.KT_ERR_UNSUPPORTED), ei.value
        assert ei.value.message


def test_kt_run_and_time_reject_bad_ops(lib):
    args = kt_lib.make_args()
    with pytest.raises(kt_lib.KtError) as ei:
        lib.run(999, args)
    assert ei.value.status == kt_lib.KT_ERR_ARG
    rc = lib.symbol("kt_time")(1, None, 0, 1, None, 0, None, None)
    assert rc == kt_lib.KT_ERR_ARG


def test_empty_shapes_are_no_ops(lib):
    # zero-sized problems return before any CUDA call
    lib.softmax_f32(0, 0, 0, 16)
    lib.layernorm_f32(0, 0, 0, 0, 16, 0, 1e-5)
    lib.gemm_f32(0, 0, 0, 0, 8, 8, False, kt_lib.KT_GEMM_FFMA)


def test_last_error_is_thread_local(lib):
    import threading
    with pytest.raises(kt_lib.KtError):
        lib.softmax_f32(0, 0, -1, 1)
    seen = {}

    def other():
        seen["msg"] = lib.last_error()
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert "negative" in lib.last_error()


def test_generated_variant_builds_and_exports(tmp_path, monkeypatch):
    monkeypatch.setenv("KT_RESULTS_DIR", str(tmp_path))
    import generator
    params = {"block_size": 128, "vec_per_thread": 8, "min_blocks": 2}
    ok, log, so = generator.ensure_variant("softmax", params)
    assert ok, log
    assert "registers" in log  # ptxas -v report is captured
    assert kt_lib.missing_symbols(so, sorted(declared_functions())) == []
    v = kt_lib.KtLibrary(so)
    meta = v.variant_params()
    assert meta["kernel"] == "softmax" and meta["block_size"] == 128
    with pytest.raises(kt_lib.KtError) as ei:
        v.layernorm_f32(1 << 20, 1 << 20, 1 << 20, 1 << 20, 4, 16, 1e-5)
    assert ei.value.status == kt_lib.KT_ERR_UNSUPPORTED


def test_nvcc_failure_is_reported(tmp_path):
    import build as kt_build
    bad = tmp_path / "bad.cu"
    bad.write_text('#include "kt_entry.cuh"\nthis is not C++;\n')
    ok, log = kt_build.compile_shared(bad, tmp_path / "bad.so")
    assert not ok and "error" in log.lower()
    assert not (tmp_path / "bad.so").exists()
