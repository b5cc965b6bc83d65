"""
kt_lib.py — the thin ctypes shim over the C ABI in include/kt_abi.h.

The reference talks to each compiled variant through a subprocess and parses
its stdout (`SAMPLE`/`TIMING`/`VERIFY_OUTPUT` lines; src/benchmark.py:135-187,
src/verifier.py:531-540). Here a variant is a shared library loaded into the
tuner's own process; every call returns a status code that this module turns
into a `KtError` carrying the library's thread-local error text.

There is no CPU fallback: if the library cannot be loaded, `load()` raises.
"""

from __future__ import annotations

import ctypes
import json
import os
import threading
from pathlib import Path
from typing import Optional, Sequence

PKG = Path(__file__).resolve().parent.parent
DEFAULT_LIB = PKG / "lib" / "libkt.so"

KT_OK = 0
KT_ERR_ARG = 1
KT_ERR_CUDA = 2
KT_ERR_TIMEOUT = 3
KT_ERR_UNSUPPORTED = 4
STATUS_NAMES = {
    KT_OK: "KT_OK",
    KT_ERR_ARG: "KT_ERR_ARG",
    KT_ERR_CUDA: "KT_ERR_CUDA",
    KT_ERR_TIMEOUT: "KT_ERR_TIMEOUT",
    KT_ERR_UNSUPPORTED: "KT_ERR_UNSUPPORTED",
}

KT_GEMM_FFMA = 0
KT_GEMM_TF32 = 1

KT_XRANK_MAX = 8
KT_XRANK_EXCHANGE_BYTES = 256

OP_IDS = {
    "softmax": 1,
    "layernorm": 2,
    "reduction": 3,
    "matmul": 4,
    "attention": 5,
    "naive_softmax": 101,
    "naive_layernorm": 102,
    "naive_reduction": 103,
    "naive_matmul": 104,
    "naive_attention": 105,
}

# Every symbol a built library must export (include/kt_abi.h).
EXPORTED_SYMBOLS = (
    "kt_last_error", "kt_version", "kt_variant_params",
    "kt_softmax_f32", "kt_layernorm_f32", "kt_reduce_workspace_bytes", "kt_reduce_sum_f32",
    "kt_reduce_sum_f32_xrank",
    "kt_gemm_f32", "kt_fa_fwd_bf16",
    "kt_naive_softmax_f32", "kt_naive_layernorm_f32", "kt_naive_reduce_sum_f32",
    "kt_naive_gemm_f32", "kt_naive_attention_bf16",
    "kt_run", "kt_time", "kt_device_error",
)

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_size = ctypes.c_size_t


class KtError(RuntimeError):
    """A non-zero status returned by the kernel library."""

    def __init__(self, status: int, message: str, call: str = ""):
        self.status = status
        self.message = message
        self.call = call
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{call}: {name}: {message}" if call else f"{name}: {message}")


class KtArgs(ctypes.Structure):
    """Mirror of `kt_args` (include/kt_abi.h)."""

    _fields_ = [
        ("in0", _vp), ("in1", _vp), ("in2", _vp),
        ("out0", _vp), ("out1", _vp),
        ("workspace", _vp), ("ws_bytes", _size),
        ("d0", _i64), ("d1", _i64), ("d2", _i64), ("d3", _i64),
        ("f0", _f32),
        ("i0", ctypes.c_int32), ("i1", ctypes.c_int32),
    ]


def make_args(in0=0, in1=0, in2=0, out0=0, out1=0, workspace=0, ws_bytes=0,
              d0=0, d1=0, d2=0, d3=0, f0=0.0, i0=0, i1=0) -> KtArgs:
    """Build a KtArgs from integers (device addresses) and sizes."""
    return KtArgs(in0 or None, in1 or None, in2 or None, out0 or None, out1 or None,
                  workspace or None, int(ws_bytes), int(d0), int(d1), int(d2), int(d3),
                  float(f0), int(i0), int(i1))


_SIGNATURES = {
    "kt_last_error": (ctypes.c_char_p, []),
    "kt_version": (_int, []),
    "kt_variant_params": (ctypes.c_char_p, []),
    "kt_softmax_f32": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "kt_layernorm_f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "kt_reduce_workspace_bytes": (_size, [_i64]),
    "kt_reduce_sum_f32": (_int, [_vp, _i64, _vp, _vp, _vp, _size, _vp]),
    "kt_reduce_sum_f32_xrank": (_int, [_vp, _i64, _vp, _vp, _vp, _size, ctypes.POINTER(_vp), _int, _int,
                                       ctypes.c_uint64, _vp]),
    "kt_gemm_f32": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp]),
    "kt_fa_fwd_bf16": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _int, _vp]),
    "kt_naive_softmax_f32": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "kt_naive_layernorm_f32": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "kt_naive_reduce_sum_f32": (_int, [_vp, _i64, _vp, _vp, _vp, _size, _vp]),
    "kt_naive_gemm_f32": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "kt_naive_attention_bf16": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _int, _vp]),
    "kt_run": (_int, [_int, ctypes.POINTER(KtArgs), _vp]),
    "kt_time": (_int, [_int, ctypes.POINTER(KtArgs), _int, _int, _vp, _size,
                       ctypes.POINTER(ctypes.c_float), _vp]),
    "kt_device_error": (_int, [_int, ctypes.POINTER(ctypes.c_int)]),
}


class KtLibrary:
    """One loaded kernel library (the default build or a tuning variant)."""

    def __init__(self, path: os.PathLike | str):
        self.path = Path(path)
        if not self.path.exists():
            raise FileNotFoundError(
                f"kernel library {self.path} not found; build it with "
                f"`python -c 'import __graft_entry__ as g; g.build()'`")
        # RTLD_LOCAL keeps each variant's identically named symbols apart.
        self._lib = ctypes.CDLL(str(self.path), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(self._lib, name)
            fn.restype = res
            fn.argtypes = args

    # -- plumbing -----------------------------------------------------------
    def last_error(self) -> str:
        msg = self._lib.kt_last_error()
        return msg.decode("utf-8", "replace") if msg else ""

    def _check(self, rc: int, call: str) -> None:
        if rc != KT_OK:
            raise KtError(rc, self.last_error(), call)

    def version(self) -> int:
        return int(self._lib.kt_version())

    def variant_params(self) -> dict:
        raw = self._lib.kt_variant_params()
        try:
            return json.loads(raw.decode()) if raw else {}
        except json.JSONDecodeError:
            return {"raw": raw.decode(errors="replace")}

    def symbol(self, name: str):
        return getattr(self._lib, name)

    # -- ops (device addresses as ints; stream = cudaStream_t as int or None) ----
    def softmax_f32(self, x: int, y: int, rows: int, cols: int, stream: Optional[int] = None) -> None:
        self._check(self._lib.kt_softmax_f32(x, y, rows, cols, stream), "kt_softmax_f32")

    def layernorm_f32(self, x: int, gamma: int, beta: int, y: int, rows: int, cols: int,
                      eps: float, stream: Optional[int] = None) -> None:
        self._check(self._lib.kt_layernorm_f32(x, gamma, beta, y, rows, cols, eps, stream),
                    "kt_layernorm_f32")

    def reduce_workspace_bytes(self, n: int) -> int:
        return int(self._lib.kt_reduce_workspace_bytes(n))

    def reduce_sum_f32(self, x: int, n: int, out64: int, out32: Optional[int], workspace: int,
                       ws_bytes: int, stream: Optional[int] = None) -> None:
        self._check(self._lib.kt_reduce_sum_f32(x, n, out64, out32, workspace, ws_bytes, stream),
                    "kt_reduce_sum_f32")

    def reduce_sum_f32_xrank(self, x: int, n: int, out64: int, out32: Optional[int], workspace: int,
                             ws_bytes: int, exchange: Sequence[int], rank: int, world: int, epoch: int,
                             stream: Optional[int] = None) -> None:
        """Whole-job sum across `world` ranks (kt_reduce_sum_f32_xrank); `exchange`
        holds every rank's exchange buffer address as mapped in this process."""
        arr = (_vp * max(len(exchange), 1))(*[int(p) or None for p in exchange]) if exchange else None
        self._check(self._lib.kt_reduce_sum_f32_xrank(x, n, out64, out32, workspace, ws_bytes, arr, rank, world,
                                                      epoch, stream), "kt_reduce_sum_f32_xrank")

    def gemm_f32(self, A: int, B: int, C: int, M: int, N: int, K: int, transpose_b: bool,
                 variant: int, stream: Optional[int] = None) -> None:
        self._check(self._lib.kt_gemm_f32(A, B, C, M, N, K, int(bool(transpose_b)), variant, stream),
                    "kt_gemm_f32")

    def fa_fwd_bf16(self, Q: int, K: int, V: int, O: int, B: int, H: int, S: int, D: int,
                    scale: float, causal: bool, stream: Optional[int] = None) -> None:
        self._check(self._lib.kt_fa_fwd_bf16(Q, K, V, O, B, H, S, D, scale, int(bool(causal)), stream),
                    "kt_fa_fwd_bf16")

    def run(self, op: int | str, args: KtArgs, stream: Optional[int] = None) -> None:
        op_id = OP_IDS[op] if isinstance(op, str) else int(op)
        self._check(self._lib.kt_run(op_id, ctypes.byref(args), stream), f"kt_run(op={op})")

    def time(self, op: int | str, args: KtArgs, warmup: int, iters: int, flush: int = 0,
             flush_bytes: int = 0, stream: Optional[int] = None) -> list[float]:
        """In-process CUDA-event samples (ms), one per timed launch."""
        op_id = OP_IDS[op] if isinstance(op, str) else int(op)
        buf = (ctypes.c_float * max(iters, 1))()
        rc = self._lib.kt_time(op_id, ctypes.byref(args), warmup, iters, flush or None, flush_bytes, buf, stream)
        self._check(rc, f"kt_time(op={op})")
        return [float(buf[i]) for i in range(iters)]

    def device_error(self, reset: bool = False) -> int:
        code = ctypes.c_int(0)
        self._check(self._lib.kt_device_error(int(reset), ctypes.byref(code)), "kt_device_error")
        return int(code.value)


_CACHE: dict[str, KtLibrary] = {}
_LOCK = threading.Lock()


def default_library_path() -> Path:
    env = os.environ.get("KT_LIBRARY")
    return Path(env) if env else DEFAULT_LIB


def load(path: Optional[os.PathLike | str] = None) -> KtLibrary:
    """Load (once per path) and return a kernel library; raises if it is missing."""
    p = Path(path) if path is not None else default_library_path()
    key = str(p.resolve()) if p.exists() else str(p)
    with _LOCK:
        lib = _CACHE.get(key)
        if lib is None:
            lib = KtLibrary(p)
            _CACHE[key] = lib
        return lib


def missing_symbols(path: os.PathLike | str, names: Sequence[str] = EXPORTED_SYMBOLS) -> list[str]:
    """Names from `names` that the library at `path` does not export."""
    lib = ctypes.CDLL(str(path), mode=os.RTLD_NOW | os.RTLD_LOCAL)
    return [n for n in names if not hasattr(lib, n)]
