"""
generator.py — emits one sm_100a kernel-library variant per parameter point.

The reference formats whole CUDA kernels plus a benchmark `main()` from
Python string templates per variant (src/generator.py:28-281) and compiles
each into an executable. Here the kernels are hand-written C++ templates in
csrc/*.cuh; a variant is a short translation unit that fixes the template
parameters with macros, restricts the build to one family (`KT_ONLY_*`) and
includes csrc/kt_entry.cuh, so every variant is a shared library exporting
the same C ABI (include/kt_abi.h). `kt_variant_params()` of the built
library returns the parameters as JSON.

Public API kept from the reference: ARCH, `_variant_tag`,
`enumerate_variants(kernel, space)` (src/generator.py:435-458),
`write_variant(kernel, params, out_path, matrix_size)` (src/generator.py:461-476),
`GENERATORS`, plus `compile_variant` (the reference's autotune.py:120-129).
Output directories are created on first use, not at import.
"""

from __future__ import annotations

import itertools
import json
import os
from pathlib import Path
from typing import Any, Optional

import build as kt_build
from parser import is_valid

ARCH = kt_build.ARCH  # "sm_100a"

PKG = Path(__file__).resolve().parent.parent


def results_dir() -> Path:
    return Path(os.environ.get("KT_RESULTS_DIR", PKG / "results"))


def gen_dir() -> Path:
    d = results_dir() / "generated"
    d.mkdir(parents=True, exist_ok=True)
    return d


def variants_dir() -> Path:
    d = results_dir() / "variants"
    d.mkdir(parents=True, exist_ok=True)
    return d


# parameter -> macro, per family; parameters absent here are runtime arguments
MACROS: dict[str, dict[str, str]] = {
    "softmax": {"block_size": "KT_SOFTMAX_BLOCK", "vec_per_thread": "KT_SOFTMAX_VPT", "min_blocks": "KT_SOFTMAX_MINB",
                "stages": "KT_SOFTMAX_STAGES", "cluster_size": "KT_SOFTMAX_CLUSTER", "tma_box": "KT_ROWS_BOX"},
    "layernorm": {"block_size": "KT_LN_BLOCK", "vec_per_thread": "KT_LN_VPT", "min_blocks": "KT_LN_MINB",
                  "stages": "KT_LN_STAGES", "cluster_size": "KT_LN_CLUSTER", "tma_box": "KT_ROWS_BOX"},
    "reduction": {"block_size": "KT_REDUCE_BLOCK", "unroll": "KT_REDUCE_UNROLL", "blocks_per_sm": "KT_REDUCE_BPSM"},
    "matmul": {"bk": "KT_FFMA_BK", "ffma_x2": "KT_FFMA_X2", "ffma_wide": "KT_FFMA_WIDE", "min_blocks": "KT_FFMA_MINB",
               "cta_tile": "KT_TC_BN", "stages": "KT_TC_STAGES"},
    "attention": {"kind": "KT_FA_KIND", "stages": "KT_FA_STAGES", "v_stages": "KT_FA_VSTAGES",
                  "poly_exp2": "KT_FA_POLY", "order": "KT_FA2_ORDER", "poly_every": "KT_FA2_POLY", "exp16": "KT_FA_EXP16",
                  "spec": "KT_FA_SPEC", "reload": "KT_FA_RELOAD", "issuers": "KT_FA_ISSUERS",
                  "alt": "KT_FA_ALT", "sbuf": "KT_FA_SBUF", "x2": "KT_FA_X2",
                  "warp_arrive": "KT_FA_WARP_ARRIVE", "spec0": "KT_FA_SPEC0", "dephase": "KT_FA_DEPHASE",
                  "psplit": "KT_FA_PSPLIT", "bn": "KT_FA_BN", "fuse": "KT_FA_FUSE"},
}
ONLY = {"softmax": "KT_ONLY_SOFTMAX", "layernorm": "KT_ONLY_LAYERNORM", "reduction": "KT_ONLY_REDUCE",
        "matmul": "KT_ONLY_GEMM", "attention": "KT_ONLY_FA"}
RUNTIME_PARAMS = {"matmul": ("variant", "transpose_b"), "attention": ("causal",)}


def _macro_value(param: str, value: Any) -> str:
    if param == "cta_tile":            # "128x256" -> N extent of the accumulator tile
        return str(int(str(value).split("x")[1]))
    if isinstance(value, bool):
        return "1" if value else "0"
    return str(value)


def _variant_tag(kernel: str, params: dict) -> str:
    """`kernel_k1v1_k2v2…` with keys sorted (the reference's tag, src/generator.py:327-331)."""
    parts = [kernel]
    for k, v in sorted(params.items()):
        parts.append(f"{k}{v}")
    return "_".join(str(p) for p in parts)


def generate_source(kernel: str, params: dict, matrix_size: Optional[int] = None) -> str:
    """Translation unit of one variant."""
    if kernel not in MACROS:
        raise ValueError(f"No generator for kernel {kernel!r}")
    macros = MACROS[kernel]
    lines = [
        "/*",
        f" * Generated {ARCH} variant of the {kernel} family: "
        + " ".join(f"{k}={v}" for k, v in sorted(params.items())),
        " * Compiled by generator.compile_variant into a shared library exporting include/kt_abi.h.",
        " */",
        f"#define {ONLY[kernel]} 1",
    ]
    for p, v in sorted(params.items()):
        if p in macros:
            lines.append(f"#define {macros[p]} {_macro_value(p, v)}")
        elif p not in RUNTIME_PARAMS.get(kernel, ()):
            raise ValueError(f"{kernel}: unknown parameter {p!r}")
    meta = {"kernel": kernel, **params}
    if matrix_size is not None:
        meta["matrix_size"] = matrix_size
    js = json.dumps(meta, sort_keys=True).replace("\\", "\\\\").replace('"', '\\"')
    lines.append(f'#define KT_VARIANT_JSON "{js}"')
    lines.append('#include "kt_entry.cuh"')
    return "\n".join(lines) + "\n"


def _gen(kernel):
    def g(params: dict, matrix_size: Optional[int] = None) -> str:
        return generate_source(kernel, params, matrix_size)
    g.__name__ = f"generate_{kernel}"
    return g


generate_softmax = _gen("softmax")
generate_layernorm = _gen("layernorm")
generate_reduction = _gen("reduction")
generate_matmul = _gen("matmul")
generate_attention = _gen("attention")

GENERATORS = {
    "softmax": generate_softmax,
    "layernorm": generate_layernorm,
    "reduction": generate_reduction,
    "matmul": generate_matmul,
    "attention": generate_attention,
}


def enumerate_variants(kernel: str, space: dict) -> list[tuple[dict, Path]]:
    """Cartesian product of the space with validity pruning; (params, .cu path) per variant."""
    keys = [k for k in space if not k.startswith("_")]
    out: list[tuple[dict, Path]] = []
    for combo in itertools.product(*(space[k] for k in keys)):
        params = dict(zip(keys, combo))
        if not is_valid(kernel, params):
            continue
        out.append((params, gen_dir() / f"{_variant_tag(kernel, params)}.cu"))
    return out


def compile_key(kernel: str, params: dict) -> str:
    """Tag of the compiled artefact: runtime-only parameters do not change the library."""
    rt = RUNTIME_PARAMS.get(kernel, ())
    return _variant_tag(kernel, {k: v for k, v in params.items() if k not in rt})


def write_variant(kernel: str, params: dict, out_path: Path, matrix_size: Optional[int] = None) -> None:
    """Write the variant's translation unit to out_path."""
    gen = GENERATORS.get(kernel)
    if gen is None:
        raise ValueError(f"No generator for kernel {kernel!r}")
    Path(out_path).parent.mkdir(parents=True, exist_ok=True)
    Path(out_path).write_text(gen(params, matrix_size=matrix_size), encoding="utf-8")


def compile_variant(src: Path, lib_path: Optional[Path] = None, timeout: int = 900) -> tuple[bool, str, Path]:
    """nvcc the variant into a shared library; returns (ok, stderr with the ptxas report, path)."""
    out = Path(lib_path) if lib_path else variants_dir() / (Path(src).stem + ".so")
    ok, err = kt_build.compile_shared(Path(src), out, timeout=timeout)
    return ok, err, out


def ensure_variant(kernel: str, params: dict, matrix_size: Optional[int] = None) -> tuple[bool, str, Path]:
    """Write + compile (cached by compile key) one variant; returns (ok, ptxas log, .so path)."""
    key = compile_key(kernel, params)
    src = gen_dir() / f"{key}.cu"
    so = variants_dir() / f"{key}.so"
    log = variants_dir() / f"{key}.ptxas.txt"
    rt = RUNTIME_PARAMS.get(kernel, ())
    cparams = {k: v for k, v in params.items() if k not in rt}
    text = generate_source(kernel, cparams, matrix_size)
    if so.exists() and src.exists() and src.read_text() == text and log.exists() \
            and so.stat().st_mtime >= max(f.stat().st_mtime for f in kt_build._sources()):
        return True, log.read_text(), so
    src.write_text(text)
    ok, err, so = compile_variant(src, so)
    if ok:
        log.write_text(err)
    return ok, err, so


if __name__ == "__main__":
    import sys
    from parser import build_kernel_profile, build_search_space
    kernel = sys.argv[1] if len(sys.argv) > 1 else "softmax"
    variants = enumerate_variants(kernel, build_search_space(build_kernel_profile(kernel)))
    print(f"Kernel: {kernel}  ->  {len(variants)} variants")
    for params, path in variants[:3]:
        write_variant(kernel, params, path)
        print(f"  Written: {path.name}")
