"""
parser.py — kernel profiles and the tuning search space.

Keeps the reference's data model (src/parser.py:37-82: `MemoryAccessPattern`,
`KernelInfo`, `KernelProfile`), its regex source scanner (src/parser.py:223-308)
and `build_search_space(profile)` (src/parser.py:311-352), and adds the
Blackwell axes the sm_100a kernels actually expose:

  memory-bound rows (softmax, layernorm):
      block_size, vec_per_thread (128-bit loads per thread, i.e. the row
      capacity held in registers), min_blocks (occupancy hint), stages
      (rows in flight per CTA through a TMA bulk-copy ring; 0 = register kernel),
      cluster_size (CTAs of a thread-block cluster that split every row and
      exchange partial statistics through distributed shared memory),
      tma_box (bytes per bulk copy of a row or chunk; 0 = one copy)
  reduction:
      block_size, unroll (16-byte loads in flight per thread), blocks_per_sm
  matmul:
      variant {ffma, tf32}, transpose_b; ffma: bk (k tile), ffma_x2 (packed
      fma.rn.f32x2 kernel), min_blocks (register budget: CTAs per SM);
      tf32 (tcgen05): cta_tile (M×N of the TMEM accumulator), stages (TMA
      pipeline depth)
  attention (tcgen05): kind (1: one query tile per CTA, 2: two ping-pong
      query tiles), stages / v_stages (K / V ring depth) and poly_exp2 for
      kind 1, order (MMA issue order) and poly_every (FMA-pipe exponential
      share) for kind 2

Each axis is a template parameter of the kernel source (see generator.py),
so every point of the space compiles to a distinct kernel. The reference's
libclang parser is kept as an optional path (libclang is absent here and the
regex scanner is used, as in the reference's fallback).
"""

from __future__ import annotations

import re
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

try:
    import clang.cindex as _ci  # noqa: F401
    _LIBCLANG_OK = True
except ImportError:
    _ci = None  # type: ignore
    _LIBCLANG_OK = False


@dataclass
class MemoryAccessPattern:
    """Memory access characteristics extracted from kernel source."""
    has_global_load: bool = False
    has_global_store: bool = False
    has_shared_mem: bool = False
    has_coalesced_hint: bool = False
    has_strided_access: bool = False
    has_reduction: bool = False
    has_warp_shuffle: bool = False
    has_tma: bool = False
    has_tensor_core: bool = False


@dataclass
class KernelInfo:
    """Kernel metadata (superset of KernelProfile)."""
    name: str
    src_path: Path
    param_names: list[str] = field(default_factory=list)
    param_types: list[str] = field(default_factory=list)
    param_count: int = 0
    has_shared_mem: bool = False
    has_unroll: bool = False
    uses_threadidx: bool = False
    uses_blockidx: bool = False
    memory: MemoryAccessPattern = field(default_factory=MemoryAccessPattern)

    def to_profile(self) -> "KernelProfile":
        return KernelProfile(name=self.name, src_path=self.src_path, block_dim=0,
                             uses_shared=self.has_shared_mem, loop_depth=1 if self.has_unroll else 0,
                             memory=self.memory)


@dataclass
class KernelProfile:
    """Optimisation-focused profile used by generator.py and search.py."""
    name: str
    src_path: Path
    block_dim: int
    uses_shared: bool
    loop_depth: int
    reduction_ops: list[str] = field(default_factory=list)
    memory: MemoryAccessPattern = field(default_factory=MemoryAccessPattern)
    raw_params: dict = field(default_factory=dict)


# ---------------------------------------------------------------------------
# Regex scanner (the reference's fallback parser, src/parser.py:223-308)
# ---------------------------------------------------------------------------

_RE_KERNEL = re.compile(r"__global__\s+(?:void\s+)?(?:__launch_bounds__\([^)]*\)\s*)?(?:void\s+)?(\w+)\s*\(")
_RE_SHARED = re.compile(r"__shared__")
_RE_STRIDE = re.compile(r"\[\s*\w+\s*\*\s*\w+\s*\+")
_RE_REDUCTION = re.compile(r"\+=|block_sum|warp_sum|fmaxf")
_RE_SHFL = re.compile(r"__shfl_\w+_sync")
_RE_TMA = re.compile(r"cp\.async\.bulk")
_RE_TC = re.compile(r"tcgen05\.mma")
_RE_LOOP = re.compile(r"\bfor\s*\(")


class RegexKernelParser:
    """Find `__global__` kernels in a CUDA source and derive a KernelProfile each."""

    def parse_to_profiles(self, src_path: Path) -> list[KernelProfile]:
        src = Path(src_path).read_text(encoding="utf-8")
        starts = [(m.group(1), m.start()) for m in _RE_KERNEL.finditer(src)]
        out: list[KernelProfile] = []
        for i, (name, start) in enumerate(starts):
            end = starts[i + 1][1] if i + 1 < len(starts) else len(src)
            body = src[start:end]
            mem = MemoryAccessPattern(
                has_global_load=True,
                has_global_store=True,
                has_shared_mem=bool(_RE_SHARED.search(body)),
                has_strided_access=bool(_RE_STRIDE.search(body)),
                has_reduction=bool(_RE_REDUCTION.search(body)),
                has_warp_shuffle=bool(_RE_SHFL.search(body)) or "warp_sum" in body or "block_sum" in body,
                has_tma=bool(_RE_TMA.search(body)),
                has_tensor_core=bool(_RE_TC.search(body)),
            )
            out.append(KernelProfile(
                name=name, src_path=Path(src_path), block_dim=0,
                uses_shared=mem.has_shared_mem,
                loop_depth=len(_RE_LOOP.findall(body)),
                reduction_ops=_RE_REDUCTION.findall(body),
                memory=mem,
            ))
        return out


class LibclangKernelParser:  # pragma: no cover - libclang is not installed in this image
    def __init__(self) -> None:
        if not _LIBCLANG_OK:
            raise RuntimeError("libclang (python package 'clang') is not installed")
        raise RuntimeError("libclang parsing of sm_100a inline PTX is not supported; use RegexKernelParser")


def make_parser():
    """Return the best available parser (the regex scanner here)."""
    if _LIBCLANG_OK:
        try:
            return LibclangKernelParser()
        except Exception as e:  # noqa: BLE001
            warnings.warn(f"libclang unavailable ({e}); using the regex parser.")
    return RegexKernelParser()


# ---------------------------------------------------------------------------
# Family profiles and search spaces
# ---------------------------------------------------------------------------

FAMILIES = ("softmax", "layernorm", "reduction", "matmul", "attention")


def family_of(profile_or_name) -> str:
    name = profile_or_name.name if isinstance(profile_or_name, KernelProfile) else str(profile_or_name)
    for fam in FAMILIES:
        if name.startswith(fam):
            return fam
    raise ValueError(f"no kernel family for {name!r}")


def build_kernel_profile(kernel: str, src_root: Optional[Path] = None) -> KernelProfile:
    """Profile of a family's sm_100a source (the reference builds these by hand, autotune.py:98-115)."""
    csrc = src_root or Path(__file__).resolve().parent.parent / "csrc"
    src = {"softmax": "softmax.cuh", "layernorm": "layernorm.cuh", "reduction": "reduce.cuh",
           "matmul": "gemm_tf32.cuh", "attention": "fa_fwd.cuh"}[kernel]
    mem = MemoryAccessPattern(
        has_global_load=True,
        has_global_store=True,
        has_strided_access=kernel == "matmul",
        has_reduction=kernel in ("reduction", "softmax", "layernorm"),
        has_shared_mem=kernel in ("matmul", "attention"),
        has_warp_shuffle=kernel in ("reduction", "softmax", "layernorm"),
        has_tma=kernel in ("matmul", "attention"),
        has_tensor_core=kernel in ("matmul", "attention"),
    )
    return KernelProfile(name=kernel, src_path=csrc / src, block_dim=0, uses_shared=mem.has_shared_mem,
                         loop_depth=2 if kernel == "matmul" else 1,
                         reduction_ops=["+="] if mem.has_reduction else [], memory=mem)


def build_search_space(profile: KernelProfile) -> dict:
    """
    Candidate parameter grid for a profile.

    For the five sm_100a families the axes are the template parameters of
    their kernels (module docstring). For any other profile the reference's
    generic grid is returned (block_size × unroll × tile_x/tile_y ×
    transpose_b × warp_shuffle, src/parser.py:311-352).
    """
    try:
        fam = family_of(profile)
    except ValueError:
        fam = None
    space: dict[str, list] = {}
    if fam in ("softmax", "layernorm"):
        space["block_size"] = [128, 256, 512, 1024]
        space["vec_per_thread"] = [1, 2, 4, 8]
        space["min_blocks"] = [1, 2, 4]
        space["stages"] = [0, 2, 3, 4]    # 0: one row per CTA in registers; n: TMA bulk-copy ring of n rows
        space["cluster_size"] = [1, 2, 4]  # CTAs of a thread-block cluster sharing each row (DSMEM exchange)
        space["tma_box"] = [0, 4096, 8192]  # bytes per bulk copy of a row or chunk (0: one copy)
    elif fam == "reduction":
        space["block_size"] = [256, 512, 1024]
        space["unroll"] = [2, 4, 8]
        space["blocks_per_sm"] = [1, 2, 4, 8]
    elif fam == "matmul":
        space["variant"] = ["tf32", "ffma"]
        space["transpose_b"] = [False, True]
        space["bk"] = [8, 16, 32]
        space["ffma_x2"] = [0, 1]         # ffma: packed fma.rn.f32x2 (two fp32 FMAs per lane per instruction)
        space["ffma_wide"] = [0, 1]       # ffma: 128x256 CTA tile, 8x16 outputs per thread (k tile 8 or 16)
        space["min_blocks"] = [1, 2]      # ffma: resident CTAs per SM asked of the register allocator
        space["cta_tile"] = ["128x128", "128x192", "128x224", "128x256"]
        space["stages"] = [3, 4, 5, 6]
    elif fam == "attention":
        space["kind"] = [1, 2]            # 1: one 128-row query tile per CTA; 2: two ping-pong query tiles
        space["stages"] = [1, 2, 3]       # kind 1: K ring depth
        space["v_stages"] = [1, 2, 3]     # kind 1: V ring depth
        space["poly_exp2"] = [0, 1, 2]    # kind 1: n of every 4 exponential pairs on the FMA pipe (polynomial)
        space["issuers"] = [1, 2]         # kind 1: threads issuing tcgen05.mma (2: S and P·V from two warps)
        space["alt"] = [0, 1]             # kind 1: softmax warps of a lane quarter take alternate S tiles (1)
        space["sbuf"] = [2, 3, 4]         # kind 1: S accumulators in TMEM (3, 4: P written over its S tile)
        space["x2"] = [0, 1]              # kind 1: exponent arguments and row sums in packed f32x2 instructions
        space["warp_arrive"] = [0, 1]     # kind 1: one mbarrier arrival per warp instead of per thread
        space["spec0"] = [0, 1]           # kind 1: first tile of an item speculates on the previous item's max
        space["dephase"] = [0, 400, 800]  # kind 1: clocks the second softmax warp of a scheduler starts late
        space["psplit"] = [1, 2, 3, 4]    # kind 1, alternate tiles: P·V issued per key range as P is stored
        space["bn"] = [128, 96]           # kind 1: keys per S tile (96: four S buffers in TMEM)
        space["fuse"] = [0, 1]            # kind 1, alternate tiles: one speculative pass per tile
        space["order"] = [0, 1]           # kind 2: MMA issue order (0 ping-pong, 1 in phase)
        space["poly_every"] = [0, 4, 8]   # kind 2: every n-th exponential pair on the FMA pipe (0: none)
        space["causal"] = [False, True]
    else:
        space["block_size"] = [64, 128, 192, 256]
        space["unroll"] = [1, 2, 4, 8] if profile.loop_depth >= 1 else [1]
        if not profile.uses_shared:
            space["tile_x"] = [16, 32]
            space["tile_y"] = [16, 32]
        else:
            space["tile_x"] = [16]
            space["tile_y"] = [16]
        space["transpose_b"] = [False, True] if profile.memory.has_strided_access else [False]
        space["warp_shuffle"] = [False, True] if profile.memory.has_reduction else [False]
    total = 1
    for v in space.values():
        total *= len(v)
    space["_total_variants"] = total
    space["_kernel"] = profile.name
    return space


def is_valid(kernel: str, params: dict) -> bool:
    """Validity pruning (the reference prunes matmul tiles, src/generator.py:446-452)."""
    if "tile_x" in params and "tile_y" in params:
        # the reference's generic grid: square tiles no larger than the block
        return params["tile_x"] == params["tile_y"] and params["tile_x"] <= params.get("block_size", 1 << 30)
    fam = family_of(kernel) if kernel in FAMILIES else kernel
    if fam in ("softmax", "layernorm"):
        if params.get("stages", 0) > 0 and params.get("min_blocks", 1) != 1:
            return False  # the staged kernel sizes its grid by occupancy; min_blocks only shapes the register kernel
        if params.get("tma_box", 0) and params.get("stages", 3) == 0 and params.get("cluster_size", 1) == 1:
            return False  # the register kernel makes no bulk copies
        return params.get("block_size", 256) * params.get("min_blocks", 1) <= 2048
    if fam == "reduction":
        return params.get("block_size", 512) * params.get("blocks_per_sm", 1) <= 2048
    if fam == "matmul":
        if params.get("variant") == "ffma":
            # the FFMA kernels ignore the tcgen05 axes: keep one representative point; the scalar
            # kernel's static shared tiles exceed 48 KB at bk=32
            if params.get("bk", 16) == 32 and not params.get("ffma_x2", 1):
                return False
            if params.get("ffma_wide", 0):
                # the wide kernel has its own fixed shape: one representative point
                if params.get("ffma_x2", 0) or params.get("bk", 8) not in (8, 16) or params.get("min_blocks", 1) != 1:
                    return False
            return params.get("cta_tile", "128x128") == "128x128" and params.get("stages", 4) == 4
        # the tcgen05 kernel ignores the FFMA axes; a stage holds a 128x32 A box and a BNx32 B box
        # (48 KB at 128x256): the 227 KB of shared memory fit 4 stages of 128x256, 5 of 128x192
        # and 128x224, 6 of 128x128
        max_stages = {"128x128": 6, "128x192": 5, "128x224": 5, "128x256": 4}[params.get("cta_tile", "128x128")]
        if params.get("stages", 4) > max_stages:
            return False
        return params.get("bk", 16) == 16 and params.get("ffma_x2", 1) == 1 and params.get("min_blocks", 2) == 2 \
            and params.get("ffma_wide", 0) == 0
    if fam == "attention":
        if params.get("kind", 1) == 2:
            # half-precision exponentials gave NaN on the first causal rows of heads whose
            # scores reach ~300 (log2 units) in this kernel: not offered
            if params.get("exp16", 0):
                return False
            # the kind-1 axes do not shape this kernel: one representative point
            return (params.get("stages", 2), params.get("v_stages", 2), params.get("poly_exp2", 0),
                    params.get("issuers", 2), params.get("alt", 0), params.get("sbuf", 2), params.get("x2", 0),
                    params.get("warp_arrive", 0), params.get("spec0", 0),
                    params.get("dephase", 0), params.get("psplit", 1),
                    params.get("bn", 128), params.get("fuse", 0)) == (2, 2, 0, 2, 0, 2, 0, 0, 0, 0, 1, 128, 0)
        if params.get("order", 0) != 0 or params.get("poly_every", 0) != 0:
            return False
        if params.get("alt", 0) and (params.get("spec", 1) != 1 or params.get("reload", 0) != 0
                                     or params.get("spec0", 0) or params.get("dephase", 0)):
            return False  # whole-row softmax: the column-half exchange axes do not shape it
        bn = params.get("bn", 128)
        if (bn // 32) % params.get("psplit", 1):
            return False  # P·V key ranges are whole 32-key chunks
        if bn == 96 and (not params.get("alt", 0) or params.get("sbuf", 4) != 4):
            return False  # 96-key tiles: four S buffers, alternate-tile softmax
        if bn == 128 and params.get("sbuf", 2) == 4:
            return False  # four 128-key S buffers leave no TMEM columns for O
        if params.get("fuse", 0) and not params.get("alt", 0):
            return False  # the fused pass belongs to the alternate-tile softmax
        if params.get("psplit", 1) != 1 and not params.get("alt", 0):
            return False  # the split P·V issue follows the whole-row P stores of the alternate-tile softmax
        if params.get("sbuf", 2) >= 3 and params.get("reload", 0):
            return False  # P over S needs the two issuers and the scores kept in registers
        # head dim 128: two Q buffers + (K + V slots) x 32 KB must fit the 227 KB of shared memory
        return params.get("stages", 2) + params.get("v_stages", 2) <= 4
    return True


# The configuration each family's default library (lib/libkt.so) is built with,
# i.e. the header defaults of the macros generator.MACROS maps the axes to
# (tests/test_host.py checks the two agree). Axes a kernel ignores carry the
# representative value is_valid keeps; runtime axes are expanded over their values.
DEFAULTS: dict[str, list[dict]] = {
    "softmax": [dict(block_size=256, vec_per_thread=4, min_blocks=1, stages=2, cluster_size=1, tma_box=0)],
    "layernorm": [dict(block_size=256, vec_per_thread=4, min_blocks=1, stages=2, cluster_size=1, tma_box=0)],
    "reduction": [dict(block_size=512, unroll=4, blocks_per_sm=4)],
    "matmul": [dict(variant="tf32", bk=16, ffma_x2=1, ffma_wide=0, min_blocks=2, cta_tile="128x256", stages=4),
               dict(variant="ffma", bk=8, ffma_x2=0, ffma_wide=1, min_blocks=1, cta_tile="128x128", stages=4)],
    "attention": [dict(kind=1, stages=2, v_stages=2, poly_exp2=1, issuers=2, alt=1, sbuf=3, x2=1, warp_arrive=0,
                       spec0=0, dephase=0, psplit=2, bn=128, fuse=0, order=0, poly_every=0)],
}


def default_points(kernel: str, space: dict) -> list[dict]:
    """The default library's configuration as points of `space` (every value of
    the runtime axes the defaults leave open), valid ones only. Strategies
    evaluate these first, so a sweep never reports a winner slower than what it
    was meant to improve on."""
    fam = family_of(kernel) if kernel in FAMILIES else kernel
    keys = [k for k in space if not k.startswith("_")]
    out: list[dict] = []
    for base in DEFAULTS.get(fam, []):
        open_keys = [k for k in keys if k not in base]
        combos = [{}]
        for k in open_keys:
            combos = [dict(c, **{k: v}) for c in combos for v in space[k]]
        for c in combos:
            pt = {k: (base[k] if k in base else c[k]) for k in keys}
            if all(pt[k] in space[k] for k in keys) and is_valid(kernel, pt) and pt not in out:
                out.append(pt)
    return out


if __name__ == "__main__":
    for fam in FAMILIES:
        prof = build_kernel_profile(fam)
        sp = build_search_space(prof)
        print(fam, sp["_total_variants"], {k: v for k, v in sp.items() if not k.startswith("_")})
