"""
occupancy.py — theoretical occupancy for sm_100a from `nvcc -Xptxas -v`.

Rebuild of the reference's sm_75 analyzer (src/occupancy.py:37-357): the same
`parse_ptxas_stderr`, `compute_occupancy`, `OccupancyInfo` and
`OccupancyAnalyzer.analyze_from_stderr / analyze / print_table`, with B200
limits and the resources an sm_100a kernel actually consumes:

  * 65,536 registers per SM, allocated per warp in units of 256;
  * 64 resident warps and 32 resident CTAs per SM;
  * 228 KiB shared memory per SM, up to 227 KiB per CTA, 1 KiB reserved per CTA,
    static + dynamic shared memory both counted;
  * 512 TMEM columns per SM (a CTA holding N columns limits residency to 512/N);
  * cluster size (a cluster's CTAs are co-scheduled on one GPC; it does not
    change per-SM residency in this model).

The reference regex-parsed only static smem and capped at 48 KiB.
"""

from __future__ import annotations

import math
import re
import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

SM100_REGS_PER_SM = 65_536
SM100_MAX_REGS_PER_THREAD = 255
SM100_REG_ALLOC_UNIT = 256          # registers, per warp
SM100_MAX_WARPS_PER_SM = 64
SM100_MAX_BLOCKS_PER_SM = 32
SM100_SMEM_PER_SM = 228 * 1024
SM100_MAX_SMEM_PER_BLOCK = 227 * 1024
SM100_SMEM_RESERVED_PER_BLOCK = 1024
SM100_TMEM_COLUMNS = 512
SM100_WARP_SIZE = 32


@dataclass
class OccupancyInfo:
    """Resource usage and derived occupancy for one compiled kernel."""
    kernel_name: str
    registers_per_thread: int
    shared_mem_bytes: int
    spill_stores: int
    spill_loads: int
    has_register_spill: bool
    occupancy: float
    active_warps: int
    block_size: int
    active_blocks: int = 0
    limiter: str = ""
    tmem_columns: int = 0


_RE_FUNC = re.compile(r"Function properties for\s+(\S+)")
_RE_COMPILING = re.compile(r"Compiling entry function '([^']+)'")
_RE_REGS_LINE = re.compile(r"Used\s+(\d+)\s+registers?", re.IGNORECASE)
_RE_SMEM_LINE = re.compile(r"(\d+)\s+bytes\s+smem", re.IGNORECASE)
_RE_SPILLS_LINE = re.compile(r"(\d+)\s+bytes?\s+spill\s+stores?", re.IGNORECASE)
_RE_SPILLL_LINE = re.compile(r"(\d+)\s+bytes?\s+spill\s+loads?", re.IGNORECASE)
_RE_BARRIERS = re.compile(r"used\s+(\d+)\s+barriers", re.IGNORECASE)


def parse_ptxas_stderr(stderr: str) -> dict[str, dict]:
    """
    Parse nvcc -Xptxas -v output into {function: {registers, smem_bytes,
    spill_stores, spill_loads, barriers}}.

    ptxas prints, per entry function::

        ptxas info    : Compiling entry function '_ZN2kt...' for 'sm_100a'
        ptxas info    : Function properties for _ZN2kt...
            0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
        ptxas info    : Used 40 registers, used 1 barriers, 256 bytes smem, ...
    """
    results: dict[str, dict] = {}
    current: Optional[str] = None
    defaults = {"registers": 0, "smem_bytes": 0, "spill_stores": 0, "spill_loads": 0, "barriers": 0}
    for line in stderr.splitlines():
        m = _RE_COMPILING.search(line) or _RE_FUNC.search(line)
        if m:
            current = m.group(1)
            results.setdefault(current, dict(defaults))
            continue
        if current is None:
            continue
        entry = results[current]
        m = _RE_REGS_LINE.search(line)
        if m:
            entry["registers"] = int(m.group(1))
            mb = _RE_BARRIERS.search(line)
            if mb:
                entry["barriers"] = int(mb.group(1))
        m = _RE_SMEM_LINE.search(line)
        if m:
            entry["smem_bytes"] = int(m.group(1))
        m = _RE_SPILLS_LINE.search(line)
        if m:
            entry["spill_stores"] = int(m.group(1))
        m = _RE_SPILLL_LINE.search(line)
        if m:
            entry["spill_loads"] = int(m.group(1))
    return results


def compute_occupancy(
    registers_per_thread: int,
    smem_bytes: int,
    block_size: int,
    dynamic_smem_bytes: int = 0,
    tmem_columns: int = 0,
    max_regs_per_sm: int = SM100_REGS_PER_SM,
    max_smem_per_sm: int = SM100_SMEM_PER_SM,
    max_warps_per_sm: int = SM100_MAX_WARPS_PER_SM,
    max_blocks_per_sm: int = SM100_MAX_BLOCKS_PER_SM,
    warp_size: int = SM100_WARP_SIZE,
) -> tuple[float, int]:
    """Theoretical occupancy on sm_100a: (fraction of 64 warps, active warps)."""
    occ, warps, _, _ = occupancy_detail(registers_per_thread, smem_bytes, block_size, dynamic_smem_bytes,
                                        tmem_columns, max_regs_per_sm, max_smem_per_sm, max_warps_per_sm,
                                        max_blocks_per_sm, warp_size)
    return occ, warps


def occupancy_detail(registers_per_thread, smem_bytes, block_size, dynamic_smem_bytes=0, tmem_columns=0,
                     max_regs_per_sm=SM100_REGS_PER_SM, max_smem_per_sm=SM100_SMEM_PER_SM,
                     max_warps_per_sm=SM100_MAX_WARPS_PER_SM, max_blocks_per_sm=SM100_MAX_BLOCKS_PER_SM,
                     warp_size=SM100_WARP_SIZE) -> tuple[float, int, int, str]:
    """(occupancy, active warps, active blocks, limiting resource)."""
    if block_size <= 0:
        return 0.0, 0, 0, "block_size"
    warps_per_block = math.ceil(block_size / warp_size)
    limits = {"blocks": max_blocks_per_sm, "warps": max_warps_per_sm // warps_per_block}
    if registers_per_thread > 0:
        regs_per_warp = math.ceil(registers_per_thread * warp_size / SM100_REG_ALLOC_UNIT) * SM100_REG_ALLOC_UNIT
        limits["registers"] = (max_regs_per_sm // regs_per_warp) // warps_per_block
    total_smem = smem_bytes + dynamic_smem_bytes
    if total_smem > 0:
        if total_smem > SM100_MAX_SMEM_PER_BLOCK:
            return 0.0, 0, 0, "smem>227KiB"
        limits["smem"] = max_smem_per_sm // (total_smem + SM100_SMEM_RESERVED_PER_BLOCK)
    if tmem_columns > 0:
        limits["tmem"] = SM100_TMEM_COLUMNS // tmem_columns
    limiter = min(limits, key=lambda k: limits[k])
    blocks = max(0, min(limits.values()))
    warps = min(blocks * warps_per_block, max_warps_per_sm)
    return (warps / max_warps_per_sm if max_warps_per_sm else 0.0), warps, blocks, limiter


class OccupancyAnalyzer:
    """Occupancy from ptxas output for sm_100a kernels."""

    def __init__(self, arch: str = "sm_100a") -> None:
        self._arch = arch

    def compile_and_parse(self, src_path: Path, out_path: Optional[Path] = None,
                          extra_flags: Optional[list] = None) -> tuple[bool, dict[str, dict]]:
        """Compile `src_path` (shared library) and parse its ptxas report."""
        import build as kt_build
        out = out_path or Path(str(src_path) + ".occ.so")
        ok, stderr = kt_build.compile_shared(Path(src_path), out, extra_flags=extra_flags)
        parsed = parse_ptxas_stderr(stderr)
        if out_path is None and out.exists():
            out.unlink()
        return ok, parsed

    @staticmethod
    def _match(parsed: dict, kernel_function: str) -> Optional[dict]:
        entry = parsed.get(kernel_function)
        if entry is None:
            for name, data in parsed.items():
                if kernel_function in name:
                    entry = data
                    break
        return entry

    def analyze_from_stderr(self, stderr: str, kernel_function: str, block_size: int,
                            dynamic_smem_bytes: int = 0, tmem_columns: int = 0) -> Optional[OccupancyInfo]:
        """Occupancy of `kernel_function` (a substring of its mangled name) from captured ptxas output."""
        entry = self._match(parse_ptxas_stderr(stderr), kernel_function)
        if entry is None:
            return None
        return self._make_info(kernel_function, entry, block_size, dynamic_smem_bytes, tmem_columns)

    def analyze(self, src_path: Path, kernel_function: str, block_size: int,
                dynamic_smem_bytes: int = 0, tmem_columns: int = 0) -> Optional[OccupancyInfo]:
        ok, parsed = self.compile_and_parse(src_path)
        entry = self._match(parsed, kernel_function)
        if entry is None:
            return None
        return self._make_info(kernel_function, entry, block_size, dynamic_smem_bytes, tmem_columns)

    @staticmethod
    def _make_info(name: str, entry: dict, block_size: int, dyn: int = 0, tmem: int = 0) -> OccupancyInfo:
        regs = entry.get("registers", 0)
        smem = entry.get("smem_bytes", 0)
        occ, warps, blocks, limiter = occupancy_detail(regs, smem, block_size, dyn, tmem)
        return OccupancyInfo(
            kernel_name=name,
            registers_per_thread=regs,
            shared_mem_bytes=smem + dyn,
            spill_stores=entry.get("spill_stores", 0),
            spill_loads=entry.get("spill_loads", 0),
            has_register_spill=entry.get("spill_stores", 0) > 0,
            occupancy=occ,
            active_warps=warps,
            block_size=block_size,
            active_blocks=blocks,
            limiter=limiter,
            tmem_columns=tmem,
        )

    @staticmethod
    def print_table(rows: list, title: str = "Occupancy Analysis") -> None:
        print(f"\n{'=' * 80}\n  {title}\n{'=' * 80}")
        print(f"{'Config':<36} {'Occ%':>6} {'Regs':>5} {'SMEM':>8} {'Spill':>6} {'Speedup':>8}")
        print("-" * 80)
        for row in rows:
            if hasattr(row, "variant"):
                config, occ = row.variant[:35], row.occupancy or 0.0
                regs, smem = row.registers_per_thread or 0, row.shared_mem_bytes or 0
                spill = "YES" if row.has_register_spill else "no"
                speedup = f"{row.speedup:.2f}x" if row.speedup else "-"
            else:
                config, occ = row.kernel_name[:35], row.occupancy
                regs, smem = row.registers_per_thread, row.shared_mem_bytes
                spill, speedup = ("YES" if row.has_register_spill else "no"), "-"
            print(f"{config:<36} {occ * 100:>5.1f}% {regs:>5} {smem:>7}B {spill:>6} {speedup:>8}")
        print("=" * 80 + "\n")
