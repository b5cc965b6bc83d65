"""
make_golden.py — regenerate tests/golden/reference_kat.npz from the reference's
own NumPy oracle.

It imports `verifier.py` read-only from the reference checkout's `src/`
directory, named by the first argument or $KT_REFERENCE_SRC (there is no
default), calls its `_ref_*` functions at the
sizes of its verify mains (src/verifier.py:221-294, :542-556) and stores the
outputs. The reference cannot travel to the GPU machine; these fixtures do.

    python tests/golden/make_golden.py <reference-checkout>/src
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

sys.dont_write_bytecode = True  # the reference tree is read-only

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_kat.npz"


def main() -> None:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KT_REFERENCE_SRC")
    if not arg:
        raise SystemExit("usage: make_golden.py <reference src/ directory> (or set KT_REFERENCE_SRC)")
    src = Path(arg)
    if not (src / "verifier.py").exists():
        raise SystemExit(f"reference verifier not found under {src}")
    sys.path.insert(0, str(src))
    import verifier  # noqa: E402  (the reference module; no import side effects)

    data = {
        "matmul_N64": verifier._ref_matmul(N=64).astype(np.float32),
        "softmax_4x16": verifier._ref_softmax(rows=4, cols=16).astype(np.float32),
        "layernorm_4x16": verifier._ref_layernorm(rows=4, cols=16).astype(np.float32),
        "attention_S512_D64": verifier._ref_attention(S=512, D=64).astype(np.float32),
        "tolerances": np.array([verifier._TOLERANCES[k] for k in
                                ("matmul", "softmax", "reduction", "layernorm", "attention")],
                               dtype=np.float64),
    }
    for blk in (64, 128, 192, 256):
        data[f"reduction_N256_blk{blk}"] = verifier._ref_reduction(N=256, block_size=blk).astype(np.float32)
    # The verifier's own comparison helper, exercised on a planted difference.
    d, ok = verifier.CorrectnessVerifier._compare(np.array([1.0, 2.0], np.float32),
                                                   np.array([1.0, 2.5], np.float32), 1e-3)
    data["compare_probe"] = np.array([d, float(ok)], dtype=np.float64)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes): {sorted(data)}")


if __name__ == "__main__":
    main()
