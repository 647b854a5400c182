"""Generate tests/golden/mx_reference_rows.npz from the reference's own kernel.

Runs the unmodified reference operator `fp4_grouped_gemm`
(kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788-2862, from the reference
install under baseline/_ref) on one B200 at the reference's campaign point --
8 experts x 4096 rows padded to 224-row segments, N = K = 4096 -- with the
block-seeded inputs of oracle/mx.py (`campaign_problem`, seed 2026), and keeps
48 of its output rows: in each expert segment the first two rows, the last
row of the first 224-row block and the first of the second, the middle row and
the last valid row.  The CPU test pins the oracle to these rows, the GPU test
pins this repository's kernel to them.

    python tests/golden/make_mx_reference.py OUT.npz     (on a B200)
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from oracle import mx as mref  # noqa: E402


def golden_rows() -> np.ndarray:
    mi = mref.campaign_m_indices()
    rows = []
    for e in range(len(mref.CAMPAIGN_ROWS)):
        seg = np.flatnonzero(mi == e)
        s0, n = int(seg[0]), int(seg.size)
        rows += [s0, s0 + 1, s0 + 223, s0 + 224, s0 + n // 2, s0 + n - 1]
    return np.asarray(rows, dtype=np.int64)


def main(argv) -> int:
    if len(argv) != 2:
        raise SystemExit(__doc__)
    mod, why = bench.load_reference_kernel()
    if mod is None:
        raise SystemExit(why)
    dev = torch.device("cuda", 0)
    args, prob = bench.mx_campaign_on_device(dev)
    c = mod.fp4_grouped_gemm(*args)
    torch.cuda.synchronize()
    rows = golden_rows()
    out = c.index_select(0, torch.from_numpy(rows).to(dev)).cpu()
    import cutlass

    np.savez_compressed(
        argv[1], seed=np.int64(bench.MX_CAMPAIGN_SEED), rows=rows,
        out_bf16_bits=out.view(torch.int16).numpy(),
        kernel_sha256=hashlib.sha256(bench.REF_KERNEL.read_bytes()).hexdigest(),
        cutlass_dsl=str(getattr(cutlass, "__version__", "unknown")),
        device=torch.cuda.get_device_name(dev))
    print("wrote", argv[1], out.shape)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
