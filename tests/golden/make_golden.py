"""Generate the golden fixtures in this directory from the reference itself.

Runs only where the reference checkout is mounted (pass its path, or set
RATCHET_REFERENCE); the GPU box and the tests use the committed .npz files.

  e2m1_cast.npz   inputs + packed codes of the reference evaluator's FP4 cast
                  (src/forgekernel/card_template/eval/leaderboard.py:608-627,
                  `_cast_to_fp4x2`): pins the E2M1 rounding (ties, -0, saturation)
  mx_sf_pack.npz  inputs + outputs of the reference kernel module's host repack
                  (kernels/gemm/fp4_grouped_gemm/b200/kernel.py `_exponent_bytes`
                  :2679, `_pack_sf_act` :2691, `_pack_sf_wgt` :2709, the
                  block->expert table :2780): pins the SF atom layout

    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(path.parent))
    spec.loader.exec_module(mod)
    return mod


def make_e2m1(ref_root: Path):
    lb = _load(ref_root / "src/forgekernel/card_template/eval/leaderboard.py", "ref_leaderboard")
    ties = [0.0, -0.0, 0.25, -0.25, 0.2500001, 0.75, -0.75, 0.7499999, 1.25, 1.2500001, 1.75,
            -1.75, 2.5, 2.5000002, 3.5, -3.5, 5.0, 5.0000005, 6.0, 7.0, -100.0, 0.1, -0.1,
            0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -4.0, 1e-8, -1e-8]
    rng = np.random.default_rng(20240601)
    rand = (rng.standard_normal(4096).astype(np.float32) * np.float32(2.5))
    x = np.concatenate([np.array(ties, dtype=np.float32), rand]).astype(np.float32)
    if x.size % 2:
        x = np.append(x, np.float32(0.0))
    packed = lb._cast_to_fp4x2(torch.from_numpy(x)).view(torch.uint8).numpy()
    np.savez_compressed(HERE / "e2m1_cast.npz", x=x, packed=packed)
    print("e2m1_cast.npz", x.shape, packed.shape)


def make_mx_sf(ref_root: Path):
    km = _load(ref_root / "kernels/gemm/fp4_grouped_gemm/b200/kernel.py", "ref_fgg_kernel")
    rng = np.random.default_rng(7)
    g, n, k = 3, 256, 512
    rows = [300, 0, 250]  # expert 1 owns zero rows
    idx = []
    for e, r in enumerate(rows):
        idx += [e] * r + [-1] * ((-r) % km.BLOCK_M)
    m_indices = np.array(idx, dtype=np.int32)
    m_total = m_indices.size
    a_sf = np.exp2(rng.integers(-6, 7, size=(m_total, k // 128))).astype(np.float32)
    b_sf = np.exp2(rng.integers(-6, 7, size=(g, n, k // 32))).astype(np.float32)
    nmb = (m_total + km.BLOCK_M - 1) // km.BLOCK_M
    nnb = n // km.BLOCK_N
    nkb = k // km.BLOCK_K
    ta, tb, tm = torch.from_numpy(a_sf), torch.from_numpy(b_sf), torch.from_numpy(m_indices)
    sf_act = km._pack_sf_act(ta, nmb, nkb, km.K_SUB).numpy()
    sf_wgt = km._pack_sf_wgt(tb, nnb, nkb, km.K_SUB).numpy()
    eb = km._exponent_bytes(ta).numpy()
    blk = tm[::km.BLOCK_M].to(torch.int32).clamp_min(0).numpy()
    offs = np.array(km._sf_offsets(224, 4), dtype=np.int64)
    np.savez_compressed(HERE / "mx_sf_pack.npz", a_sf=a_sf, b_sf=b_sf, m_indices=m_indices,
                        sf_act=sf_act, sf_wgt=sf_wgt, exp_bytes=eb, blk_expert=blk,
                        sf_offsets_224x4=offs, g=g, n=n, k=k,
                        block_m=km.BLOCK_M, block_n=km.BLOCK_N, block_k=km.BLOCK_K)
    print("mx_sf_pack.npz", sf_act.shape, sf_wgt.shape, blk)


def main(argv):
    # the reference checkout: first argument, else $RATCHET_REFERENCE
    arg = argv[1] if len(argv) > 1 else os.environ.get("RATCHET_REFERENCE")
    if not arg:
        raise SystemExit("usage: make_golden.py <reference checkout> "
                         "(or set RATCHET_REFERENCE)")
    ref_root = Path(arg)
    if not ref_root.exists():
        raise SystemExit(f"reference checkout not found at {ref_root}")
    make_e2m1(ref_root)
    make_mx_sf(ref_root)


if __name__ == "__main__":
    main(sys.argv)
