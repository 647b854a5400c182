"""Oracle for the reference operator `fp4_grouped_gemm` -- test infrastructure.

Restates kernels/gemm/fp4_grouped_gemm/b200/kernel.py:

  semantics (kernel.py:14-26), for a valid row i with g = m_indices[i] >= 0:
      C[i, j] = sum_k A_deq[i, k] * B_deq[g, j, k]
      A_deq[i, k]    = float(a[i, k]) * a_sf[i, k // 128]
      B_deq[g, j, k] = e2m1(nibble_k of b[g, j, k // 2]) * b_sf[g, j, k // 32]
  fp32 accumulation, bf16 output; padding rows (m_indices == -1) unchecked
  (kernel.py:31-33); expert segments start at multiples of 224 rows (:28-31).

  host repack (kernel.py:1006-1018, :2679-2741, :2780):
      exponent byte of an fp32 power of two = bits >> 23
      SF atom byte offset (r % 32) * 16 + ((r // 32) % 4) * 4 + j + (r // 128) * 512
      activation tiles [M_blocks, K_blocks, 1024] (224 rows, 1x128 scale x4)
      weight tiles     [G, N_blocks, K_blocks, 512]
      block -> expert  m_indices[::224].clamp_min(0)
"""
from __future__ import annotations

import numpy as np

from .nvfp4 import e2m1_decode, unpack_nibbles

BLOCK_M = 224  # kernel.py:274 (the alignment of every expert segment)
BLOCK_N = 128
BLOCK_K = 128
K_SUB = 4      # K=32 sub-blocks per 128-deep K block


def exponent_bytes(sf: np.ndarray) -> np.ndarray:
    """kernel.py:2679-2681: UE8M0 byte of an exact power of two."""
    bits = np.ascontiguousarray(sf, dtype=np.float32).view(np.int32)
    return (bits >> 23).astype(np.uint8)


def sf_offsets(rows: int, k_sub: int):
    """kernel.py:1006-1011: (row, sub-block, byte offset) of one blocked SF tile."""
    return [(r, j, (r % 32) * 16 + ((r // 32) % 4) * 4 + j + (r // 128) * 512)
            for r in range(rows) for j in range(k_sub)]


def sf_tile_bytes(rows: int, k_sub: int) -> int:
    """kernel.py:1014-1018: whole 128-row atoms."""
    return ((rows + 127) // 128) * 128 * k_sub


def pack_sf_act(a_sf: np.ndarray, num_m_blocks: int, num_k_blocks: int) -> np.ndarray:
    """kernel.py:2691-2707: activation scales -> [MB, KB, 1024] blocked tiles,
    the 1x128 byte replicated into the four K32 slots."""
    eb = exponent_bytes(a_sf)                       # [M_total, KB]
    m_total = eb.shape[0]
    cos = sf_tile_bytes(BLOCK_M, K_SUB)
    out = np.zeros((num_m_blocks, num_k_blocks, cos), dtype=np.uint8)
    for r, j, off in sf_offsets(BLOCK_M, K_SUB):
        rows = np.minimum(np.arange(num_m_blocks) * BLOCK_M + r, m_total - 1)
        out[:, :, off] = eb[rows, :num_k_blocks]
    return out


def pack_sf_wgt(b_sf: np.ndarray, num_n_blocks: int, num_k_blocks: int) -> np.ndarray:
    """kernel.py:2709-2741: weight scales -> [G, NB, KB, 512] blocked tiles."""
    g = b_sf.shape[0]
    eb = exponent_bytes(b_sf).reshape(g, num_n_blocks, BLOCK_N, num_k_blocks, K_SUB)
    out = np.zeros((g, num_n_blocks, num_k_blocks, sf_tile_bytes(BLOCK_N, K_SUB)), dtype=np.uint8)
    for r, j, off in sf_offsets(BLOCK_N, K_SUB):
        out[:, :, :, off] = eb[:, :, r, :, j]
    return out


def block_expert(m_indices: np.ndarray) -> np.ndarray:
    """kernel.py:2780: the expert of every 224-row block."""
    return np.maximum(np.asarray(m_indices, dtype=np.int32)[::BLOCK_M], 0).astype(np.int32)


def e4m3fn_decode(a: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bytes -> fp32 (sign, 4-bit exponent bias 7, 3-bit mantissa)."""
    b = np.asarray(a, dtype=np.uint8).astype(np.uint32)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    val = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8) * np.exp2(e.astype(np.float64) - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


def dequant_act(a_bytes: np.ndarray, a_sf: np.ndarray) -> np.ndarray:
    """A_deq[i, k] = float(a[i, k]) * a_sf[i, k // 128]."""
    x = e4m3fn_decode(a_bytes)
    return (x * np.repeat(np.asarray(a_sf, np.float32), 128, axis=1)).astype(np.float32)


def dequant_wgt(b: np.ndarray, b_sf: np.ndarray) -> np.ndarray:
    """B_deq[g, j, k] = e2m1(nibble_k) * b_sf[g, j, k // 32]."""
    vals = e2m1_decode(unpack_nibbles(b))
    return (vals * np.repeat(np.asarray(b_sf, np.float32), 32, axis=-1)).astype(np.float32)


def fp4_grouped_gemm(a, a_sf, b, b_sf, m_indices, as_bf16: bool = True):
    """Reference semantics of kernel.py:2788 on numpy inputs (a: e4m3 bytes).
    Rows with m_indices == -1 are returned as zeros (their value is unchecked)."""
    import torch

    m_total = a.shape[0]
    n = b.shape[1]
    ad = torch.from_numpy(dequant_act(a, a_sf))
    c = torch.zeros((m_total, n), dtype=torch.float32)
    mi = np.asarray(m_indices, dtype=np.int64)
    for g in range(b.shape[0]):
        rows = np.nonzero(mi == g)[0]
        if rows.size == 0:
            continue
        bd = torch.from_numpy(dequant_wgt(b[g], b_sf[g]))
        c[torch.from_numpy(rows)] = ad[torch.from_numpy(rows)] @ bd.T
    return c.to(torch.bfloat16) if as_bf16 else c


def random_problem(group_rows, n: int, k: int, seed: int = 0):
    """Seeded MX problem in the reference's layout: each expert segment padded
    to a multiple of 224 rows with m_indices = -1 rows.  Activations e4m3 from
    N(0,1) clamped to +-2 (leaderboard.py:599-601), weights random E2M1 codes,
    scales random powers of two."""
    import torch

    rng = np.random.default_rng(seed)
    g = len(group_rows)
    idx = []
    for e, r in enumerate(group_rows):
        pad = (-r) % BLOCK_M
        idx += [e] * r + [-1] * pad
    m_indices = np.array(idx, dtype=np.int32)
    m_total = m_indices.size
    x = np.clip(rng.standard_normal((m_total, k), dtype=np.float32), -2, 2)
    a = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    a_sf = np.exp2(rng.integers(-3, 4, size=(m_total, k // 128))).astype(np.float32)
    b = rng.integers(0, 256, size=(g, n, k // 2), dtype=np.uint8)
    b_sf = np.exp2(rng.integers(-4, 3, size=(g, n, k // 32))).astype(np.float32)
    return {"a": a, "a_sf": a_sf, "b": b, "b_sf": b_sf, "m_indices": m_indices}


# ----------------------------------------------- campaign-point inputs
# The reference's own campaign point (kernel.py:1-8, :213, :286): G = 8
# experts x 4096 rows, each segment padded to a multiple of 224 rows,
# N = K = 4096.  Every 224-row block of activations and the weight tensor come
# from their own seeded streams, so any block can be regenerated alone (the
# CPU checks of the golden rows rebuild only the blocks they need).
CAMPAIGN_ROWS = (4096,) * 8
CAMPAIGN_N = 4096
CAMPAIGN_K = 4096


def campaign_m_indices(group_rows=CAMPAIGN_ROWS) -> np.ndarray:
    idx = []
    for e, r in enumerate(group_rows):
        idx += [e] * r + [-1] * ((-r) % BLOCK_M)
    return np.array(idx, dtype=np.int32)


def campaign_act_block(seed: int, xb: int, k: int = CAMPAIGN_K):
    """Activation rows [224 * xb, 224 * xb + 224): e4m3 bytes of N(0,1) clamped
    to +-2 (the reference evaluator's FP8 draw, leaderboard.py:599-601) and
    power-of-two 1x128 scales in [2^-3, 2^3]."""
    import torch

    rng = np.random.default_rng([seed, 1, xb])
    x = np.clip(rng.standard_normal((BLOCK_M, k), dtype=np.float32), -2, 2)
    a = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    a_sf = np.exp2(rng.integers(-3, 4, size=(BLOCK_M, k // 128))).astype(np.float32)
    return a, a_sf


def campaign_weights(seed: int, g: int = 8, n: int = CAMPAIGN_N, k: int = CAMPAIGN_K):
    """Expert weights: random packed E2M1 codes and power-of-two 1x32 scales in
    [2^-4, 2^2]."""
    rng = np.random.default_rng([seed, 2])
    b = rng.integers(0, 256, size=(g, n, k // 2), dtype=np.uint8)
    b_sf = np.exp2(rng.integers(-4, 3, size=(g, n, k // 32))).astype(np.float32)
    return b, b_sf


def campaign_problem(seed: int, group_rows=CAMPAIGN_ROWS, n: int = CAMPAIGN_N,
                     k: int = CAMPAIGN_K) -> dict:
    m_indices = campaign_m_indices(group_rows)
    blocks = [campaign_act_block(seed, xb, k) for xb in range(m_indices.size // BLOCK_M)]
    b, b_sf = campaign_weights(seed, len(group_rows), n, k)
    return {"a": np.concatenate([x for x, _ in blocks]),
            "a_sf": np.concatenate([s for _, s in blocks]),
            "b": b, "b_sf": b_sf, "m_indices": m_indices}


def campaign_rows_output(seed: int, rows, group_rows=CAMPAIGN_ROWS, n: int = CAMPAIGN_N,
                         k: int = CAMPAIGN_K, as_bf16: bool = True):
    """The oracle's output for the given (valid) rows of the campaign problem,
    regenerating only the activation blocks those rows live in."""
    import torch

    m_indices = campaign_m_indices(group_rows)
    b, b_sf = campaign_weights(seed, len(group_rows), n, k)
    rows = np.asarray(rows, dtype=np.int64)
    out = torch.zeros((rows.size, n), dtype=torch.float32)
    blocks = {}
    for xb in np.unique(rows // BLOCK_M):
        blocks[int(xb)] = campaign_act_block(seed, int(xb), k)
    a = np.stack([blocks[int(r // BLOCK_M)][0][r % BLOCK_M] for r in rows])
    a_sf = np.stack([blocks[int(r // BLOCK_M)][1][r % BLOCK_M] for r in rows])
    ad = torch.from_numpy(dequant_act(a, a_sf))
    for g in np.unique(m_indices[rows]):
        sel = np.nonzero(m_indices[rows] == g)[0]
        bd = torch.from_numpy(dequant_wgt(b[g], b_sf[g]))
        out[torch.from_numpy(sel)] = ad[torch.from_numpy(sel)] @ bd.T
    return out.to(torch.bfloat16) if as_bf16 else out
