"""NVFP4 oracle (numpy; torch only for the large fp32 matmul) -- test infrastructure.

Format (restated from the reference):
  * E2M1 code = sign bit 3 + magnitude index into {0, 0.5, 1, 1.5, 2, 3, 4, 6}
    (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:22-26).
  * Two codes per byte, element 2j in the LOW nibble of byte j (kernel.py:22-24;
    tasks/muse_prefill_boundary/reference/submission.py:538-542 `_codes`).
  * One E4M3 scale per 16 contiguous K elements and one fp32 per-tensor
    (decode) scale g: x = e2m1(q) * e4m3(s) * g
    (submission.py:1847-1880, the NVFP4 decode of the Muse expert weights).

Quantisation recipe (fixed so the device quantiser matches it bit for bit):
  gs  = 2688 / amax          (2688 = 448 * 6; 1 when amax == 0), g = 1 / gs
  s   = e4m3_rn_satfinite((blockmax / 6) * gs)
  q   = e2m1_rne(x * (gs / float(s)))      (0 where s == 0)
E2M1 rounding uses the thresholds of the SOL-ExecBench FP4 cast carried by the
reference evaluator (src/forgekernel/card_template/eval/leaderboard.py:608-627):
round to nearest, ties to the even code, saturate at 6, sign from x < 0.

GEMM semantics: C_g = alpha_g * (deq(A_g) @ deq(B_g)^T), deq = e2m1 x e4m3
(no global scale), alpha_g = gA_g * gB_g, fp32 accumulation, bf16 output.
"""
from __future__ import annotations

import numpy as np

E2M1_MAGNITUDES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
# code -> value, codes 8..15 negative (8 is -0)
E2M1_VALUES = np.concatenate([E2M1_MAGNITUDES, -E2M1_MAGNITUDES]).astype(np.float32)

# Upper edges of the magnitude bins and whether the edge itself rounds down
# (leaderboard.py:611-619: `x <= 0.25` -> 0, `x < 0.75` -> 1, `x <= 1.25` -> 2,
# `x < 1.75` -> 3, `x <= 2.5` -> 4, `x < 3.5` -> 5, `x <= 5.0` -> 6, else 7).
_E2M1_EDGES = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
_E2M1_EDGE_INCLUSIVE = np.array([True, False, True, False, True, False, True])


def e2m1_encode(y: np.ndarray) -> np.ndarray:
    """fp32 -> E2M1 codes (uint8 in [0, 15]), RNE on codes, saturating at 6."""
    y = np.asarray(y, dtype=np.float32)
    a = np.abs(y)
    # searchsorted 'left' counts edges strictly below a; an inclusive edge equal
    # to a must not be counted, an exclusive one must.
    mag = np.searchsorted(_E2M1_EDGES, a, side="left").astype(np.uint8)
    at_edge = np.zeros(a.shape, dtype=bool)
    idx = np.minimum(mag, len(_E2M1_EDGES) - 1)
    at_edge = (_E2M1_EDGES[idx] == a) & (mag < len(_E2M1_EDGES))
    bump = at_edge & ~_E2M1_EDGE_INCLUSIVE[idx]
    mag = mag + bump.astype(np.uint8)
    sign = (y < 0).astype(np.uint8) << 3
    return (mag | sign).astype(np.uint8)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    return E2M1_VALUES[np.asarray(codes, dtype=np.uint8) & 15]


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[..., K] codes -> [..., K/2] bytes, element 2j in the low nibble."""
    c = np.asarray(codes, dtype=np.uint8)
    assert c.shape[-1] % 2 == 0
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """[..., K/2] bytes -> [..., K] codes (submission.py:538-542)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 15
    out[..., 1::2] = p >> 4
    return out


# ----------------------------------------------------------------- E4M3 (fn)
def _e4m3_table() -> np.ndarray:
    """Values of the non-negative finite E4M3 bytes 0x00..0x7E."""
    b = np.arange(0x7F, dtype=np.uint32)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    sub = m * 2.0 ** -9
    norm = (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7.0)
    return np.where(e == 0, sub, norm).astype(np.float32)


E4M3_TABLE = _e4m3_table()  # strictly increasing, max 448


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """Non-negative E4M3 bytes -> fp32 (scales are never negative here)."""
    b = np.asarray(b, dtype=np.uint8)
    return E4M3_TABLE[np.minimum(b & 0x7F, 0x7E)]


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """Non-negative fp32 -> E4M3 byte, round to nearest even, saturate at 448."""
    v = np.asarray(v, dtype=np.float32)
    t = E4M3_TABLE
    hi = np.clip(np.searchsorted(t, v, side="left"), 0, len(t) - 1)
    lo = np.maximum(hi - 1, 0)
    dlo = np.abs(v.astype(np.float64) - t[lo])
    dhi = np.abs(t[hi].astype(np.float64) - v)
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(v >= t[-1], len(t) - 1, code)
    return code.astype(np.uint8)


# ------------------------------------------------------------- quantisation
def global_encode_scale(amax: float) -> np.float32:
    amax = np.float32(amax)
    return np.float32(2688.0) / amax if amax > 0 else np.float32(1.0)


def nvfp4_quantize(x: np.ndarray, amax: float | None = None):
    """Row-major [rows, K] fp32 -> (codes [rows, K/2] u8, sf [rows, K/16] u8, g fp32).

    `g` is the per-tensor decode scale (1 / gs) that goes into alpha."""
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    assert k % 16 == 0
    if amax is None:
        amax = float(np.abs(x).max()) if x.size else 0.0
    gs = global_encode_scale(amax)
    blk = x.reshape(rows, k // 16, 16)
    bmax = np.abs(blk).max(axis=-1)
    sval = (bmax / np.float32(6.0)).astype(np.float32) * gs
    sf = e4m3_encode(sval.astype(np.float32))
    sdec = e4m3_decode(sf)
    with np.errstate(divide="ignore"):
        inv = np.where(sdec == 0, np.float32(0.0), gs / np.where(sdec == 0, 1, sdec)).astype(np.float32)
    y = (blk * inv[..., None]).astype(np.float32)
    codes = e2m1_encode(y).reshape(rows, k)
    return pack_nibbles(codes), sf, np.float32(np.float32(1.0) / gs)


def nvfp4_dequantize(codes: np.ndarray, sf: np.ndarray, g: float = 1.0) -> np.ndarray:
    """(codes [rows, K/2], sf [rows, K/16]) -> fp32 [rows, K] = e2m1 * e4m3 * g."""
    vals = e2m1_decode(unpack_nibbles(codes))
    rows, k = vals.shape
    s = e4m3_decode(sf).astype(np.float32)
    out = vals.reshape(rows, k // 16, 16) * s[..., None]
    return (out.reshape(rows, k) * np.float32(g)).astype(np.float32)


# ------------------------------------------------------------ grouped GEMM
def grouped_gemm(a_list, a_sf_list, b_list, b_sf_list, alpha, as_bf16: bool = True):
    """Reference grouped GEMM: per group alpha_g * deq(A_g) @ deq(B_g)^T.

    Inputs are numpy arrays (codes, E4M3 bytes).  The products are exact in
    fp32 and accumulated by torch's fp32 CPU matmul; the result is rounded to
    bf16 once (returned as a torch bfloat16 tensor, or fp32 if as_bf16=False).
    """
    import torch

    outs = []
    for g in range(len(a_list)):
        a = torch.from_numpy(nvfp4_dequantize(a_list[g], a_sf_list[g]))
        b = torch.from_numpy(nvfp4_dequantize(b_list[g], b_sf_list[g]))
        c = (a @ b.T) * float(np.float32(alpha[g]))
        outs.append(c.to(torch.bfloat16) if as_bf16 else c)
    return outs


def gated_grouped_gemm(a_list, a_sf_list, b13_list, b13_sf_list, alpha):
    """Reference of the gated gate+up epilogue: per group, with b13 rows
    [0, I) the gate projection and [I, 2I) the up projection,
        hh = alpha_g * deq(A_g) @ deq(B13_g)^T          (fp32)
        h  = bf16(silu(hh[:, :I]) * hh[:, I:])
    (tasks/muse_prefill_boundary/reference/submission.py:1096, the reference's
    own check of its fused SiLU * up epilogue)."""
    import torch

    outs = []
    for c in grouped_gemm(a_list, a_sf_list, b13_list, b13_sf_list, alpha, as_bf16=False):
        i = c.shape[1] // 2
        outs.append((torch.nn.functional.silu(c[:, :i]) * c[:, i:]).to(torch.bfloat16))
    return outs


def random_problem(m_list, n: int, k: int, seed: int = 0, w_std: float = 1.0):
    """Seeded synthetic NVFP4 problem: N(0,1) activations, N(0, w_std) weights,
    each tensor quantised with its own global scale.  Returns a dict of numpy
    arrays: a, a_sf, b, b_sf (lists), alpha (fp32 [G]), plus the fp32 sources
    are not kept (they are not needed for parity)."""
    rng = np.random.default_rng(seed)
    out = {"a": [], "a_sf": [], "b": [], "b_sf": [], "alpha": [], "m": list(m_list)}
    for m in m_list:
        x = rng.standard_normal((m, k), dtype=np.float32)
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(w_std)).astype(np.float32)
        qa, sa, ga = nvfp4_quantize(x) if m > 0 else (np.zeros((0, k // 2), np.uint8), np.zeros((0, k // 16), np.uint8), np.float32(1.0))
        qb, sb, gb = nvfp4_quantize(w)
        out["a"].append(qa)
        out["a_sf"].append(sa)
        out["b"].append(qb)
        out["b_sf"].append(sb)
        out["alpha"].append(np.float32(ga * gb))
    out["alpha"] = np.array(out["alpha"], dtype=np.float32)
    return out


def check_close(got, ref, rel_max: float = 1e-2, rtol: float = 2e-2, atol_frac: float = 1e-2):
    """Tolerance of the operator: max|err| / max|ref| <= rel_max, and per element
    |err| <= rtol * |ref| + atol_frac * max|ref|.  Returns (ok, stats)."""
    import torch

    g = got.float()
    r = ref.float()
    if g.shape != r.shape:
        return False, {"error": f"shape {tuple(g.shape)} != {tuple(r.shape)}"}
    if g.numel() == 0:
        return True, {"max_abs": 0.0, "rel": 0.0, "bad": 0}
    if not torch.isfinite(g).all():
        return False, {"error": "non-finite output"}
    d = (g - r).abs()
    scale = float(r.abs().max())
    rel = float(d.max()) / scale if scale > 0 else float(d.max())
    bad = int((d > rtol * r.abs() + atol_frac * scale).sum())
    ok = rel <= rel_max and bad == 0
    return ok, {"max_abs": float(d.max()), "rel": rel, "bad": bad, "max_ref": scale}


def nvfp4_dequantize_torch(codes, sf, g: float = 1.0):
    """Same values as nvfp4_dequantize, computed with torch CPU ops (all host
    threads); used by the timed CPU baseline.  codes/sf: uint8 torch tensors."""
    import torch

    lut = torch.from_numpy(E2M1_VALUES)
    lo = (codes & 15).long()
    hi = (codes >> 4).long()
    rows, half = codes.shape
    vals = torch.stack((lut[lo], lut[hi]), dim=-1).reshape(rows, half * 2)
    s = torch.from_numpy(E4M3_TABLE)[torch.clamp(sf.long() & 0x7F, max=0x7E)]
    out = (vals.reshape(rows, -1, 16) * s.unsqueeze(-1)).reshape(rows, half * 2)
    return out * float(np.float32(g)) if g != 1.0 else out
