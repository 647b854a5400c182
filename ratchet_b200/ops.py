"""Host-side mirror of the reference operator API, over the C ABI.

Two operators:

* `nvfp4_grouped_gemm(a_list, a_sf_list, b_list, b_sf_list, problem_sizes, alpha)`
  -> one bf16 [M_g, N] output per group (views of one buffer).  NVFP4 x NVFP4:
  E2M1 codes packed two per byte, one E4M3 scale per 16 K, fp32 alpha_g
  (= product of the two per-tensor global decode scales).

* `fp4_grouped_gemm(a, a_sf, b, b_sf, m_indices) -> c`, the reference's own
  signature and semantics (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788-2862):
  MXFP8 activations x MXFP4 expert weights, contiguous M grouping.

Caching follows the reference's identity discipline (kernel.py:2743-2786): a
key of (data_ptr, shape, stride, dtype, device, _version) per source tensor,
and the cache entry holds the source tensors so their addresses cannot be
recycled while it lives.  Like the reference, the caches are not thread-safe.

Everything runs on the current CUDA stream; nothing here synchronises the host.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Sequence

import numpy as np
import torch

from . import _lib

_U8_DTYPES = {torch.uint8, torch.int8, torch.float8_e4m3fn}
if hasattr(torch, "float4_e2m1fn_x2"):
    _U8_DTYPES.add(torch.float4_e2m1fn_x2)

_CACHE_MAX = 8


def _identity(t: torch.Tensor):
    return (int(t.data_ptr()), tuple(t.shape), tuple(t.stride()), str(t.dtype), str(t.device),
            int(getattr(t, "_version", 0)))


def _as_u8(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype not in _U8_DTYPES:
        raise ValueError(f"{name}: dtype {t.dtype} is not a byte type (uint8/int8/float8/float4x2)")
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_get_device = getattr(torch._C, "_cuda_getDevice", None)
_capturing = getattr(torch._C, "_cuda_isCurrentStreamCapturing", None)


def _stream_ptr(device: torch.device) -> int:
    if _raw_stream is not None and device.index is not None:
        return int(_raw_stream(device.index))
    return int(torch.cuda.current_stream(device).cuda_stream)


def _is_current(device: torch.device) -> bool:
    """True when `device` is the current CUDA device (no context switch needed)."""
    cur = _get_device() if _get_device is not None else torch.cuda.current_device()
    return device.index is None or device.index == cur


# Workspaces reused per (device, stream): calls on one stream are ordered, so
# the next call's prepare kernel (which waits for the previous GEMM before it
# touches memory) may overwrite the previous call's workspace.  Not used while
# the stream is being captured into a CUDA graph (the graph keeps its own).
_WS: OrderedDict = OrderedDict()
_WS_MAX = 8


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    if _capturing is not None and _capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=device)
    key = (device.index, stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = ws
        while len(_WS) > _WS_MAX:  # the oldest stream's buffer returns to torch's allocator
            _WS.popitem(last=False)
    else:
        _WS.move_to_end(key)
    return ws


# Host arrays for the per-group problem description, reused per group count
# (the C ABI reads them during the call only).
_SCRATCH: dict = {}


def _scratch(G: int):
    sc = _SCRATCH.get(G)
    if sc is None:
        sc = (np.empty(G, dtype=np.int32), np.empty(G, dtype=np.uint64),
              np.empty(G, dtype=np.uint64))
        _SCRATCH[G] = sc
    return sc


def _ptr_array(tensors) -> np.ndarray:
    return np.fromiter((t.data_ptr() for t in tensors), dtype=np.uint64, count=len(tensors))


class _LRU(OrderedDict):
    def get_or(self, key, make):
        hit = self.get(key)
        if hit is not None:
            self.move_to_end(key)
            return hit
        val = make()
        while len(self) >= _CACHE_MAX:
            self.popitem(last=False)
        self[key] = val
        return val


_PACKS = _LRU()
_MX_PREP = _LRU()
_last_ws: torch.Tensor | None = None


class WeightPack:
    """Device-side packed weights of one NVFP4 group list: per-group TMA
    descriptors plus the scales in the MMA's 512-byte SF atoms."""

    def __init__(self, b_list: Sequence[torch.Tensor], b_sf_list: Sequence[torch.Tensor]):
        if len(b_list) != len(b_sf_list) or not b_list:
            raise ValueError("b_list and b_sf_list must be non-empty and of equal length")
        G = len(b_list)
        if G > _lib.FGG_MAX_GROUPS:
            raise ValueError(f"{G} groups > FGG_MAX_GROUPS={_lib.FGG_MAX_GROUPS}")
        b0 = b_list[0]
        if b0.dim() != 2:
            raise ValueError(f"b[0] must be 2-D [N, K/2], got {tuple(b0.shape)}")
        n, k = int(b0.shape[0]), int(b0.shape[1]) * 2
        bs, sfs = [], []
        for g, (b, s) in enumerate(zip(b_list, b_sf_list)):
            b = _as_u8(b, f"b[{g}]")
            s = _as_u8(s, f"b_sf[{g}]")
            if tuple(b.shape) != (n, k // 2):
                raise ValueError(f"b[{g}] has shape {tuple(b.shape)}, expected {(n, k // 2)}")
            if tuple(s.shape) != (n, k // 16):
                raise ValueError(f"b_sf[{g}] has shape {tuple(s.shape)}, expected {(n, k // 16)}")
            if not (b.is_cuda and s.is_cuda and b.is_contiguous() and s.is_contiguous()):
                raise ValueError(f"group {g}: weights must be contiguous CUDA tensors")
            bs.append(b)
            sfs.append(s)
        self.G, self.n, self.k = G, n, k
        self.device = b0.device
        # The pack keeps its source tensors alive, so their id()s stay unique
        # while it is cached; their version counters reveal in-place writes.
        self.sources = (tuple(b_list), tuple(b_sf_list))
        self.versions = _versions(b_list, b_sf_list)
        L = _lib.lib()
        nbytes = int(L.fgg_nvfp4_weight_pack_bytes(G, n, k))
        if nbytes == 0:
            raise ValueError(f"unsupported weight geometry G={G} N={n} K={k}")
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        pb, psf = _ptr_array(bs), _ptr_array(sfs)
        w = _lib.FggNvfp4Weights(G, n, k, pb.ctypes.data, psf.ctypes.data)
        with torch.cuda.device(self.device):
            _lib.check(L.fgg_nvfp4_pack_weights(w, self.buf.data_ptr(), nbytes,
                                                _stream_ptr(self.device)),
                       "fgg_nvfp4_pack_weights")


def _versions(b_list, b_sf_list) -> list[int]:
    return [t._version for t in b_list] + [t._version for t in b_sf_list]


def pack_weights(b_list, b_sf_list) -> WeightPack:
    """Packed weights for these tensors, cached on tensor identity: the same
    tensor objects, unmodified since the pack was built (version counters)."""
    key = (tuple(map(id, b_list)), tuple(map(id, b_sf_list)))
    hit = _PACKS.get(key)
    if hit is not None and hit.versions == _versions(b_list, b_sf_list):
        _PACKS.move_to_end(key)
        return hit
    if hit is not None:
        del _PACKS[key]
    return _PACKS.get_or(key, lambda: WeightPack(b_list, b_sf_list))


def nvfp4_grouped_gemm(a_list, a_sf_list, b_list, b_sf_list, problem_sizes=None, alpha=None,
                       *, pack: WeightPack | None = None, out: torch.Tensor | None = None,
                       b_index=None) -> list[torch.Tensor]:
    """Per group g: C_g = alpha_g * deq(A_g) @ deq(B_g)^T as bf16 [M_g, N].

    a_list[g]    [M_g, K/2]  packed E2M1 codes (uint8 / float4_e2m1fn_x2)
    a_sf_list[g] [M_g, K/16] E4M3 scales (float8_e4m3fn / uint8), row-major
    b_list[g]    [N, K/2], b_sf_list[g] [N, K/16]  (packed once, cached)
    problem_sizes  G rows of (M_g, N, K), checked against the tensors
    alpha        G floats or an fp32 tensor (default 1)
    out          optional contiguous bf16 [sum M_g, N] on the weights' device;
                 the returned per-group tensors are row slices of it
    b_index      optional: problem group g multiplies with weight group
                 b_index[g] (b_list then holds the weight groups, any count);
                 several problem groups may share one weight group
    """
    return _nvfp4_grouped(a_list, a_sf_list, b_list, b_sf_list, problem_sizes, alpha, pack, out,
                          b_index, silu_mul=False)


def nvfp4_grouped_gemm_silu_mul(a_list, a_sf_list, b_list, b_sf_list, problem_sizes=None,
                                alpha=None, *, pack: WeightPack | None = None,
                                out: torch.Tensor | None = None, b_index=None) -> list[torch.Tensor]:
    """Fused gate+up projection with the SiLU * up epilogue (the gated expert
    path of tasks/muse_prefill_boundary/reference/submission.py:31-33, :1096).

    b_list[g] [2I, K/2] / b_sf_list[g] [2I, K/16] hold the gate and up rows in
    chunks of 16 gate rows followed by the 16 up rows of the same outputs
    (interleave_gate_up builds that order from gate rows then up rows).
    Returns per group h_g [M_g, I] bf16 with
        h_g = silu(alpha_g * A_g B_gate^T) * (alpha_g * A_g B_up^T),
    computed in fp32 from the accumulators and rounded once.  Everything else
    as nvfp4_grouped_gemm; `out`, when given, is bf16 [sum M_g, I]."""
    return _nvfp4_grouped(a_list, a_sf_list, b_list, b_sf_list, problem_sizes, alpha, pack, out,
                          b_index, silu_mul=True)


def interleave_gate_up(w13: torch.Tensor, w13_sf: torch.Tensor):
    """Rows [0, I) gate, [I, 2I) up -> the row order of the silu_mul epilogue:
    for each c, gate rows 16c..16c+15 then up rows I+16c..I+16c+15.  Works on
    the codes [2I, K/2] and the scales [2I, K/16] alike (a row permutation)."""
    rows = int(w13.shape[0])
    if rows % 32 != 0 or int(w13_sf.shape[0]) != rows:
        raise ValueError(f"gate+up weights need 2I rows with I % 16 == 0, got {rows}")
    half = rows // 2
    c = torch.arange(half // 16, device=w13.device).view(-1, 1)
    i = torch.arange(16, device=w13.device).view(1, -1)
    perm = torch.cat([16 * c + i, half + 16 * c + i], dim=1).reshape(-1)
    # as bytes: index_select has no kernels for the fp8 / fp4 dtypes
    return tuple(t.view(torch.uint8).index_select(0, perm).view(t.dtype) for t in (w13, w13_sf))


def nvfp4_expert_mlp(a_list, a_sf_list, alpha13, w13_list, w13_sf_list, w2_list, w2_sf_list,
                     w2_scale, *, pack13: WeightPack | None = None,
                     pack2: WeightPack | None = None):
    """Per group g, the gated expert MLP on NVFP4 operands:
        h_g = silu(alpha13_g A_g W13_gate^T) * (alpha13_g A_g W13_up^T)   (bf16)
        h -> NVFP4 (one decode scale s_h over all groups' rows)
        y_g = (s_h * w2_scale_g) * deq(h_g) @ deq(W2_g)^T                 (bf16)
    w13_list[g] in the interleave_gate_up row order ([2I, K/2]); w2_list[g]
    [H, I/2]; w2_scale: G fp32 decode scales of W2.  Three launches after the
    gate+up GEMM: amax, quantise, down GEMM.  Returns (y_list, h) with h the
    bf16 [sum M_g, I] intermediate."""
    ms = [int(a.shape[0]) for a in a_list]
    inter = int(w13_list[0].shape[0]) // 2
    h = torch.empty((sum(ms), inter), dtype=torch.bfloat16, device=w13_list[0].device)
    nvfp4_grouped_gemm_silu_mul(a_list, a_sf_list, w13_list, w13_sf_list, alpha=alpha13,
                                pack=pack13, out=h)
    hc, hs, hg = quantize_nvfp4(h)
    h_codes = list(hc.split(ms))
    h_sf = list(hs.split(ms))
    w2s = torch.as_tensor(w2_scale, dtype=torch.float32, device=h.device).reshape(-1)
    y = nvfp4_grouped_gemm(h_codes, h_sf, w2_list, w2_sf_list, alpha=(hg * w2s).contiguous(),
                           pack=pack2)
    return y, h


def _nvfp4_grouped(a_list, a_sf_list, b_list, b_sf_list, problem_sizes, alpha, pack, out,
                   b_index, silu_mul: bool) -> list[torch.Tensor]:
    global _last_ws
    G = len(a_list)
    if G == 0 or G != len(a_sf_list) or len(b_list) != len(b_sf_list) or not b_list:
        raise ValueError("a_list/a_sf_list and b_list/b_sf_list must be non-empty, pairwise equal length")
    if b_index is None:
        if len(b_list) != G:
            raise ValueError(f"{G} activation groups but {len(b_list)} weight groups "
                             "(pass b_index to map groups to weights)")
        bidx = None
    else:
        bidx = np.asarray([int(i) for i in b_index], dtype=np.int32)
        if bidx.shape != (G,) or (bidx < 0).any() or (bidx >= len(b_list)).any():
            raise ValueError(f"b_index must hold {G} weight-group indices in [0, {len(b_list)})")
    if pack is None:
        pack = pack_weights(b_list, b_sf_list)
    n, k, dev = pack.n, pack.k, pack.device
    ps = None
    if problem_sizes is not None:
        ps = problem_sizes.tolist() if isinstance(problem_sizes, torch.Tensor) else problem_sizes
        if len(ps) != G:
            raise ValueError(f"problem_sizes has {len(ps)} entries for {G} groups")
    kh, ks = k // 2, k // 16
    # One pass over the groups (decode calls carry hundreds), no per-group
    # views: byte dtypes are read through their data pointers as they are.
    ms = [0] * G
    m_arr, pa, psf = _scratch(G)
    u8 = _U8_DTYPES
    for g in range(G):
        a = a_list[g]
        s = a_sf_list[g]
        sa = a.shape
        m = sa[0] if len(sa) == 2 else -1
        if ps is not None:
            row = ps[g]
            if len(row) != 3 or row[0] != m or row[1] != n or row[2] != k:
                raise ValueError(f"problem_sizes[{g}]={tuple(row)} disagrees with the tensors "
                                 f"(M={m}, N={n}, K={k})")
        if a.dtype not in u8:
            _as_u8(a, f"a[{g}]")
        if s.dtype not in u8:
            _as_u8(s, f"a_sf[{g}]")
        if m < 0 or sa[1] != kh or s.shape != (m, ks):
            raise ValueError(f"group {g}: a {tuple(sa)} / a_sf {tuple(s.shape)} do not match "
                             f"[M, {kh}] / [M, {ks}] for K={k}")
        if m and not (a.is_cuda and s.is_cuda and a.is_contiguous() and s.is_contiguous()):
            raise ValueError(f"group {g}: activations must be contiguous CUDA tensors")
        ms[g] = m
        pa[g] = a.data_ptr()
        psf[g] = s.data_ptr()
    m_arr[:] = ms
    if alpha is None:
        alpha_t = torch.ones(G, dtype=torch.float32, device=dev)
    elif isinstance(alpha, torch.Tensor):
        alpha_t = alpha
        if alpha_t.dtype != torch.float32 or alpha_t.device != dev or not alpha_t.is_contiguous():
            alpha_t = alpha_t.to(device=dev, dtype=torch.float32).contiguous()
    else:
        alpha_t = torch.tensor([float(x) for x in alpha], dtype=torch.float32, device=dev)
    if alpha_t.numel() != G:
        raise ValueError(f"alpha has {alpha_t.numel()} entries for {G} groups")
    total = sum(ms)
    n_out = n // 2 if silu_mul else n
    if silu_mul and n % 32 != 0:
        raise ValueError(f"N={n}: gate and up rows come in chunks of 16 + 16")
    if out is None:
        out = torch.empty((total, n_out), dtype=torch.bfloat16, device=dev)
    elif (out.dtype != torch.bfloat16 or out.shape != (total, n_out) or not out.is_contiguous()
          or out.device != dev):
        raise ValueError(f"out must be a contiguous bf16 [{total}, {n_out}] tensor on {dev}")
    L = _lib.lib()
    prob = _lib.FggNvfp4Problem(G, n, k, m_arr.ctypes.data, pa.ctypes.data, psf.ctypes.data,
                                alpha_t.data_ptr(), out.data_ptr(),
                                None if bidx is None else bidx.ctypes.data, len(b_list))
    nbytes = int(L.fgg_nvfp4_workspace_bytes(prob))
    if nbytes == 0:
        _lib.check(L.fgg_nvfp4_grouped_gemm(prob, None, None, 0, None), "nvfp4_grouped_gemm")
    entry = L.fgg_nvfp4_grouped_gemm_silu_mul if silu_mul else L.fgg_nvfp4_grouped_gemm
    if _is_current(dev):
        stream = _stream_ptr(dev)
        ws = _workspace(dev, stream, nbytes)
        rc = entry(prob, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream)
    else:
        with torch.cuda.device(dev):
            stream = _stream_ptr(dev)
            ws = _workspace(dev, stream, nbytes)
            rc = entry(prob, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream)
    _lib.check(rc, "nvfp4_grouped_gemm")
    _last_ws = ws
    return list(out.split_with_sizes(ms))


# Problem structs and workspaces of the contiguous-rows entry, per geometry:
# a repeated call only patches pointers (no per-group host work at all).
_ROWS: OrderedDict = OrderedDict()


def nvfp4_grouped_gemm_rows(a: torch.Tensor, a_sf: torch.Tensor, offsets: torch.Tensor,
                            b_list=None, b_sf_list=None, alpha=None, *,
                            pack: WeightPack | None = None, out: torch.Tensor | None = None,
                            row_scale: torch.Tensor | None = None,
                            b_index: torch.Tensor | None = None,
                            max_group_rows: int = 0) -> torch.Tensor:
    """Grouped GEMM over contiguous token rows, group sizes on the device.

    The reference operator's own M-grouped layout (one concatenated activation
    tensor, kernels/gemm/fp4_grouped_gemm/b200/kernel.py:10-37) in NVFP4: group
    g owns rows [offsets[g], offsets[g+1]) of
      a      [R, K/2] packed E2M1 codes (uint8 / float4_e2m1fn_x2)
      a_sf   [R, K/16] E4M3 scales
      out    [R, N] bf16 (allocated when not given; rows outside every group
             are left as they are)
    offsets: int32 CUDA tensor [G + 1] (nondecreasing, offsets[G] <= R); it may
    be written by an earlier kernel on the stream -- the host never reads it.
    Weights come from `pack` (or b_list / b_sf_list, packed and cached);
    alpha: fp32 CUDA tensor [G]; row_scale: optional fp32 CUDA tensor [R]
    (out = alpha_g * row_scale_r * acc); b_index: optional int32 CUDA tensor
    [G] naming each group's packed weight group; max_group_rows: a host bound
    on every group's rows (<= 16 selects the decode tiles).  Host work per
    call does not depend on G: no per-group Python."""
    global _last_ws
    if pack is None:
        if b_list is None or b_sf_list is None:
            raise ValueError("give pack= or b_list / b_sf_list")
        pack = pack_weights(b_list, b_sf_list)
    n, k, dev = pack.n, pack.k, pack.device
    # device checks on the index (get_device(): -1 on the host), which is
    # cheaper than building and comparing device objects
    di = dev.index if dev.type == "cuda" else -1
    a_u8 = a if a.dtype is torch.uint8 else _as_u8(a, "a")
    s_u8 = a_sf if a_sf.dtype is torch.uint8 else _as_u8(a_sf, "a_sf")
    if a_u8.dim() != 2 or a_u8.shape[1] != k // 2 or s_u8.shape != (a_u8.shape[0], k // 16):
        raise ValueError(f"a {tuple(a_u8.shape)} / a_sf {tuple(s_u8.shape)} do not match "
                         f"[R, {k // 2}] / [R, {k // 16}] for K={k}")
    if not (a_u8.is_contiguous() and s_u8.is_contiguous() and a_u8.get_device() == di
            and s_u8.get_device() == di):
        raise ValueError(f"a and a_sf must be contiguous tensors on {dev}")
    if (offsets.dtype is not torch.int32 or offsets.dim() != 1 or offsets.get_device() != di
            or not offsets.is_contiguous()):
        raise ValueError(f"offsets must be a contiguous int32 tensor on {dev}")
    G = offsets.shape[0] - 1
    R = a_u8.shape[0]
    if alpha is None:
        alpha = torch.ones(G, dtype=torch.float32, device=dev)
    if (alpha.dtype is not torch.float32 or alpha.numel() != G or alpha.get_device() != di
            or not alpha.is_contiguous()):
        raise ValueError(f"alpha must be a contiguous fp32 tensor of {G} values on {dev}")
    if out is None:
        out = torch.empty((R, n), dtype=torch.bfloat16, device=dev)
    elif (out.dtype is not torch.bfloat16 or out.shape != (R, n) or not out.is_contiguous()
          or out.get_device() != di):
        raise ValueError(f"out must be a contiguous bf16 [{R}, {n}] tensor on {dev}")
    if row_scale is not None or b_index is not None:
        for name, t, dt, cnt in (("row_scale", row_scale, torch.float32, R),
                                 ("b_index", b_index, torch.int32, G)):
            if t is not None and (t.dtype is not dt or t.numel() != cnt or t.get_device() != di
                                  or not t.is_contiguous()):
                raise ValueError(f"{name} must be a contiguous {dt} tensor of {cnt} values "
                                 f"on {dev}")
    L = _lib.lib()
    key = (dev.index, G, n, k, R, int(max_group_rows), b_index is not None, pack.G)
    hit = _ROWS.get(key)
    if hit is None:
        prob = _lib.FggNvfp4RowsProblem(G, n, k, R, 0, 0, 0, 0, 0, 0, 0, pack.G,
                                        int(max_group_rows))
        nbytes = int(L.fgg_nvfp4_rows_workspace_bytes(prob))
        if nbytes == 0:
            _lib.check(L.fgg_nvfp4_grouped_gemm_rows(prob, None, None, 0, None), "grouped GEMM rows")
        hit = [prob, nbytes]
        _ROWS[key] = hit
        while len(_ROWS) > _CACHE_MAX:
            _ROWS.popitem(last=False)
    else:
        _ROWS.move_to_end(key)
    prob, nbytes = hit
    prob.offsets = offsets.data_ptr()
    prob.a = a_u8.data_ptr()
    prob.a_sf = s_u8.data_ptr()
    prob.alpha = alpha.data_ptr()
    prob.out = out.data_ptr()
    prob.row_scale = row_scale.data_ptr() if row_scale is not None else None
    prob.b_index = b_index.data_ptr() if b_index is not None else None
    if _is_current(dev):
        stream = _stream_ptr(dev)
        ws = _workspace(dev, stream, nbytes)
        rc = L.fgg_nvfp4_grouped_gemm_rows(prob, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream)
    else:
        with torch.cuda.device(dev):
            stream = _stream_ptr(dev)
            ws = _workspace(dev, stream, nbytes)
            rc = L.fgg_nvfp4_grouped_gemm_rows(prob, pack.buf.data_ptr(), ws.data_ptr(), nbytes,
                                               stream)
    _lib.check(rc, "nvfp4_grouped_gemm_rows")
    _last_ws = ws
    return out


class _MxPrepared:
    def __init__(self, ws: torch.Tensor, sources):
        self.ws = ws
        self.sources = sources
        self.ready = False


def fp4_grouped_gemm(a: torch.Tensor, a_sf: torch.Tensor, b: torch.Tensor, b_sf: torch.Tensor,
                     m_indices: torch.Tensor) -> torch.Tensor:
    """Returns c [M_total, N] bf16; row i = dequant(a[i]) @ dequant(b[m_indices[i]])^T.

    Same contract as kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788-2862:
    a [M_total, K] float8_e4m3fn, a_sf [M_total, K/128] fp32 powers of two,
    b [G, N, K/2] int8/uint8 packed e2m1, b_sf [G, N, K/32] fp32 powers of two,
    m_indices [M_total] int32 (-1 = padding, segments aligned to 224 rows).
    ValueError for N % 128 or K % 128 (kernel.py:2811-2816)."""
    global _last_ws
    if a.dim() != 2 or b.dim() != 3:
        raise ValueError("a must be [M_total, K] and b [G, N, K/2]")
    m_total, k = int(a.shape[0]), int(a.shape[1])
    g, n = int(b.shape[0]), int(b.shape[1])
    if n % 128 != 0:
        raise ValueError(f"N={n} is not a multiple of BLOCK_N=128")
    if k % 128 != 0:
        raise ValueError(f"K={k} is not a multiple of BLOCK_K=128")
    if int(b.shape[2]) * 2 != k:
        raise ValueError(f"b has K/2={int(b.shape[2])}, a has K={k}")
    if tuple(a_sf.shape) != (m_total, k // 128) or a_sf.dtype != torch.float32:
        raise ValueError(f"a_sf must be fp32 [{m_total}, {k // 128}]")
    if tuple(b_sf.shape) != (g, n, k // 32) or b_sf.dtype != torch.float32:
        raise ValueError(f"b_sf must be fp32 [{g}, {n}, {k // 32}]")
    if tuple(m_indices.shape) != (m_total,) or m_indices.dtype != torch.int32:
        raise ValueError(f"m_indices must be int32 [{m_total}]")
    a_u8 = _as_u8(a, "a")
    b_u8 = _as_u8(b, "b")
    for name, t in (("a", a_u8), ("a_sf", a_sf), ("b", b_u8), ("b_sf", b_sf), ("m_indices", m_indices)):
        if not (t.is_cuda and t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous CUDA tensor")
    dev = a.device
    c = torch.empty((m_total, n), dtype=torch.bfloat16, device=dev)
    L = _lib.lib()
    prob = _lib.FggMxProblem(m_total, n, k, g, a_u8.data_ptr(), a_sf.data_ptr(), b_u8.data_ptr(),
                             b_sf.data_ptr(), m_indices.data_ptr(), c.data_ptr(), 0)
    nbytes = int(L.fgg_mx_workspace_bytes(prob))
    if nbytes == 0:
        _lib.check(L.fgg_mx_grouped_gemm(prob, None, 0, None), "fp4_grouped_gemm")
    key = (_identity(a_sf), _identity(b_sf), _identity(m_indices), m_total, n, k, g)
    prep = _MX_PREP.get_or(key, lambda: _MxPrepared(
        torch.empty(nbytes, dtype=torch.uint8, device=dev), (a_sf, b_sf, m_indices)))
    prob.reuse_prepared = 1 if prep.ready else 0
    if _is_current(dev):
        rc = L.fgg_mx_grouped_gemm(prob, prep.ws.data_ptr(), nbytes, _stream_ptr(dev))
    else:
        with torch.cuda.device(dev):
            rc = L.fgg_mx_grouped_gemm(prob, prep.ws.data_ptr(), nbytes, _stream_ptr(dev))
    _lib.check(rc, "fp4_grouped_gemm")
    prep.ready = True
    _last_ws = prep.ws
    return c


def quantize_nvfp4(x: torch.Tensor, amax: torch.Tensor | None = None):
    """Quantise a CUDA [rows, K] fp32/bf16 tensor to NVFP4 on the device.

    Returns (codes uint8 [rows, K/2], sf float8_e4m3fn [rows, K/16], g) where g
    is the fp32 per-tensor decode scale (0-dim device tensor): x ~ e2m1 * sf * g."""
    if x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D CUDA tensor")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"x dtype {x.dtype} must be float32 or bfloat16")
    rows, k = int(x.shape[0]), int(x.shape[1])
    if k % 16 != 0:
        raise ValueError(f"K={k} must be a multiple of 16")
    dev = x.device
    if _is_current(dev):
        return _quantize_on(x, amax, dev, rows, k)
    with torch.cuda.device(dev):
        return _quantize_on(x, amax, dev, rows, k)


def _quantize_on(x, amax, dev, rows, k):
    dt = 0 if x.dtype == torch.float32 else 1
    L = _lib.lib()
    s = _stream_ptr(dev)
    if amax is None:
        amax_t = torch.empty((), dtype=torch.float32, device=dev)
        _lib.check(L.fgg_amax(x.data_ptr(), dt, x.numel(), amax_t.data_ptr(), s), "fgg_amax")
    else:
        amax_t = amax.to(device=dev, dtype=torch.float32).reshape(()).contiguous()
    codes = torch.empty((rows, k // 2), dtype=torch.uint8, device=dev)
    sf = torch.empty((rows, k // 16), dtype=torch.uint8, device=dev)
    g = torch.empty((), dtype=torch.float32, device=dev)  # written by the kernel
    _lib.check(L.fgg_nvfp4_quantize(x.data_ptr(), dt, rows, k, amax_t.data_ptr(),
                                    codes.data_ptr(), sf.data_ptr(), g.data_ptr(), s),
               "fgg_nvfp4_quantize")
    return codes, sf.view(torch.float8_e4m3fn), g


def _set_last_ws(ws: torch.Tensor) -> None:
    """Record the workspace of a GEMM launched outside this module (last_status reads it)."""
    global _last_ws
    _last_ws = ws


def last_status() -> int:
    """Synchronise the current stream and return the device status word of the
    most recent GEMM call (0 = ok); raises FggError on a device timeout."""
    if _last_ws is None:
        return 0
    L = _lib.lib()
    dev = _last_ws.device
    with torch.cuda.device(dev):
        rc = L.fgg_read_device_status(_last_ws.data_ptr(), _stream_ptr(dev))
    _lib.check(rc, "device status")
    return 0


def clear_caches() -> None:
    _PACKS.clear()
    _MX_PREP.clear()
    _ROWS.clear()
