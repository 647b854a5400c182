"""fgg_nvfp4_grouped_gemm_rows: the grouped GEMM over contiguous token rows
with the group offsets in device memory, against the CPU oracle (operator
tolerance: max|err| / max|ref| <= 1e-2; per element |err| <= 2e-2 |ref| +
1e-2 max|ref|) and, where the same problem fits it, against the per-group-list
entry point.

Covers the three kernels (CTA pair, one CTA per tile, decode tiles), empty
groups, rows past the last group (never written), a device weight-group index,
a per-row scale, and malformed offsets (status 0x203, nothing written).
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref
from ratchet_b200 import _lib

pytestmark = pytest.mark.gpu


def _rows_problem(ms, n, k, max_rows, seed, wg=None, bidx=None, w_std=1.0):
    """Activation groups in one [max_rows] buffer; weight groups `wg` (default
    one per group)."""
    rng = np.random.default_rng(seed)
    G = len(ms)
    wgroups = G if wg is None else wg
    W = [ref.nvfp4_quantize((rng.standard_normal((n, k), dtype=np.float32) * np.float32(w_std)))
         for _ in range(wgroups)]
    x = rng.standard_normal((max_rows, k), dtype=np.float32)
    qa, sa, ga = ref.nvfp4_quantize(x)
    off = np.zeros(G + 1, dtype=np.int32)
    off[1:] = np.cumsum(ms)
    assert off[-1] <= max_rows
    alpha = np.asarray([ga * W[(g if bidx is None else bidx[g])][2] * (1.0 + 0.25 * g)
                        for g in range(G)], dtype=np.float32)
    return dict(W=W, qa=qa, sa=sa, off=off, alpha=alpha, bidx=bidx)


def _run_rows(P, n, k, dev, row_scale=None, max_group_rows=0, offsets=None, sentinel=True):
    import ratchet_b200 as rb

    L = _lib.lib()
    G = len(P["off"]) - 1
    b = [torch.from_numpy(w[0]).to(dev) for w in P["W"]]
    b_sf = [torch.from_numpy(w[1]).to(dev).view(torch.float8_e4m3fn) for w in P["W"]]
    pack = rb.pack_weights(b, b_sf)
    a = torch.from_numpy(P["qa"]).to(dev)
    a_sf = torch.from_numpy(P["sa"]).to(dev)
    max_rows = a.shape[0]
    off = torch.from_numpy(P["off"] if offsets is None else offsets).to(dev)
    alpha = torch.from_numpy(P["alpha"]).to(dev)
    bidx = None if P["bidx"] is None else torch.tensor(P["bidx"], dtype=torch.int32, device=dev)
    rs = None if row_scale is None else torch.from_numpy(row_scale).to(dev)
    out = torch.full((max_rows, n), float("nan") if sentinel else 0.0, dtype=torch.bfloat16,
                     device=dev)
    prob = _lib.FggNvfp4RowsProblem(
        G, n, k, max_rows, off.data_ptr(), a.data_ptr(), a_sf.data_ptr(), alpha.data_ptr(),
        out.data_ptr(), 0 if rs is None else rs.data_ptr(), 0 if bidx is None else bidx.data_ptr(),
        len(P["W"]), max_group_rows)
    nbytes = L.fgg_nvfp4_rows_workspace_bytes(prob)
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.fgg_nvfp4_grouped_gemm_rows(prob, pack.buf.data_ptr(), ws.data_ptr(), nbytes,
                                             stream), "fgg_nvfp4_grouped_gemm_rows")
    rc = L.fgg_read_device_status(ws.data_ptr(), stream)
    return out, rc, int(ws[:4].view(torch.int32).item())


def _oracle(P, row_scale=None):
    outs = []
    off = P["off"]
    for g in range(len(off) - 1):
        w = P["W"][g if P["bidx"] is None else P["bidx"][g]]
        a = P["qa"][off[g]:off[g + 1]]
        s = P["sa"][off[g]:off[g + 1]]
        c = ref.grouped_gemm([a], [s], [w[0]], [w[1]], [P["alpha"][g]], as_bf16=False)[0]
        if row_scale is not None:
            c = c * torch.from_numpy(row_scale[off[g]:off[g + 1]])[:, None]
        outs.append(c.to(torch.bfloat16))
    return outs


def _check(out, P, row_scale=None):
    off = P["off"]
    for g, want in enumerate(_oracle(P, row_scale)):
        ok, st = ref.check_close(out[off[g]:off[g + 1]].cpu(), want)
        assert ok, f"group {g} rows [{off[g]}, {off[g + 1]}): {st}"
    # rows past the last group are never written
    assert torch.isnan(out[int(off[-1]):].float()).all()


@pytest.mark.parametrize("ms,n,k,extra", [
    ([300, 0, 17, 224, 1, 225], 256, 512, 40),    # CTA pairs, empty group, tile edges
    ([5, 130, 0, 225], 384, 768, 3),              # one CTA per tile (N % 256 != 0)
    ([881, 676, 555, 323], 512, 1024, 0),         # larger groups, K % 256 == 0
    ([64, 33], 256, 320, 7),                      # K tail (K % 256 != 0)
])
def test_rows_matches_oracle(cuda_device, ms, n, k, extra):
    P = _rows_problem(ms, n, k, sum(ms) + extra, seed=sum(ms) + n)
    out, rc, st = _run_rows(P, n, k, cuda_device)
    assert rc == _lib.FGG_OK, hex(st)
    _check(out, P)


def test_rows_decode_tiles(cuda_device):
    """max_group_rows <= 16 selects the decode kernel."""
    rng = np.random.default_rng(3)
    ms = [int(v) for v in rng.integers(0, 17, size=40)]
    P = _rows_problem(ms, 384, 1024, sum(ms) + 5, seed=3, w_std=0.02)
    out, rc, st = _run_rows(P, 384, 1024, cuda_device, max_group_rows=16)
    assert rc == _lib.FGG_OK, hex(st)
    _check(out, P)


def test_rows_weight_index_and_row_scale(cuda_device):
    """Six problem groups over three packed weight groups through a device
    b_index, and a per-row factor applied with alpha."""
    ms = [40, 0, 230, 17, 300, 9]
    bidx = [2, 0, 1, 2, 0, 1]
    P = _rows_problem(ms, 256, 512, sum(ms) + 11, seed=77, wg=3, bidx=bidx)
    rs = np.random.default_rng(5).uniform(0.25, 4.0, size=sum(ms) + 11).astype(np.float32)
    out, rc, st = _run_rows(P, 256, 512, cuda_device, row_scale=rs)
    assert rc == _lib.FGG_OK, hex(st)
    _check(out, P, row_scale=rs)


def test_rows_matches_list_entry(cuda_device):
    """Same inputs through the per-group-list entry point: identical bits
    (same tiles, same summation order)."""
    import ratchet_b200 as rb

    ms = [300, 17, 64, 0, 229]
    n, k = 512, 1024
    P = _rows_problem(ms, n, k, sum(ms), seed=12)
    out, rc, st = _run_rows(P, n, k, cuda_device)
    assert rc == _lib.FGG_OK, hex(st)
    dev = cuda_device
    a = torch.from_numpy(P["qa"]).to(dev)
    s = torch.from_numpy(P["sa"]).to(dev).view(torch.float8_e4m3fn)
    b = [torch.from_numpy(w[0]).to(dev) for w in P["W"]]
    b_sf = [torch.from_numpy(w[1]).to(dev).view(torch.float8_e4m3fn) for w in P["W"]]
    lst = rb.nvfp4_grouped_gemm(list(a.split(ms)), list(s.split(ms)), b, b_sf, None,
                                torch.from_numpy(P["alpha"]).to(dev))
    rb.last_status()
    assert torch.equal(torch.cat(lst), out)


def test_rows_malformed_offsets_refused(cuda_device):
    """Decreasing offsets: no tile runs, status 0x203, the output keeps its prefill."""
    ms = [100, 50, 80]
    P = _rows_problem(ms, 256, 512, 300, seed=9)
    bad = P["off"].copy()
    bad[2] = bad[1] - 10
    out, rc, st = _run_rows(P, 256, 512, cuda_device, offsets=bad)
    assert rc == _lib.FGG_ETIMEOUT and st == 0x203
    assert torch.isnan(out.float()).all()
    past = P["off"].copy()
    past[-1] = 301                                 # beyond max_rows
    out, rc, st = _run_rows(P, 256, 512, cuda_device, offsets=past)
    assert st == 0x203 and torch.isnan(out.float()).all()
