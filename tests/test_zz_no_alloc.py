"""fgg_nvfp4_grouped_gemm_noalloc: the NVFP4 grouped GEMM with its scratch in
the library's fixed device array instead of a caller workspace.

Who needs it: a caller that cannot allocate device memory at call time -- a
serving loop that owns a fixed memory budget, or a host without an allocator on
its call path.  The call takes only inputs, outputs and an optional status
pointer; its scratch (descriptors, tile list, repacked token scales, status
words) lives in one FGG_NOALLOC_SCRATCH_BYTES array per device, shared by every
call, so calls on one device must not overlap in time.

The GPU cases make the shared scratch dirty by construction (a call of another
shape goes first), then compare two calls in a row with the CPU oracle and with
the workspace entry point fgg_nvfp4_grouped_gemm, within the operator's
tolerance (max|err| / max|ref| <= 1e-2; per element |err| <= 2e-2 * |ref| +
1e-2 * max|ref|), reading the device status word back through status_out.  The
file sorts last so that a run that stops at the first failure has run every
other test first; the cases also pass when run alone.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref
from ratchet_b200 import _lib


def _fake_problem(ms, n, k):
    G = len(ms)
    m = np.asarray(ms, dtype=np.int32)
    fake = np.full(G, 1 << 20, dtype=np.uint64)  # never dereferenced: refused first
    return _lib.FggNvfp4Problem(G, n, k, m.ctypes.data, fake.ctypes.data, fake.ctypes.data,
                                1 << 20, 1 << 20), (m, fake)


def test_oversize_problem_refused_before_device_work():
    L = _lib.lib()
    p, keep = _fake_problem([224 * 300], 256, 8192)
    need = L.fgg_nvfp4_workspace_bytes(p)
    assert need > _lib.FGG_NOALLOC_SCRATCH_BYTES
    rc = L.fgg_nvfp4_grouped_gemm_noalloc(p, None, None, None)
    assert rc == _lib.FGG_EWORKSPACE
    assert b"static scratch" in L.fgg_last_error_detail()


def test_misaligned_status_out_refused_before_device_work():
    L = _lib.lib()
    p, keep = _fake_problem([40, 7], 256, 512)
    rc = L.fgg_nvfp4_grouped_gemm_noalloc(p, None, (1 << 20) + 2, None)
    assert rc == _lib.FGG_EALIGN
    assert b"status_out" in L.fgg_last_error_detail()


def _close(got, want):
    g, w = got.float(), want.float()
    scale = w.abs().max().item()
    err = (g - w).abs()
    if scale == 0.0:
        return err.max().item() == 0.0
    return (err.max().item() / scale <= 1e-2
            and bool((err <= 2e-2 * w.abs() + 1e-2 * scale).all()))


CASES = {
    "pair": ([0, 1, 17, 224, 300, 40], 256, 512),   # CTA-pair kernel (N % 256 == 0)
    "single": ([5, 130, 225], 384, 768),            # one CTA per tile (N % 256 != 0)
    "decode": ([1, 16, 0, 9], 512, 1024),           # every M <= 16
}


class _Case:
    """Device inputs of one case and the C problem struct over them."""

    def __init__(self, ms, n, k, seed, dev):
        import ratchet_b200 as rb
        from ratchet_b200 import ops

        self.ms, self.n, self.k = ms, n, k
        self.prob = ref.random_problem(ms, n, k, seed=seed)
        t = lambda xs: [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in xs]
        self.a = t(self.prob["a"])
        self.a_sf = t(self.prob["a_sf"])
        b = t(self.prob["b"])
        b_sf = [s.view(torch.float8_e4m3fn) for s in t(self.prob["b_sf"])]
        self.alpha = torch.from_numpy(self.prob["alpha"]).to(dev)
        self.pack = rb.pack_weights(b, b_sf)
        self.m_arr = np.asarray(ms, np.int32)
        self.pa, self.psf = ops._ptr_array(self.a), ops._ptr_array(self.a_sf)
        self.rows = sum(ms)

    def problem(self, out):
        return _lib.FggNvfp4Problem(len(self.ms), self.n, self.k, self.m_arr.ctypes.data,
                                    self.pa.ctypes.data, self.psf.ctypes.data,
                                    self.alpha.data_ptr(), out.data_ptr())

    def noalloc(self, out, status, stream):
        L = _lib.lib()
        status.fill_(-1)
        _lib.check(L.fgg_nvfp4_grouped_gemm_noalloc(self.problem(out), self.pack.buf.data_ptr(),
                                                    status.data_ptr(), stream),
                   "fgg_nvfp4_grouped_gemm_noalloc")


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_oracle_and_workspace_entry_two_calls(cuda_device, case):
    dev = cuda_device
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    ms, n, k = CASES[case]
    c = _Case(ms, n, k, seed=len(ms) * 1000 + n, dev=dev)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)

    # another shape first, so this case starts on scratch that holds another
    # call's descriptors, tile list and scales whatever ran before it
    other = _Case([230, 3, 64] if case != "pair" else [9, 2], 256, 256, seed=99, dev=dev)
    junk = torch.empty((other.rows, 256), dtype=torch.bfloat16, device=dev)
    other.noalloc(junk, status, stream)

    want = torch.empty((c.rows, n), dtype=torch.bfloat16, device=dev)
    pw = c.problem(want)
    nbytes = L.fgg_nvfp4_workspace_bytes(pw)
    assert 0 < nbytes <= _lib.FGG_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _lib.check(L.fgg_nvfp4_grouped_gemm(pw, c.pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream),
               "fgg_nvfp4_grouped_gemm")

    got = []
    for _ in range(2):
        out = torch.full((c.rows, n), float("nan"), dtype=torch.bfloat16, device=dev)
        c.noalloc(out, status, stream)
        torch.cuda.synchronize(dev)
        assert status.item() == 0, f"device status 0x{status.item():x}"
        got.append(out)
    _lib.check(L.fgg_read_device_status(ws.data_ptr(), stream), "fgg_read_device_status")
    refs = ref.grouped_gemm(c.prob["a"], c.prob["a_sf"], c.prob["b"], c.prob["b_sf"],
                            c.prob["alpha"])
    for i, out in enumerate(got):
        assert torch.isfinite(out.float()).all(), f"call {i}: rows left unwritten"
        assert _close(out, want), f"call {i} differs from the workspace entry point"
        for g, (o, r) in enumerate(zip(out.split(ms), refs)):
            ok, st = ref.check_close(o.cpu(), r)
            assert ok, f"call {i} group {g}: {st}"


@pytest.mark.gpu
def test_noalloc_all_groups_empty(cuda_device):
    """Every M_g = 0: no kernel runs, status_out reads 0 and nothing is written."""
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    busy = _Case([300, 17], 256, 512, seed=7, dev=dev)       # leaves the scratch dirty
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    busy.noalloc(torch.empty((busy.rows, 256), dtype=torch.bfloat16, device=dev), status, stream)
    empty = _Case([0, 0, 0], 256, 512, seed=8, dev=dev)
    sentinel = torch.full((4, 256), float("nan"), dtype=torch.bfloat16, device=dev)
    empty.noalloc(sentinel, status, stream)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    assert torch.isnan(sentinel.float()).all()
