"""fgg_nvfp4_grouped_gemm_noalloc: the NVFP4 grouped GEMM with its scratch in
the library's fixed device array instead of a caller workspace.

The GPU cases compare two calls in a row of the no-alloc entry point with the
workspace entry point fgg_nvfp4_grouped_gemm on the same inputs, within the
operator's tolerance (max|err| / max|ref| <= 1e-2; per element |err| <=
2e-2 * |ref| + 1e-2 * max|ref|), and read the device status word back through
status_out.  The file sorts last so that the shared scratch has already been
through every other test's calls when these run (they also pass alone).
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


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_workspace_entry_two_calls(cuda_device, case):
    import ratchet_b200 as rb
    from ratchet_b200 import ops

    ms, n, k = CASES[case]
    prob = ref.random_problem(ms, n, k, seed=len(ms) * 1000 + n)
    dev = cuda_device
    a = [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in prob["a"]]
    a_sf = [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in prob["a_sf"]]
    b = [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in prob["b"]]
    b_sf = [torch.from_numpy(np.ascontiguousarray(x)).to(dev).view(torch.float8_e4m3fn)
            for x in prob["b_sf"]]
    alpha = torch.from_numpy(prob["alpha"]).to(dev)
    pack = rb.pack_weights(b, b_sf)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    rows = sum(ms)
    m_arr = np.asarray(ms, np.int32)
    pa, psf = ops._ptr_array(a), ops._ptr_array(a_sf)

    def problem(out):
        return _lib.FggNvfp4Problem(len(ms), n, k, m_arr.ctypes.data, pa.ctypes.data,
                                    psf.ctypes.data, alpha.data_ptr(), out.data_ptr())

    want = torch.empty((rows, n), dtype=torch.bfloat16, device=dev)
    pw = problem(want)
    nbytes = L.fgg_nvfp4_workspace_bytes(pw)
    assert 0 < nbytes <= _lib.FGG_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _lib.check(L.fgg_nvfp4_grouped_gemm(pw, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream),
               "fgg_nvfp4_grouped_gemm")

    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    got = []
    for _ in range(2):
        out = torch.full((rows, n), float("nan"), dtype=torch.bfloat16, device=dev)
        status.fill_(-1)
        _lib.check(L.fgg_nvfp4_grouped_gemm_noalloc(problem(out), pack.buf.data_ptr(),
                                                    status.data_ptr(), stream),
                   "fgg_nvfp4_grouped_gemm_noalloc")
        torch.cuda.synchronize(dev)
        assert status.item() == 0, f"device status 0x{status.item():x}"
        got.append(out)
    _lib.check(L.fgg_read_device_status(ws.data_ptr(), stream), "fgg_read_device_status")
    for i, out in enumerate(got):
        assert torch.isfinite(out.float()).all(), f"call {i}: rows left unwritten"
        assert _close(out, want), f"call {i} differs from the workspace entry point"
