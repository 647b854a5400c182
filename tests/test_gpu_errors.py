"""The device error paths, driven without a fault.

Every wait in the GEMM kernels is bounded: when it runs out (about one second)
the kernel records a status code in its workspace, raises a CTA-wide abort
flag, drains its copies, frees TMEM and returns.  A weight pack built for
another problem is refused by the kernel before its first load (status 0x201).
These tests make both happen on purpose and check that the host sees the
status, that the output is left untouched, and that the next call is clean:

  * a weight pack whose header names a different N (all pointers valid, every
    byte the call could touch inside the pack), through the workspace entry
    point (fgg_read_device_status) and the no-alloc one (status_out);
  * the test hook FGG_DEBUG_NO_LOADS: the producer arms no stage, so the MMA
    role waits on a full barrier that nothing completes until its limit;
  * the MX operator's cached path, which skips the prepare kernel, must not
    report an earlier call's status.
"""
import numpy as np
import pytest
import torch

from oracle import mx as mref
from oracle import nvfp4 as ref
from ratchet_b200 import _lib

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {0x101, 0x102, 0x103}


def _dev(prob, dev):
    t = lambda xs: [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in xs]
    return (t(prob["a"]), [s.view(torch.float8_e4m3fn) for s in t(prob["a_sf"])], t(prob["b"]),
            [s.view(torch.float8_e4m3fn) for s in t(prob["b_sf"])],
            torch.from_numpy(prob["alpha"]).to(dev))


def _problem(ms, n, k, a, a_sf, alpha, out):
    from ratchet_b200 import ops

    m_arr = np.asarray(ms, np.int32)
    pa, psf = ops._ptr_array(a), ops._ptr_array(a_sf)
    p = _lib.FggNvfp4Problem(len(ms), n, k, m_arr.ctypes.data, pa.ctypes.data, psf.ctypes.data,
                             alpha.data_ptr(), out.data_ptr())
    return p, (m_arr, pa, psf)


def _status_word(ws):
    return int(ws[:4].view(torch.int32).item())


@pytest.fixture
def no_debug_flags():
    L = _lib.lib()
    L.fgg_debug_set_flags(0)
    yield L
    L.fgg_debug_set_flags(0)


def test_mismatched_weight_pack_is_refused(cuda_device, no_debug_flags):
    """A pack packed for N=512 given to an N=256 problem: the kernel reads the
    pack header, sets status 0x201 and issues no load; the output keeps its
    NaN prefill.  A correct call on the same workspace afterwards is clean."""
    import ratchet_b200 as rb

    L = no_debug_flags
    dev = cuda_device
    ms, k = [64, 200], 512
    prob = ref.random_problem(ms, 256, k, seed=41)
    a, a_sf, b, b_sf, alpha = _dev(prob, dev)
    wrong = ref.random_problem([1, 1], 512, k, seed=42)
    _, _, bw, bw_sf, _ = _dev(wrong, dev)
    wrong_pack = rb.pack_weights(bw, bw_sf)       # header: G=2, N=512, K=512
    assert wrong_pack.buf.numel() >= L.fgg_nvfp4_weight_pack_bytes(2, 256, k)
    out = torch.full((sum(ms), 256), float("nan"), dtype=torch.bfloat16, device=dev)
    p, keep = _problem(ms, 256, k, a, a_sf, alpha, out)
    nbytes = L.fgg_nvfp4_workspace_bytes(p)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.fgg_nvfp4_grouped_gemm(p, wrong_pack.buf.data_ptr(), ws.data_ptr(), nbytes,
                                        stream), "grouped gemm")
    rc = L.fgg_read_device_status(ws.data_ptr(), stream)
    assert rc == _lib.FGG_ETIMEOUT
    assert b"0x201" in L.fgg_last_error_detail()
    assert _status_word(ws) == 0x201
    assert torch.isnan(out.float()).all(), "a refused call wrote output"

    # the no-alloc entry point reports the same through status_out
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    _lib.check(L.fgg_nvfp4_grouped_gemm_noalloc(p, wrong_pack.buf.data_ptr(), status.data_ptr(),
                                                stream), "noalloc")
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0x201
    assert torch.isnan(out.float()).all()

    # the right pack on the same workspace: clean status, correct output
    good = rb.pack_weights(b, b_sf)
    _lib.check(L.fgg_nvfp4_grouped_gemm(p, good.buf.data_ptr(), ws.data_ptr(), nbytes, stream),
               "grouped gemm")
    assert L.fgg_read_device_status(ws.data_ptr(), stream) == _lib.FGG_OK
    refs = ref.grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["alpha"])
    for g, (o, r) in enumerate(zip(out.split(ms), refs)):
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g}: {st}"


@pytest.mark.parametrize("ms,n", [([300, 40], 256), ([5, 9, 16], 256), ([100], 384)],
                         ids=["pair", "decode", "single"])
def test_bounded_wait_runs_out(cuda_device, no_debug_flags, ms, n):
    """FGG_DEBUG_NO_LOADS: no stage is ever armed, so the MMA role's first
    wait runs out after about a second.  The call returns, the status word
    holds a timeout code, the output is untouched, and the next call (hook
    off) is correct on the same workspace: the context stays usable."""
    import ratchet_b200 as rb

    L = no_debug_flags
    dev = cuda_device
    k = 512
    prob = ref.random_problem(ms, n, k, seed=sum(ms) + n)
    a, a_sf, b, b_sf, alpha = _dev(prob, dev)
    pack = rb.pack_weights(b, b_sf)
    out = torch.full((sum(ms), n), float("nan"), dtype=torch.bfloat16, device=dev)
    p, keep = _problem(ms, n, k, a, a_sf, alpha, out)
    nbytes = L.fgg_nvfp4_workspace_bytes(p)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    L.fgg_debug_set_flags(_lib.FGG_DEBUG_NO_LOADS)
    _lib.check(L.fgg_nvfp4_grouped_gemm(p, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream),
               "grouped gemm")
    L.fgg_debug_set_flags(0)
    assert L.fgg_read_device_status(ws.data_ptr(), stream) == _lib.FGG_ETIMEOUT
    assert _status_word(ws) in TIMEOUT_CODES, hex(_status_word(ws))
    assert torch.isnan(out.float()).all(), "a kernel that loaded nothing wrote output"

    _lib.check(L.fgg_nvfp4_grouped_gemm(p, pack.buf.data_ptr(), ws.data_ptr(), nbytes, stream),
               "grouped gemm")
    assert L.fgg_read_device_status(ws.data_ptr(), stream) == _lib.FGG_OK
    refs = ref.grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["alpha"])
    for g, (o, r) in enumerate(zip(out.split(ms), refs)):
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g}: {st}"


def test_mx_cached_call_does_not_keep_an_old_status(cuda_device, no_debug_flags):
    """fp4_grouped_gemm caches its scale repack on tensor identity and then
    skips the prepare kernel.  After a call that ran out (hook on), the next,
    cached call must clear the status word itself and report clean."""
    import ratchet_b200 as rb

    L = no_debug_flags
    prob = mref.random_problem([300, 100], 256, 512, seed=5)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda_device) for k, v in prob.items()}
    args = (t["a"].view(torch.float8_e4m3fn), t["a_sf"], t["b"], t["b_sf"], t["m_indices"])
    rb.fp4_grouped_gemm(*args)
    assert rb.last_status() == 0
    L.fgg_debug_set_flags(_lib.FGG_DEBUG_NO_LOADS)
    rb.fp4_grouped_gemm(*args)                    # cached repack, GEMM runs out
    L.fgg_debug_set_flags(0)
    with pytest.raises(_lib.FggError):
        rb.last_status()
    c = rb.fp4_grouped_gemm(*args)                # cached again: must be clean
    assert rb.last_status() == 0
    r = mref.fp4_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["m_indices"])
    valid = torch.from_numpy(prob["m_indices"] >= 0)
    ok, st = ref.check_close(c.cpu()[valid], r[valid])
    assert ok, st
