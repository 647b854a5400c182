"""CPU checks of the C ABI: the library loads without a GPU, exports every
function include/fgg_api.h declares, sizes its buffers, and rejects bad
arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from ratchet_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fgg_api.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(fgg_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_library_loads_and_reports_version(L):
    assert L.fgg_version().decode().startswith("fgg ")
    assert "sm_100a" in L.fgg_version().decode()


def test_every_declared_function_is_exported(L):
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), f"{n} declared in fgg_api.h but not exported"


def test_binding_covers_header(L):
    assert sorted(_lib.exported_symbols()) == declared_functions()


def test_error_strings(L):
    for code in range(8):
        assert L.fgg_error_string(code)
    assert L.fgg_error_string(_lib.FGG_EBADSHAPE) == b"unsupported shape"


def _pack_bytes_py(g, n, k):
    nk64p = ((k // 64) + 3) // 4 * 4
    off = 0
    def take(nbytes, align):
        nonlocal off
        off = (off + align - 1) // align * align
        at = off
        off += nbytes
        return at
    take(16, 256)
    take(g * 128, 128)
    take(g * (n // 128) * nk64p * 512, 256)
    return off


@pytest.mark.parametrize("g,n,k", [(1, 256, 512), (8, 4096, 7168), (256, 7168, 2048), (3, 128, 320)])
def test_weight_pack_bytes(L, g, n, k):
    assert L.fgg_nvfp4_weight_pack_bytes(g, n, k) == _pack_bytes_py(g, n, k)


def _problem(ms, n, k):
    G = len(ms)
    m = np.asarray(ms, dtype=np.int32)
    fake = np.full(G, 1 << 20, dtype=np.uint64)  # never dereferenced by the size query
    keep = (m, fake)
    return _lib.FggNvfp4Problem(G, n, k, m.ctypes.data, fake.ctypes.data, fake.ctypes.data,
                                1 << 20, 1 << 20), keep


def _ws_bytes_py(ms, n, k):
    bn = 16 if max(ms) <= 16 else 224
    ch = (bn + 127) // 128
    nk256 = (k + 255) // 256
    nk64p = 4 * nk256
    xts = sum((m + bn - 1) // bn for m in ms)
    pair = bn == 224 and n % 256 == 0   # CTA pairs cover 256 weight rows per tile
    tiles = xts * (n // (256 if pair else 128))
    off = 0
    def take(nbytes, align):
        nonlocal off
        off = (off + align - 1) // align * align
        off += nbytes
    take(256, 256)
    take(len(ms) * 128, 128)
    take(len(ms) * 16, 256)
    take(max(tiles, 1) * 4, 256)
    # token scales: ch atoms of 512 B per (token tile, MMA)
    take(max(xts, 1) * nk64p * ch * 512, 256)
    return off


@pytest.mark.parametrize("ms,n,k", [([128], 256, 512), ([0, 1, 224, 225], 256, 768),
                                    ([3, 16, 9], 7168, 2048), ([881, 676, 555], 4096, 7168),
                                    ([300, 40], 384, 512)])
def test_workspace_bytes(L, ms, n, k):
    p, keep = _problem(ms, n, k)
    assert L.fgg_nvfp4_workspace_bytes(p) == _ws_bytes_py(ms, n, k)


@pytest.mark.parametrize("n,k", [(200, 512), (256, 100), (256, 32), (0, 512)])
def test_bad_shape_rejected_before_device(L, n, k):
    p, keep = _problem([16], n, k)
    assert L.fgg_nvfp4_workspace_bytes(p) == 0
    rc = L.fgg_nvfp4_grouped_gemm(p, None, None, 0, None)
    assert rc == _lib.FGG_EBADSHAPE
    assert L.fgg_last_error_detail()


def test_too_many_groups_rejected(L):
    p, keep = _problem([1] * (_lib.FGG_MAX_GROUPS + 1), 256, 512)
    assert L.fgg_nvfp4_grouped_gemm(p, None, None, 0, None) == _lib.FGG_EINVAL


def test_negative_m_rejected(L):
    p, keep = _problem([4, -1], 256, 512)
    assert L.fgg_nvfp4_grouped_gemm(p, None, None, 0, None) == _lib.FGG_EINVAL


def test_small_workspace_rejected(L):
    p, keep = _problem([64], 256, 512)
    need = L.fgg_nvfp4_workspace_bytes(p)
    rc = L.fgg_nvfp4_grouped_gemm(p, ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 21), need - 1, None)
    assert rc == _lib.FGG_EWORKSPACE


def test_mx_shape_rules_follow_reference(L):
    """kernel.py:2811-2816: N % 128 and K % 128 are ValueErrors in the reference."""
    bad_n = _lib.FggMxProblem(448, 200, 512, 2, 1, 1, 1, 1, 1, 1, 0)
    bad_k = _lib.FggMxProblem(448, 256, 192, 2, 1, 1, 1, 1, 1, 1, 0)
    assert L.fgg_mx_grouped_gemm(bad_n, None, 0, None) == _lib.FGG_EBADSHAPE
    assert L.fgg_mx_grouped_gemm(bad_k, None, 0, None) == _lib.FGG_EBADSHAPE
    ok = _lib.FggMxProblem(448, 256, 512, 2, 1, 1, 1, 1, 1, 1, 0)
    assert L.fgg_mx_workspace_bytes(ok) > 0


def test_quantize_rejects_bad_k(L):
    assert L.fgg_nvfp4_quantize(1, 0, 4, 24, 1, 8, 1, None, None) == _lib.FGG_EBADSHAPE


def test_check_maps_codes_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.FGG_EBADSHAPE, "x")
    with pytest.raises(_lib.FggError):
        _lib.check(_lib.FGG_ETIMEOUT, "x")


def test_b_index_validated_before_device(L):
    """A problem group may name a shared weight group; out-of-range indices and
    a bad weight-group count are refused on the host."""
    G = 3
    m = np.asarray([16, 0, 40], dtype=np.int32)
    fake = np.full(G, 1 << 20, dtype=np.uint64)
    bad = np.asarray([0, 2, 1], dtype=np.int32)
    p = _lib.FggNvfp4Problem(G, 256, 512, m.ctypes.data, fake.ctypes.data, fake.ctypes.data,
                             1 << 20, 1 << 20, bad.ctypes.data, 2)
    assert L.fgg_nvfp4_workspace_bytes(p) == 0
    assert L.fgg_nvfp4_grouped_gemm(p, None, None, 0, None) == _lib.FGG_EINVAL
    assert b"b_index[1]=2" in L.fgg_last_error_detail()
    good = np.asarray([0, 1, 1], dtype=np.int32)
    p = _lib.FggNvfp4Problem(G, 256, 512, m.ctypes.data, fake.ctypes.data, fake.ctypes.data,
                             1 << 20, 1 << 20, good.ctypes.data, 0)
    assert L.fgg_nvfp4_grouped_gemm(p, None, None, 0, None) == _lib.FGG_EINVAL
    p.num_weight_groups = 2
    assert L.fgg_nvfp4_workspace_bytes(p) > 0


def _peers(world=2, rank=0, capacity=4, n=64, base=0x10000, flag_off=0):
    p = _lib.FggMoePeers()
    p.world, p.rank, p.capacity, p.n = world, rank, capacity, n
    p.epoch, p.counters, p.status = base, base + 8, base + 20
    for r in range(max(world, 0)):
        if r < _lib.FGG_PEERS_MAX:
            p.gathered[r] = base + 0x1000 * (r + 1)
            p.recv[r] = base + 0x100000 * (r + 1)
            p.flags[r] = base + 0x200 + 0x100 * r + flag_off
    p.owner, p.num_experts, p.routes = base + 0x800, 8, base + 0x900
    p.wait_ms = 0
    return p


def test_peer_descriptions_validated_before_device(L):
    """The peer exchange entries check the description before any device
    call: world, rank, n, null state words, misaligned buffers, the wait kind."""
    import ctypes

    def wait(p, kind=0):
        return L.fgg_moe_wait_peers(ctypes.byref(p), kind, None)

    assert wait(_peers(), 2) == _lib.FGG_EINVAL
    assert wait(_peers(world=0)) == _lib.FGG_EBADSHAPE
    assert wait(_peers(world=_lib.FGG_PEERS_MAX + 1)) == _lib.FGG_EBADSHAPE
    assert wait(_peers(rank=2)) == _lib.FGG_EBADSHAPE
    assert wait(_peers(n=60)) == _lib.FGG_EBADSHAPE
    assert wait(_peers(capacity=0)) == _lib.FGG_EBADSHAPE
    p = _peers()
    p.status = None
    assert wait(p) == _lib.FGG_EINVAL
    p = _peers()
    p.recv[1] = None
    assert wait(p) == _lib.FGG_EINVAL
    p = _peers()
    p.routes = None
    assert wait(p) == _lib.FGG_EINVAL
    p = _peers()
    p.num_experts = 0
    assert wait(p) == _lib.FGG_EBADSHAPE
    assert wait(_peers(flag_off=4)) == _lib.FGG_EALIGN
    p = _peers()
    p.gathered[0] += 8
    assert wait(p) == _lib.FGG_EALIGN
    assert L.fgg_moe_sum_peers(ctypes.byref(_peers()), 5, None, None) == _lib.FGG_EBADSHAPE
    assert L.fgg_moe_sum_peers(ctypes.byref(_peers()), 3, None, None) == _lib.FGG_EINVAL


def test_peer_handles_validated(L):
    import ctypes

    assert L.fgg_peer_handle_bytes() == 64
    assert L.fgg_peer_alloc(0, ctypes.byref(ctypes.c_void_p())) == _lib.FGG_EINVAL
    assert L.fgg_peer_export(None, ctypes.create_string_buffer(64)) == _lib.FGG_EINVAL
    assert L.fgg_peer_import(None, ctypes.byref(ctypes.c_void_p())) == _lib.FGG_EINVAL
    assert L.fgg_peer_free(None) == _lib.FGG_OK
    assert L.fgg_peer_close(None) == _lib.FGG_OK


def test_peer_wait_limit_validated(L):
    import ctypes

    p = _peers()
    p.wait_ms = -1
    assert L.fgg_moe_wait_peers(ctypes.byref(p), 0, None) == _lib.FGG_EINVAL
