"""CPU checks of the Python operator layer: argument validation mirrors the
reference (ValueError for shapes, kernel.py:2811-2816), CPU tensors are
refused (there is no CPU fallback), and the identity cache key tracks the
reference's discipline (kernel.py:2746-2748)."""
import pytest
import torch

import ratchet_b200 as rb
from ratchet_b200 import ops


def _mx_args(m_total=448, n=256, k=512, g=2, device="cpu"):
    return (torch.zeros((m_total, k), dtype=torch.float8_e4m3fn, device=device),
            torch.ones((m_total, k // 128), device=device),
            torch.zeros((g, n, k // 2), dtype=torch.uint8, device=device),
            torch.ones((g, n, k // 32), device=device),
            torch.zeros((m_total,), dtype=torch.int32, device=device))


def test_mx_rejects_n_not_multiple_of_128():
    a, asf, b, bsf, mi = _mx_args(n=200)
    with pytest.raises(ValueError, match="BLOCK_N"):
        rb.fp4_grouped_gemm(a, asf, b, bsf, mi)


def test_mx_rejects_k_not_multiple_of_128():
    a, asf, b, bsf, mi = _mx_args(k=192)
    with pytest.raises(ValueError, match="BLOCK_K"):
        rb.fp4_grouped_gemm(a, asf, b, bsf, mi)


def test_mx_rejects_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        rb.fp4_grouped_gemm(*_mx_args())


def test_mx_rejects_wrong_scale_dtype():
    a, asf, b, bsf, mi = _mx_args()
    with pytest.raises(ValueError, match="a_sf"):
        rb.fp4_grouped_gemm(a, asf.half(), b, bsf, mi)


def test_nvfp4_rejects_cpu_weights():
    b = [torch.zeros((256, 256), dtype=torch.uint8)]
    bsf = [torch.zeros((256, 32), dtype=torch.uint8)]
    with pytest.raises(ValueError, match="CUDA"):
        rb.pack_weights(b, bsf)


def test_nvfp4_rejects_mismatched_lists():
    with pytest.raises(ValueError):
        rb.nvfp4_grouped_gemm([], [], [], [])


def test_nvfp4_rejects_non_byte_dtype():
    with pytest.raises(ValueError, match="byte type"):
        ops._as_u8(torch.zeros(4, dtype=torch.float32), "x")


def test_identity_key_tracks_version_and_view():
    t = torch.zeros(8, dtype=torch.uint8)
    k0 = ops._identity(t)
    t.add_(1)                      # in-place write bumps _version
    assert ops._identity(t) != k0
    assert ops._identity(t[:4]) != ops._identity(t)


def test_lru_evicts_oldest():
    lru = ops._LRU()
    for i in range(ops._CACHE_MAX + 3):
        lru.get_or(i, lambda i=i: i)
    assert len(lru) == ops._CACHE_MAX
    assert 0 not in lru and (ops._CACHE_MAX + 2) in lru


def test_quantize_rejects_cpu():
    with pytest.raises(ValueError):
        rb.quantize_nvfp4(torch.zeros((4, 32)))


def test_problem_sizes_checked_against_tensors():
    """problem_sizes rows (M_g, N, K) must agree with the activation tensors;
    checked before any device work (a stand-in pack with no device buffer)."""
    import types

    fake = types.SimpleNamespace(n=256, k=128, device=torch.device("cpu"))
    a = [torch.zeros((m, 64), dtype=torch.uint8) for m in (3, 0, 17)]
    sf = [torch.zeros((m, 8), dtype=torch.uint8) for m in (3, 0, 17)]
    b = [None] * 3

    def call(ps):
        return rb.nvfp4_grouped_gemm(a, sf, b, b, ps, pack=fake)

    with pytest.raises(ValueError, match=r"problem_sizes\[0\]"):
        call([(4, 256, 128), (0, 256, 128), (17, 256, 128)])
    with pytest.raises(ValueError, match=r"problem_sizes\[0\]"):
        call(torch.tensor([[3, 128, 128], [0, 256, 128], [17, 256, 128]]))
    with pytest.raises(ValueError, match="3 groups"):
        call([(3, 256, 128)])
    # agreeing sizes pass the check and stop at the CPU tensors: no CPU fallback
    with pytest.raises(ValueError, match="CUDA"):
        call([(3, 256, 128), (0, 256, 128), (17, 256, 128)])
    with pytest.raises(ValueError, match=r"group 0: a \(3, 32\)"):
        rb.nvfp4_grouped_gemm([torch.zeros((3, 32), dtype=torch.uint8), a[1], a[2]], sf, b, b,
                              pack=fake)


def test_interleave_gate_up_order():
    """Rows come out as 16 gate rows, then the 16 up rows of the same outputs."""
    inter, k2 = 48, 4
    w = torch.arange(2 * inter, dtype=torch.uint8).view(-1, 1).repeat(1, k2)
    sf = w[:, :2].clone().view(torch.float8_e4m3fn)
    wi, sfi = rb.interleave_gate_up(w, sf)
    rows = wi[:, 0].tolist()
    want = []
    for c in range(inter // 16):
        want += list(range(16 * c, 16 * c + 16)) + list(range(inter + 16 * c, inter + 16 * c + 16))
    assert rows == want
    assert sfi.dtype == torch.float8_e4m3fn
    assert sfi.view(torch.uint8)[:, 0].tolist() == want
    with pytest.raises(ValueError):
        rb.interleave_gate_up(w[:40], sf[:40])
