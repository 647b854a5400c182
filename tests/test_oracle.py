"""CPU checks of the oracle: pinned against fixtures generated from the
reference itself (tests/golden/make_golden.py) and against third-party format
implementations (torch's float8_e4m3fn cast)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import mx as mref
from oracle import nvfp4 as ref

GOLDEN = Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------- golden pins
def test_e2m1_matches_reference_cast():
    """E2M1 rounding == leaderboard.py:608-627 `_cast_to_fp4x2`, including the
    tie points, -0 and saturation."""
    d = np.load(GOLDEN / "e2m1_cast.npz")
    codes = ref.e2m1_encode(d["x"])
    assert np.array_equal(ref.pack_nibbles(codes), d["packed"])


def test_mx_exponent_bytes_match_reference():
    d = np.load(GOLDEN / "mx_sf_pack.npz")
    assert np.array_equal(mref.exponent_bytes(d["a_sf"]), d["exp_bytes"])


def test_mx_sf_offsets_match_reference():
    d = np.load(GOLDEN / "mx_sf_pack.npz")
    assert np.array_equal(np.array(mref.sf_offsets(224, 4)), d["sf_offsets_224x4"])


def test_mx_pack_sf_act_matches_reference():
    d = np.load(GOLDEN / "mx_sf_pack.npz")
    k = int(d["k"])
    m_total = d["a_sf"].shape[0]
    got = mref.pack_sf_act(d["a_sf"], (m_total + 223) // 224, k // 128)
    assert np.array_equal(got, d["sf_act"])


def test_mx_pack_sf_wgt_matches_reference():
    d = np.load(GOLDEN / "mx_sf_pack.npz")
    n, k = int(d["n"]), int(d["k"])
    got = mref.pack_sf_wgt(d["b_sf"], n // 128, k // 128)
    assert np.array_equal(got, d["sf_wgt"])


def test_mx_block_expert_matches_reference():
    d = np.load(GOLDEN / "mx_sf_pack.npz")
    assert np.array_equal(mref.block_expert(d["m_indices"]), d["blk_expert"])


# ------------------------------------------------------------- formats
def test_e4m3_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    v = np.abs(rng.standard_normal(100000).astype(np.float32)) * np.float32(60)
    t = ref.E4M3_TABLE
    mids = ((t[:-1].astype(np.float64) + t[1:]) / 2).astype(np.float32)  # exact ties
    v = np.concatenate([v, t, mids, np.array([0, 1e-12, 448, 447.9], np.float32)])
    mine = ref.e4m3_encode(v)
    theirs = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, theirs)


def test_e4m3_saturates():
    assert ref.e4m3_encode(np.array([448.0, 470.0, 1e9], np.float32)).tolist() == [0x7E] * 3


def test_e4m3_decode_matches_torch():
    b = np.arange(0x7F, dtype=np.uint8)
    theirs = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(ref.e4m3_decode(b), theirs)


def test_nibble_order_low_is_even():
    codes = np.array([[1, 2, 3, 4]], dtype=np.uint8)
    p = ref.pack_nibbles(codes)
    assert p.tolist() == [[0x21, 0x43]]
    assert np.array_equal(ref.unpack_nibbles(p), codes)


def test_e2m1_decode_table():
    assert ref.e2m1_decode(np.arange(16)).tolist() == [0, 0.5, 1, 1.5, 2, 3, 4, 6,
                                                       -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]


# ------------------------------------------------------------- quantiser
def test_quantize_roundtrip_error_bound():
    """Every element lands within half an E2M1 step of its scaled value."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 512), dtype=np.float32)
    q, s, g = ref.nvfp4_quantize(x)
    d = ref.nvfp4_dequantize(q, s, g)
    blk_scale = np.repeat(ref.e4m3_decode(s) * g, 16, axis=1)
    # largest E2M1 gap is 2 (between 4 and 6): error <= 1 * block scale,
    # plus the e4m3 rounding of the scale itself (<= 1/16 relative)
    assert np.all(np.abs(d - x) <= blk_scale * 1.0 + np.abs(x) * 0.07 + 1e-7)


def test_quantize_zero_and_tiny_blocks():
    x = np.zeros((2, 32), np.float32)
    x[1, 16:] = 1e-20
    q, s, g = ref.nvfp4_quantize(x)
    assert np.all(q[0] == 0) and np.all(s[0] == 0)
    assert np.all(ref.nvfp4_dequantize(q, s, g)[0] == 0)


def test_quantize_all_zero_tensor():
    q, s, g = ref.nvfp4_quantize(np.zeros((4, 64), np.float32))
    assert g == np.float32(1.0) and not q.any() and not s.any()


def test_quantize_amax_block_hits_six():
    x = np.zeros((1, 16), np.float32)
    x[0, 5] = -3.0
    q, s, g = ref.nvfp4_quantize(x)
    codes = ref.unpack_nibbles(q)[0]
    assert codes[5] == 0x8 | 7  # -6
    assert ref.e4m3_decode(s)[0, 0] == 448.0


def test_torch_dequant_equals_numpy():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((40, 256), dtype=np.float32)
    q, s, g = ref.nvfp4_quantize(x)
    a = ref.nvfp4_dequantize(q, s, g)
    b = ref.nvfp4_dequantize_torch(torch.from_numpy(q), torch.from_numpy(s), g).numpy()
    assert np.array_equal(a, b)


# ------------------------------------------------------------- GEMM oracle
def test_grouped_gemm_exact_small_integers():
    """Products of E2M1 x E4M3 values are exact; with K=16 the fp32 sum is
    exact too, so the oracle must equal a float64 reference exactly."""
    rng = np.random.default_rng(3)
    k = 16
    ca = rng.integers(0, 16, size=(5, k), dtype=np.uint8)
    cb = rng.integers(0, 16, size=(7, k), dtype=np.uint8)
    sa = np.full((5, 1), 0x38, np.uint8)  # 1.0
    sb = np.full((7, 1), 0x40, np.uint8)  # 2.0
    out = ref.grouped_gemm([ref.pack_nibbles(ca)], [sa], [ref.pack_nibbles(cb)], [sb],
                           np.array([1.0], np.float32), as_bf16=False)[0].numpy()
    exact = ref.e2m1_decode(ca).astype(np.float64) @ (ref.e2m1_decode(cb).astype(np.float64) * 2).T
    assert np.array_equal(out, exact.astype(np.float32))


def test_grouped_gemm_linearity_in_alpha():
    p = ref.random_problem([9, 4], 128, 64, seed=4)
    o1 = ref.grouped_gemm(p["a"], p["a_sf"], p["b"], p["b_sf"], np.ones(2, np.float32), as_bf16=False)
    o2 = ref.grouped_gemm(p["a"], p["a_sf"], p["b"], p["b_sf"], np.full(2, 4.0, np.float32), as_bf16=False)
    for x, y in zip(o1, o2):
        assert torch.equal(x * 4, y)


def test_check_close_rejects_wrong_and_accepts_ulp():
    r = torch.randn(32, 64)
    ok, _ = ref.check_close(r.to(torch.bfloat16), r.to(torch.bfloat16))
    assert ok
    bad = r.clone()
    bad[3, 5] += 0.5 * r.abs().max()
    ok, st = ref.check_close(bad.to(torch.bfloat16), r)
    assert not ok and st["bad"] >= 1


def test_mx_oracle_matches_direct_formula():
    p = mref.random_problem([5, 0, 3], 128, 256, seed=2)
    c = mref.fp4_grouped_gemm(p["a"], p["a_sf"], p["b"], p["b_sf"], p["m_indices"], as_bf16=False)
    a = mref.e4m3fn_decode(p["a"]).astype(np.float64)
    i = 0  # row 0 belongs to expert 0
    j = 7
    codes = ref.unpack_nibbles(p["b"][0, j])
    bval = ref.e2m1_decode(codes).astype(np.float64) * np.repeat(p["b_sf"][0, j], 32)
    aval = a[i] * np.repeat(p["a_sf"][i], 128)
    assert abs(float(c[i, j]) - float(aval @ bval)) <= 1e-4 * max(1.0, abs(float(aval @ bval)))
    pad_rows = np.nonzero(p["m_indices"] < 0)[0]
    assert float(c[pad_rows].abs().max()) == 0.0


MX_REF_ROWS = Path(__file__).resolve().parent / "golden" / "mx_reference_rows.npz"


@pytest.mark.skipif(not MX_REF_ROWS.exists(), reason="reference kernel rows not generated")
def test_mx_oracle_matches_reference_kernel_rows():
    """The MX oracle against output rows of the reference's own kernel
    (kernels/gemm/fp4_grouped_gemm/b200/kernel.py, run unmodified on a B200 by
    tests/golden/make_mx_reference.py) at its campaign point: same seeded
    inputs, the operator tolerance (the two differ in fp32 summation order)."""
    import torch

    from oracle import mx as mref
    from oracle import nvfp4 as ref

    d = np.load(MX_REF_ROWS)
    rows = d["rows"]
    got = torch.from_numpy(d["out_bf16_bits"]).view(torch.bfloat16)
    want = mref.campaign_rows_output(int(d["seed"]), rows)
    ok, st = ref.check_close(got, want)
    assert ok, st
