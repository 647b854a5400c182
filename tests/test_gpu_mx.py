"""GPU parity of the reference-format operator fp4_grouped_gemm (MXFP8 x MXFP4)
against the oracle restating kernels/gemm/fp4_grouped_gemm/b200/kernel.py:14-26.
Padding rows (m_indices == -1) are unchecked, as in the reference contract."""
import numpy as np
import pytest
import torch

from oracle import mx as mref
from oracle import nvfp4 as ref

pytestmark = pytest.mark.gpu


def _run(prob, dev):
    import ratchet_b200 as rb

    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    c = rb.fp4_grouped_gemm(t["a"].view(torch.float8_e4m3fn), t["a_sf"], t["b"], t["b_sf"],
                            t["m_indices"])
    rb.last_status()
    return c


def _check(prob, c):
    r = mref.fp4_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["m_indices"])
    valid = torch.from_numpy(prob["m_indices"] >= 0)
    ok, st = ref.check_close(c.cpu()[valid], r[valid])
    assert ok, st


@pytest.mark.parametrize("rows", [[224], [100, 0, 300, 1], [500, 224, 225]])
@pytest.mark.parametrize("n", [256, 384])
def test_mx_small(cuda_device, rows, n):
    """N=256 runs on CTA pairs, N=384 on single CTAs."""
    prob = mref.random_problem(rows, n, 512, seed=len(rows))
    _check(prob, _run(prob, cuda_device))


def test_mx_cached_prepare_reuse(cuda_device):
    """The second call on the same scale tensors reuses the device repack."""
    prob = mref.random_problem([300, 200], 384, 1024, seed=9)
    c1 = _run(prob, cuda_device)
    import ratchet_b200 as rb

    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda_device) for k, v in prob.items()}
    c2 = rb.fp4_grouped_gemm(t["a"].view(torch.float8_e4m3fn), t["a_sf"], t["b"], t["b_sf"],
                             t["m_indices"])
    c3 = rb.fp4_grouped_gemm(t["a"].view(torch.float8_e4m3fn), t["a_sf"], t["b"], t["b_sf"],
                             t["m_indices"])
    assert torch.equal(c2, c3)
    _check(prob, c1)
    _check(prob, c3)


@pytest.mark.slow
def test_mx_campaign_point_scaled(cuda_device):
    """The reference campaign geometry (G=8, N=K=4096) at ~1/4 of its rows."""
    rng = np.random.default_rng(0)
    rows = [int(v) for v in rng.integers(600, 1400, size=8)]
    prob = mref.random_problem(rows, 4096, 4096, seed=1)
    _check(prob, _run(prob, cuda_device))


@pytest.mark.slow
def test_mx_campaign_matches_reference_kernel_rows(cuda_device):
    """fp4_grouped_gemm at the reference's campaign point (8 x 4096 rows,
    N = K = 4096) against output rows that the reference's own kernel produced
    on the same seeded inputs (tests/golden/make_mx_reference.py), under the
    operator tolerance."""
    from pathlib import Path

    import bench
    import ratchet_b200 as rb

    fx = Path(__file__).resolve().parent / "golden" / "mx_reference_rows.npz"
    if not fx.exists():
        pytest.skip("reference kernel rows not generated")
    d = np.load(fx)
    args, _ = bench.mx_campaign_on_device(cuda_device, seed=int(d["seed"]))
    c = rb.fp4_grouped_gemm(*args)
    rb.last_status()
    rows = torch.from_numpy(d["rows"]).to(cuda_device)
    want = torch.from_numpy(d["out_bf16_bits"]).view(torch.bfloat16)
    ok, st = ref.check_close(c.index_select(0, rows).cpu(), want)
    assert ok, st
