"""Full-size GPU parity of the benchmark configurations against the CPU oracle.

Inputs are drawn on the device exactly as bench.py draws them (seeded N(0,1)
activations, N(0, w_std) weights, each tensor quantised to NVFP4 by the device
quantiser, which is bit-exact against the oracle's), copied to the host, and
the oracle's dequantise -> fp32 matmul -> bf16 is compared with the kernel's
output under the operator tolerance (max|err| / max|ref| <= 1e-2; per element
|err| <= 2e-2 |ref| + 1e-2 max|ref|).

  config 4  dense M = N = K = 8192 (the pair kernel, 32 K steps x 1184 tiles):
            a seeded sample of 512 output rows, every column
  config 5  decode: 256 groups, M_g ~ U[1, 16], N = 7168, K = 2048,
            W ~ N(0, 0.02) (the BN = 16 kernel with two K steps per stage):
            every group, every row
"""
import numpy as np
import pytest
import torch

import bench
from oracle import nvfp4 as ref

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _host(t):
    return t.view(torch.uint8).cpu()


def _deq(codes, sf):
    return ref.nvfp4_dequantize_torch(_host(codes), _host(sf))


def _check_rows(got, want, what):
    ok, st = ref.check_close(got.cpu(), want)
    assert ok, f"{what}: {st}"
    return st


def test_config4_dense_full_size(cuda_device):
    import ratchet_b200 as rb

    wl = bench.workload("dense")
    s = bench.make_set(wl, seed=0, dev=cuda_device)
    out = rb.nvfp4_grouped_gemm(s["a"], s["a_sf"], s["b"], s["b_sf"], s["sizes"], s["alpha"])[0]
    rb.last_status()
    rows = np.sort(np.random.default_rng(4).choice(8192, size=512, replace=False))
    idx = torch.from_numpy(rows).to(cuda_device)
    a_rows = _deq(s["a"][0].index_select(0, idx), s["a_sf"][0].view(torch.uint8).index_select(0, idx))
    b = _deq(s["b"][0], s["b_sf"][0])
    alpha = float(s["alpha"][0].item())
    want = ((a_rows @ b.T) * alpha).to(torch.bfloat16)
    st = _check_rows(out.index_select(0, idx), want, "dense 8192^3 sample rows")
    assert st["rel"] < 1e-2


def test_config5_decode_full_size(cuda_device):
    import ratchet_b200 as rb

    wl = bench.workload("decode")
    assert len(wl["m"]) == 256 and max(wl["m"]) <= 16
    s = bench.make_set(wl, seed=0, dev=cuda_device)
    outs = rb.nvfp4_grouped_gemm(s["a"], s["a_sf"], s["b"], s["b_sf"], s["sizes"], s["alpha"])
    rb.last_status()
    alpha = s["alpha"].cpu().numpy()
    worst = 0.0
    for g in range(len(wl["m"])):
        a = _deq(s["a"][g], s["a_sf"][g])
        b = _deq(s["b"][g], s["b_sf"][g])
        want = ((a @ b.T) * float(alpha[g])).to(torch.bfloat16)
        st = _check_rows(outs[g], want, f"decode group {g} (M={wl['m'][g]})")
        worst = max(worst, st["rel"])
    assert worst < 1e-2
