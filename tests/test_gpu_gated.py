"""GPU parity of the gated gate+up GEMM (SiLU * up epilogue) and of the
expert MLP built on it, against the CPU oracle.  Tolerance: the operator's
(max|err|/max|ref| <= 1e-2; per element |err| <= 2e-2 |ref| + 1e-2 max|ref|).
The MLP is checked stage by stage on identical inputs: the intermediate
against the oracle of the first GEMM, the output against the oracle of the
second GEMM fed with the device's own quantised intermediate."""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref

pytestmark = pytest.mark.gpu


def _dev(prob, dev):
    t = lambda arrs: [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in arrs]
    return (t(prob["a"]), [s.view(torch.float8_e4m3fn) for s in t(prob["a_sf"])], t(prob["b"]),
            [s.view(torch.float8_e4m3fn) for s in t(prob["b_sf"])],
            torch.from_numpy(prob["alpha"]).to(dev))


@pytest.mark.parametrize("ms,inter,k", [
    ([0, 1, 15, 224, 225, 300], 128, 512),   # CTA-pair kernel (N = 256)
    ([37, 250], 192, 256),                    # single-CTA kernel (N = 384)
    ([3, 16, 9], 256, 512),                   # decode tiles (every M <= 16)
])
def test_silu_mul_matches_oracle(cuda_device, ms, inter, k):
    import ratchet_b200 as rb

    prob = ref.random_problem(ms, 2 * inter, k, seed=11)
    a, a_sf, b, b_sf, alpha = _dev(prob, cuda_device)
    w = [rb.interleave_gate_up(bb, ss) for bb, ss in zip(b, b_sf)]
    outs = rb.nvfp4_grouped_gemm_silu_mul(a, a_sf, [x[0] for x in w], [x[1] for x in w],
                                          alpha=alpha)
    rb.last_status()
    refs = ref.gated_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["alpha"])
    for g, (o, r) in enumerate(zip(outs, refs)):
        assert tuple(o.shape) == (ms[g], inter)
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g} (M={ms[g]}): {st}"


def test_expert_mlp_stages(cuda_device):
    import ratchet_b200 as rb

    ms, hidden, inter = [40, 0, 230], 256, 128
    dev = cuda_device
    prob = ref.random_problem(ms, 2 * inter, hidden, seed=12)
    a, a_sf, b13, b13_sf, alpha13 = _dev(prob, dev)
    w13 = [rb.interleave_gate_up(bb, ss) for bb, ss in zip(b13, b13_sf)]
    rng = np.random.default_rng(13)
    w2 = [ref.nvfp4_quantize(rng.standard_normal((hidden, inter), dtype=np.float32))
          for _ in ms]
    w2c = [torch.from_numpy(c).to(dev) for c, _, _ in w2]
    w2s = [torch.from_numpy(s).to(dev).view(torch.float8_e4m3fn) for _, s, _ in w2]
    w2g = torch.tensor([float(g) for _, _, g in w2], device=dev)
    y, h = rb.nvfp4_expert_mlp(a, a_sf, alpha13, [x[0] for x in w13], [x[1] for x in w13],
                               w2c, w2s, w2g)
    rb.last_status()
    # stage 1: the intermediate
    h_ref = torch.cat(ref.gated_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"],
                                             prob["alpha"]))
    ok, st = ref.check_close(h.cpu(), h_ref)
    assert ok, f"intermediate: {st}"
    # stage 2: the down projection of the device's own quantised intermediate
    hc, hs, hg = rb.quantize_nvfp4(h)
    hc, hs = hc.cpu().numpy(), hs.view(torch.uint8).cpu().numpy()
    offs = np.concatenate([[0], np.cumsum(ms)])
    y_ref = ref.grouped_gemm([hc[offs[g]:offs[g + 1]] for g in range(len(ms))],
                             [hs[offs[g]:offs[g + 1]] for g in range(len(ms))],
                             [c for c, _, _ in w2], [s for _, s, _ in w2],
                             np.array([np.float32(hg.item()) * g for _, _, g in w2],
                                      dtype=np.float32))
    for g, (o, r) in enumerate(zip(y, y_ref)):
        assert tuple(o.shape) == (ms[g], hidden)
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g}: {st}"
