"""GPU parity of the NVFP4 grouped GEMM and quantiser against the CPU oracle.

Tolerance (the operator's stated bar): max|err| / max|ref| <= 1e-2 and, per
element, |err| <= 2e-2 * |ref| + 1e-2 * max|ref|.  The kernel and the oracle
see identical quantised inputs; they differ only in fp32 summation order and
the final bf16 rounding, so observed errors sit near one bf16 ulp.
The quantiser is byte work: bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref

pytestmark = pytest.mark.gpu


def _dev_problem(prob, dev):
    t = lambda arrs: [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in arrs]
    return (t(prob["a"]), [s.view(torch.float8_e4m3fn) for s in t(prob["a_sf"])], t(prob["b"]),
            [s.view(torch.float8_e4m3fn) for s in t(prob["b_sf"])],
            torch.from_numpy(prob["alpha"]).to(dev))


def _run_and_check(prob, n, k, dev, check_status=True):
    import ratchet_b200 as rb

    a, a_sf, b, b_sf, alpha = _dev_problem(prob, dev)
    sizes = [(m, n, k) for m in prob["m"]]
    outs = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, sizes, alpha)
    if check_status:
        rb.last_status()
    refs = ref.grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["alpha"])
    worst = 0.0
    for g, (o, r) in enumerate(zip(outs, refs)):
        assert tuple(o.shape) == (prob["m"][g], n)
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g} (M={prob['m'][g]}): {st}"
        worst = max(worst, st.get("rel", 0.0))
    return outs, worst


def test_quantizer_bitexact(cuda_device):
    import ratchet_b200 as rb

    rng = np.random.default_rng(7)
    x = rng.standard_normal((96, 1024), dtype=np.float32)
    x[3, :16] = 0.0                       # an all-zero block (scale 0)
    x[5, 16:32] *= 1e-3                   # a tiny block
    x[9, 100] = 37.0                      # the tensor amax lives in one block
    codes, sf, g = rb.quantize_nvfp4(torch.from_numpy(x).to(cuda_device))
    rc, rs, rg = ref.nvfp4_quantize(x)
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), rs)
    assert np.float32(g.item()) == rg


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantizer_unaligned_input_bitexact(cuda_device, dtype):
    """An input that does not start on a 16-byte boundary takes the scalar-load
    form of the quantiser: the same bytes as the oracle."""
    import ratchet_b200 as rb

    rng = np.random.default_rng(17)
    x = rng.standard_normal((37, 160), dtype=np.float32)
    xt = torch.from_numpy(x).to(dtype)
    raw = torch.empty(xt.numel() + 1, dtype=dtype, device=cuda_device)
    view = raw[1:].view(xt.shape)
    view.copy_(xt.to(cuda_device))
    assert view.data_ptr() % 16 != 0
    codes, sf, g = rb.quantize_nvfp4(view)
    rc, rs, rg = ref.nvfp4_quantize(xt.float().numpy())
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), rs)
    assert np.float32(g.item()) == rg


def test_quantizer_bf16_input(cuda_device):
    import ratchet_b200 as rb

    rng = np.random.default_rng(8)
    xb = torch.from_numpy(rng.standard_normal((33, 256), dtype=np.float32)).to(torch.bfloat16)
    codes, sf, g = rb.quantize_nvfp4(xb.to(cuda_device))
    rc, rs, rg = ref.nvfp4_quantize(xb.float().numpy())
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(sf.view(torch.uint8).cpu().numpy(), rs)


def test_quantizer_decode_scale_of_zero_tensor(cuda_device):
    """amax 0: gs = 1, so the decode scale written by the kernel is exactly 1,
    and every code and scale byte is 0 (also for an empty tensor)."""
    import ratchet_b200 as rb

    codes, sf, g = rb.quantize_nvfp4(torch.zeros((8, 64), device=cuda_device))
    assert float(g.item()) == 1.0
    assert int(codes.sum()) == 0 and int(sf.view(torch.uint8).sum()) == 0
    _, _, g0 = rb.quantize_nvfp4(torch.zeros((0, 64), device=cuda_device))
    assert float(g0.item()) == 1.0


def test_config1_single_group(cuda_device):
    """M=128, N=256, K=512, one group."""
    prob = ref.random_problem([128], 256, 512, seed=0)
    _, worst = _run_and_check(prob, 256, 512, cuda_device)
    assert worst < 1e-2


@pytest.mark.parametrize("k", [256, 512, 768, 320])
def test_ragged_groups_and_k_tails(cuda_device, k):
    """Ragged M (empty, 1, 15..17, tile edges 224/225), K not a multiple of 256."""
    ms = [0, 1, 15, 16, 17, 100, 224, 225, 449]
    prob = ref.random_problem(ms, 256, k, seed=k)
    _run_and_check(prob, 256, k, cuda_device)


@pytest.mark.parametrize("n", [384, 640])
def test_single_cta_path(cuda_device, n):
    """N % 256 != 0 takes the one-CTA kernel (pairs need 256 weight rows)."""
    prob = ref.random_problem([300, 17, 224, 1], n, 512, seed=n)
    _run_and_check(prob, n, 512, cuda_device)


@pytest.mark.parametrize("ms", [[32], [33], [200], [230, 31, 96]])
def test_pair_partial_tiles(cuda_device, ms):
    """Pair tiles whose token count is not a multiple of 32 split unevenly."""
    prob = ref.random_problem(ms, 512, 768, seed=sum(ms))
    _run_and_check(prob, 512, 768, cuda_device)


def test_decode_tiles(cuda_device):
    """All groups M <= 16 take the BN=16 decode configuration."""
    rng = np.random.default_rng(3)
    ms = [int(v) for v in rng.integers(1, 17, size=20)]
    prob = ref.random_problem(ms, 384, 1024, seed=3, w_std=0.02)
    _run_and_check(prob, 384, 1024, cuda_device)


def test_repeat_calls_bitwise_identical(cuda_device):
    prob = ref.random_problem([300, 17, 64], 512, 1024, seed=11)
    o1, _ = _run_and_check(prob, 512, 1024, cuda_device)
    o2, _ = _run_and_check(prob, 512, 1024, cuda_device)
    for x, y in zip(o1, o2):
        assert torch.equal(x, y)


def test_streams_and_workspace_reuse(cuda_device):
    """Back-to-back calls of different shapes on two streams, no host sync in
    between: each (device, stream) reuses one workspace, so every call must
    see only its own tile list and scales."""
    import ratchet_b200 as rb

    probs = [ref.random_problem([300, 17, 64], 512, 1024, seed=21),
             ref.random_problem([5, 230], 256, 512, seed=22),
             ref.random_problem([9, 16, 3, 12], 256, 768, seed=23)]
    dev_inputs = [_dev_problem(p, cuda_device) for p in probs]
    streams = [torch.cuda.Stream(cuda_device), torch.cuda.Stream(cuda_device)]
    torch.cuda.synchronize()
    outs = []
    for rep in range(3):
        for i, (p, (a, a_sf, b, b_sf, alpha)) in enumerate(zip(probs, dev_inputs)):
            with torch.cuda.stream(streams[(i + rep) % 2]):
                outs.append((i, rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha)))
    torch.cuda.synchronize()
    rb.last_status()
    refs = [ref.grouped_gemm(p["a"], p["a_sf"], p["b"], p["b_sf"], p["alpha"]) for p in probs]
    for i, o in outs:
        for g, (x, r) in enumerate(zip(o, refs[i])):
            ok, st = ref.check_close(x.cpu(), r)
            assert ok, f"problem {i} group {g}: {st}"


def test_scale_rows_not_16_byte_aligned(cuda_device):
    """K % 256 == 0 normally takes the prepare kernel's 16-byte scale loads;
    scale tensors that start 4 bytes into a buffer must take the 4-byte path
    and give the same results."""
    import ratchet_b200 as rb

    prob = ref.random_problem([200, 37, 5], 256, 512, seed=31)
    a, a_sf, b, b_sf, alpha = _dev_problem(prob, cuda_device)
    shifted = []
    for s in a_sf:
        raw = torch.empty(s.numel() + 4, dtype=torch.uint8, device=cuda_device)
        view = raw[4:].view(s.shape)
        view.copy_(s.view(torch.uint8))
        assert view.data_ptr() % 16 == 4
        shifted.append(view.view(torch.float8_e4m3fn))
    outs = rb.nvfp4_grouped_gemm(a, shifted, b, b_sf, None, alpha)
    rb.last_status()
    refs = ref.grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["alpha"])
    for g, (o, r) in enumerate(zip(outs, refs)):
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g}: {st}"
    aligned = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha)
    for x, y in zip(outs, aligned):
        assert torch.equal(x, y)


def test_alpha_applied_per_group(cuda_device):
    import ratchet_b200 as rb

    prob = ref.random_problem([40, 50], 256, 512, seed=5)
    a, a_sf, b, b_sf, _ = _dev_problem(prob, cuda_device)
    o1 = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, [1.0, 1.0])
    o2 = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, [2.0, 0.5])
    assert torch.equal(o2[0].float(), (o1[0].float() * 2).to(torch.bfloat16).float())
    assert torch.equal(o2[1].float(), (o1[1].float() * 0.5).to(torch.bfloat16).float())


def test_bad_shapes_raise(cuda_device):
    import ratchet_b200 as rb

    prob = ref.random_problem([8], 256, 512, seed=1)
    a, a_sf, b, b_sf, alpha = _dev_problem(prob, cuda_device)
    with pytest.raises(ValueError):
        rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, [(9, 256, 512)], alpha)
    bad_b = [torch.zeros((200, 256), dtype=torch.uint8, device=cuda_device)]
    bad_sf = [torch.zeros((200, 32), dtype=torch.uint8, device=cuda_device)]
    with pytest.raises(ValueError):
        rb.nvfp4_grouped_gemm(a, a_sf, bad_b, bad_sf, None, alpha)


def test_pack_cache_tracks_inplace_weight_writes(cuda_device):
    """A cached weight pack is reused for the same tensors and rebuilt after an
    in-place write to any of them."""
    import ratchet_b200 as rb

    prob = ref.random_problem([64, 30], 256, 512, seed=11)
    a, a_sf, b, b_sf, alpha = _dev_problem(prob, cuda_device)
    p1 = rb.pack_weights(b, b_sf)
    assert rb.pack_weights(b, b_sf) is p1
    o1 = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha)
    b[1].copy_(b[0])  # group 1 now holds group 0's weights
    b_sf[1].copy_(b_sf[0])
    p2 = rb.pack_weights(b, b_sf)
    assert p2 is not p1
    o2 = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha)
    assert torch.equal(o1[0], o2[0])
    refs = ref.grouped_gemm(prob["a"], prob["a_sf"], [prob["b"][0]] * 2, [prob["b_sf"][0]] * 2,
                            prob["alpha"])
    ok, st = ref.check_close(o2[1].cpu(), refs[1])
    assert ok, st


def test_out_parameter(cuda_device):
    import ratchet_b200 as rb

    prob = ref.random_problem([17, 0, 230], 256, 512, seed=12)
    a, a_sf, b, b_sf, alpha = _dev_problem(prob, cuda_device)
    want = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha)
    out = torch.full((247, 256), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    got = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha, out=out)
    assert all(g.data_ptr() == out[r:].data_ptr() for g, r in zip(got, [0, 17, 17]) if g.numel())
    assert torch.equal(torch.cat(got), torch.cat(want))
    with pytest.raises(ValueError):
        rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, alpha, out=out[:-1])


@pytest.mark.parametrize("n", [256, 384])
def test_shared_weight_groups(cuda_device, n):
    """b_index: five activation groups over two packed weight groups (the
    layout of expert chunks after an all-to-all dispatch)."""
    import ratchet_b200 as rb

    ms = [40, 0, 230, 17, 300]
    bidx = [1, 0, 1, 1, 0]
    wprob = ref.random_problem([1, 1], n, 512, seed=21)       # two weight groups
    aprob = ref.random_problem(ms, n, 512, seed=22)           # five activation groups
    a, a_sf, _, _, _ = _dev_problem(aprob, cuda_device)
    _, _, b, b_sf, _ = _dev_problem(wprob, cuda_device)
    alpha = np.asarray([0.25 * (g + 1) for g in range(5)], dtype=np.float32)
    outs = rb.nvfp4_grouped_gemm(a, a_sf, b, b_sf, None, torch.from_numpy(alpha).to(cuda_device),
                                 b_index=bidx)
    refs = ref.grouped_gemm(aprob["a"], aprob["a_sf"], [wprob["b"][i] for i in bidx],
                            [wprob["b_sf"][i] for i in bidx], alpha)
    for g, (o, r) in enumerate(zip(outs, refs)):
        ok, st = ref.check_close(o.cpu(), r)
        assert ok, f"group {g}: {st}"
    rb.last_status()


@pytest.mark.slow
def test_config2_full_size(cuda_device):
    """BASELINE configs[1] at full size: 8 groups, M ~ U[64, 1024], N=4096, K=7168."""
    rng = np.random.default_rng(0)
    ms = [int(v) for v in rng.integers(64, 1025, size=8)]
    prob = ref.random_problem(ms, 4096, 7168, seed=0)
    _run_and_check(prob, 4096, 7168, cuda_device)
