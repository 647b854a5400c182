"""Expert-parallel MoE layer on B200 with the tcgen05 grouped GEMM, against
the CPU oracle: world size 1 on one GPU, and two ranks when two GPUs are
visible, over NCCL and over the peer transport; and the layer's byte-moving kernels (pack, expand plan, expand rows,
router-weighted reduce, partial-row sum) against plain PyTorch, bit-exact for
the integer and byte work.  GEMM tolerance: the operator's (max|err|/max|ref|
<= 1e-2; per element |err| <= 2e-2 |ref| + 1e-2 max|ref|)."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref
from ratchet_b200 import moe

pytestmark = pytest.mark.gpu

E, N, K, TOPK = 8, 256, 512, 4


def _weights(seed=1):
    rng = np.random.default_rng(seed)
    return [ref.nvfp4_quantize(rng.standard_normal((N, K), dtype=np.float32)) for _ in range(E)]


def _expected(xc, xs, xg, ids, w_all, w=None):
    """bf16(sum_k w[t,k] * bf16(xg * g_e * deq(x_t) . deq(W_e))) per token."""
    X = torch.from_numpy(ref.nvfp4_dequantize(xc, xs))
    Wd = [torch.from_numpy(ref.nvfp4_dequantize(c, s)) for c, s, _ in w_all]
    T = ids.shape[0]
    acc = torch.zeros((T, N))
    for e in range(E):
        sel = np.argwhere(ids == e)
        if len(sel):
            t = torch.from_numpy(sel[:, 0])
            y = ((X[t] @ Wd[e].T) * float(np.float32(xg * w_all[e][2]))).to(torch.bfloat16).float()
            wk = 1.0 if w is None else torch.from_numpy(w[sel[:, 0], sel[:, 1]])[:, None]
            acc.index_add_(0, t, y * wk)
    return acc.to(torch.bfloat16)


def _layer(w_all, owner, slot, rank, dev, max_tokens=None, transport="nccl"):
    mine = sorted(np.flatnonzero(owner == rank).tolist(), key=lambda e: slot[e])
    return moe.ExpertParallelMoE([torch.from_numpy(w_all[e][0]).to(dev) for e in mine],
                                 [torch.from_numpy(w_all[e][1]).to(dev).view(torch.float8_e4m3fn)
                                  for e in mine],
                                 [float(w_all[e][2]) for e in mine], owner, slot,
                                 max_tokens=max_tokens, transport=transport)


def _check(layer, rank, T, dev, w_all):
    rng = np.random.default_rng(100 + rank)
    xc, xs, xg = ref.nvfp4_quantize(rng.standard_normal((T, K), dtype=np.float32))
    ids, w = moe.zipf_routing(T, E, TOPK, seed=30 + rank)
    ids[3, 2] = -1  # an absent route
    args = (torch.from_numpy(xc).to(dev), torch.from_numpy(xs).to(dev).view(torch.float8_e4m3fn),
            float(xg), torch.from_numpy(ids).to(dev))
    # both forwards before the oracle's host work, so that ranks with more
    # tokens do not fall behind between two collective forwards
    got = layer.forward(*args)
    summed = layer.forward(*args, torch.from_numpy(w).to(dev))
    ok, st = ref.check_close(got.cpu().float(), _expected(xc, xs, xg, ids, w_all).float())
    ok2, st2 = ref.check_close(summed.cpu().float(), _expected(xc, xs, xg, ids, w_all, w).float())
    layer.check()
    return ok and ok2, (st, st2)


def test_moe_world1(cuda_device):
    import ratchet_b200 as rb

    w_all = _weights()
    owner, slot = moe.place_experts(moe.expert_popularity(E, seed=2), 1)
    layer = _layer(w_all, owner, slot, 0, cuda_device)
    ok, st = _check(layer, 0, 333, cuda_device, w_all)
    assert ok, st
    rb.last_status()
    layer.check()


def _graph_matches_eager(layer, rank, T, dev, replays=3):
    """Capture the layer's forward, replay it `replays` times (the peer
    transport alternates its buffer halves by epoch), and compare every
    replay with an eager forward of the same inputs, bit for bit."""
    rng = np.random.default_rng(500 + rank)
    xc, xs, xg = ref.nvfp4_quantize(rng.standard_normal((T, K), dtype=np.float32))
    ids, w = moe.zipf_routing(T, E, TOPK, seed=60 + rank)
    # the decode scale as a device tensor: a capture reads it, never copies it
    args = (torch.from_numpy(xc).to(dev), torch.from_numpy(xs).to(dev).view(torch.float8_e4m3fn),
            torch.tensor([float(xg)], device=dev), torch.from_numpy(ids).to(dev),
            torch.from_numpy(w).to(dev))
    want = layer.forward(*args).clone()
    replay, out = layer.capture(*args)
    same = True
    for _ in range(replays):
        out.zero_()
        replay()
        torch.cuda.synchronize(dev)
        same = same and torch.equal(out, want)
    layer.check()
    return same


def test_moe_world1_peer_transport(cuda_device):
    """The peer transport's kernels on one GPU (the only peer is this rank):
    dispatch into the mapped buffer, bounded waits, expand from the epoch's
    buffer half, reduce into the return buffer, sum; eager forwards over both
    halves, then graph replays equal to an eager forward."""
    w_all = _weights()
    owner, slot = moe.place_experts(moe.expert_popularity(E, seed=2), 1)
    layer = _layer(w_all, owner, slot, 0, cuda_device, max_tokens=400, transport="p2p")
    for _ in range(2):  # four forwards: each buffer half twice
        ok, st = _check(layer, 0, 333, cuda_device, w_all)
        assert ok, st
    assert int(layer.bufs["pstate"][0].item()) == 4   # the epoch counts the forwards
    assert _graph_matches_eager(layer, 0, 271, cuda_device)
    layer.release()


def test_peer_wait_gives_up_and_reports(cuda_device):
    """A wait on a flag that nothing sets: a two-rank description whose second
    rank's buffers are plain local memory that no kernel signals.  The wait
    kernel gives up after its time limit (200 ms here) with status 0x301 in
    the status word, returns, and the device stays usable."""
    import ctypes

    from ratchet_b200 import _lib

    L = _lib.lib()
    C, n = 4, 64
    rb = int(L.fgg_moe_record_bytes(K, TOPK))
    gathered = [torch.zeros(2 * 2 * C * rb, dtype=torch.uint8, device=cuda_device) for _ in range(2)]
    recv = [torch.zeros(2 * C * n, dtype=torch.bfloat16, device=cuda_device) for _ in range(2)]
    flags = [torch.zeros(2 * _lib.FGG_PEERS_MAX, dtype=torch.int64, device=cuda_device)
             for _ in range(2)]
    state = torch.zeros(4, dtype=torch.int64, device=cuda_device)
    owner = torch.zeros(E, dtype=torch.int32, device=cuda_device)
    routes = torch.zeros(C, dtype=torch.int32, device=cuda_device)
    p = _lib.FggMoePeers()
    p.owner, p.num_experts, p.routes = owner.data_ptr(), E, routes.data_ptr()
    p.wait_ms = 200  # a short limit: nothing will ever set the second rank's flag
    p.world, p.rank, p.capacity, p.n = 2, 0, C, n
    base = state.data_ptr()
    p.epoch, p.counters, p.status = base, base + 8, base + 20
    for r in range(2):
        p.gathered[r], p.recv[r], p.flags[r] = (gathered[r].data_ptr(), recv[r].data_ptr(),
                                                flags[r].data_ptr())
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    _lib.check(L.fgg_moe_wait_peers(ctypes.byref(p), 0, stream), "fgg_moe_wait_peers")
    torch.cuda.synchronize(cuda_device)
    assert (int(state[2].item()) >> 32) == 0x301
    assert float(torch.ones(8, device=cuda_device).sum().item()) == 8.0


@pytest.mark.parametrize("kh,ks", [(3584, 448), (36, 4)])
def test_gather_rows_bitexact(cuda_device, kh, ks):
    """fgg_moe_gather_rows is a byte copy: equal to index_select; an index
    outside the source is skipped and raises the flag."""
    from ratchet_b200 import _lib

    L = _lib.lib()
    g = torch.Generator(device=cuda_device).manual_seed(5)
    src_c = torch.randint(0, 256, (300, kh), dtype=torch.uint8, device=cuda_device, generator=g)
    src_s = torch.randint(0, 256, (300, ks), dtype=torch.uint8, device=cuda_device, generator=g)
    idx = torch.randint(0, 300, (1000,), dtype=torch.int32, device=cuda_device, generator=g)
    out_c = torch.empty((1000, kh), dtype=torch.uint8, device=cuda_device)
    out_s = torch.empty((1000, ks), dtype=torch.uint8, device=cuda_device)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fgg_moe_gather_rows(src_c.data_ptr(), src_s.data_ptr(), 300, kh, ks, idx.data_ptr(),
                                     1000, out_c.data_ptr(), out_s.data_ptr(), bad.data_ptr(), st),
               "gather")
    assert torch.equal(out_c, src_c.index_select(0, idx.long()))
    assert torch.equal(out_s, src_s.index_select(0, idx.long()))
    assert int(bad.item()) == 0
    idx[7] = 300  # one past the end: skipped, flagged
    _lib.check(L.fgg_moe_gather_rows(src_c.data_ptr(), src_s.data_ptr(), 300, kh, ks, idx.data_ptr(),
                                     1000, out_c.data_ptr(), out_s.data_ptr(), bad.data_ptr(), st),
               "gather")
    assert int(bad.item()) == 1


@pytest.mark.parametrize("world,T", [(1, 4096), (4, 333), (8, 1)])
def test_plan_matches_stable_argsort(cuda_device, world, T):
    """fgg_moe_plan is exactly the stable sort of the routes by (owner, slot):
    integer work, bit-exact; an expert id out of range is flagged, skipped."""
    from ratchet_b200 import _lib

    L = _lib.lib()
    Ex, topk = 64, 8
    owner, slot = moe.place_experts(moe.expert_popularity(Ex, seed=4), world)
    ids, _ = moe.zipf_routing(T, Ex, topk, seed=5)
    key = torch.from_numpy((owner[ids] * (Ex // world) + slot[ids]).reshape(-1).astype(np.int64))
    order = torch.argsort(key, stable=True)
    dev = cuda_device
    d_ids = torch.from_numpy(ids).to(dev)
    o, s_ = torch.from_numpy(owner).to(dev), torch.from_numpy(slot).to(dev)
    counts = torch.empty(Ex, dtype=torch.int32, device=dev)
    src = torch.empty(T * topk, dtype=torch.int32, device=dev)
    pos = torch.empty(T * topk, dtype=torch.int32, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fgg_moe_plan(d_ids.data_ptr(), T, topk, o.data_ptr(), s_.data_ptr(), Ex, world,
                              Ex // world, counts.data_ptr(), src.data_ptr(), pos.data_ptr(),
                              bad.data_ptr(), st), "plan")
    assert counts.cpu().tolist() == torch.bincount(key, minlength=Ex).tolist()
    assert torch.equal(src.cpu().long(), order // topk)
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel())
    assert torch.equal(pos.cpu().long(), inv)
    assert int(bad.item()) == 0
    d_ids.view(-1)[0] = Ex  # out of range: flagged, position -1
    _lib.check(L.fgg_moe_plan(d_ids.data_ptr(), T, topk, o.data_ptr(), s_.data_ptr(), Ex, world,
                              Ex // world, counts.data_ptr(), src.data_ptr(), pos.data_ptr(),
                              bad.data_ptr(), st), "plan")
    assert int(bad.item()) == 1 and int(pos[0].item()) == -1


def test_combine_matches_fp32_reference(cuda_device):
    """fgg_moe_combine against plain PyTorch fp32: sum_k w[t,k] * rows[route[t,k]],
    rounded to bf16 once (tolerance: one bf16 ulp of the result)."""
    from ratchet_b200 import _lib

    L = _lib.lib()
    T, k, n = 257, 8, 4096
    g = torch.Generator(device=cuda_device).manual_seed(6)
    rows = torch.randn((T * k, n), generator=g, device=cuda_device).to(torch.bfloat16)
    route = torch.randperm(T * k, generator=g, device=cuda_device).to(torch.int32)
    w = torch.rand((T, k), generator=g, device=cuda_device)
    out = torch.empty((T, n), dtype=torch.bfloat16, device=cuda_device)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.check(L.fgg_moe_combine(rows.data_ptr(), T * k, route.data_ptr(), w.data_ptr(), T, k, n,
                                 out.data_ptr(), bad.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "combine")
    want = (rows.float()[route.long()].view(T, k, n) * w[..., None]).sum(1)
    err = (out.float() - want).abs()
    assert (err <= want.abs() * 2.0 ** -7 + 1e-6).all()
    assert int(bad.item()) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, result_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        w_all = _weights()
        owner, slot = moe.place_experts(moe.expert_popularity(E, seed=2), world)
        layer = _layer(w_all, owner, slot, rank, dev, max_tokens=300)
        ok, st = _check(layer, rank, 120 + 23 * rank, dev, w_all)
        # the same forward with the partial rows summed by NCCL's reduce-scatter
        layer.combine = "reduce_scatter"
        ok2, st2 = _check(layer, rank, 120 + 23 * rank, dev, w_all)
        # the peer transport: records and partial rows stored into the other
        # rank's buffers by this library's kernels; each buffer half twice,
        # then graph replays equal to an eager forward
        peer = _layer(w_all, owner, slot, rank, dev, max_tokens=300, transport="p2p")
        ok3, st3 = True, []
        for _ in range(2):
            # the oracle's host work takes longer on the ranks with more tokens;
            # line the ranks up so that no flag wait spans it
            dist.barrier()
            o, s3 = _check(peer, rank, 120 + 23 * rank, dev, w_all)
            ok3, st3 = ok3 and o, st3 + [s3]
        ok4 = _graph_matches_eager(peer, rank, 100 + 25 * rank, dev)
        peer.release()
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{int(ok and ok2 and ok3 and ok4)} {st} {st2} {st3} graph={ok4}\n")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_nccl_and_peer_ranks(cuda_device, tmp_path, world):
    """world ranks, one GPU each (skipped with fewer GPUs)."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        line = (tmp_path / f"rank{r}.txt").read_text()
        assert line.startswith("1 "), f"rank {r}: {line}"


@pytest.mark.slow
def test_moe_config3_world1_full_size(cuda_device):
    """BASELINE config 3 at full size on one GPU: 4096 tokens, top-8 of 64
    experts (Zipf 1.1), N = 4096, K = 7168, with the router-weighted combine.
    A seeded sample of 256 tokens is checked, every route of each against the
    oracle: out[t] = bf16(sum_k w[t,k] * bf16(alpha_e * deq(x_t) . deq(W_e)))."""
    import bench
    import ratchet_b200 as rb

    wl = bench.workload("moe")
    d = bench.moe_setup(wl, 1, 0, cuda_device)
    layer = moe.ExpertParallelMoE(d["wc"], d["wsf"], d["wg"], d["owner"], d["slot"])
    out = layer.forward(d["xc"], d["xs"], d["xg"], d["ids"], d["wts"])
    rb.last_status()
    layer.check()
    T = wl["tokens"]
    sample = np.sort(np.random.default_rng(11).choice(T, size=256, replace=False))
    idx = torch.from_numpy(sample).to(cuda_device)
    x = ref.nvfp4_dequantize_torch(d["xc"].index_select(0, idx).cpu(),
                                   d["xs"].view(torch.uint8).index_select(0, idx).cpu())
    ids = d["ids_all"][sample]
    w = d["w_all"][sample]
    xg = float(d["xg"].item())
    acc = torch.zeros((len(sample), wl["n"]))
    for slot_i, e in enumerate(d["mine"]):
        hit = np.argwhere(ids == e)
        if not len(hit):
            continue
        wd = ref.nvfp4_dequantize_torch(d["wc"][slot_i].cpu(), d["wsf"][slot_i].view(torch.uint8).cpu())
        alpha = float(np.float32(np.float32(xg) * np.float32(d["wg"][slot_i].item())))
        rows = torch.from_numpy(hit[:, 0])
        y = ((x[rows] @ wd.T) * alpha).to(torch.bfloat16).float()
        acc.index_add_(0, rows, y * torch.from_numpy(w[hit[:, 0], hit[:, 1]])[:, None])
    want = acc.to(torch.bfloat16)
    ok, st = ref.check_close(out.index_select(0, idx).cpu(), want)
    assert ok, st


def _tok_view(codes, sf, ids, w, scale):
    from ratchet_b200 import _lib

    t = _lib.FggMoeTokens()
    t.num_tokens, t.topk, t.k = int(ids.shape[0]), int(ids.shape[1]), int(codes.shape[1]) * 2
    t.codes, t.codes_stride = codes.data_ptr(), codes.stride(0)
    t.sf, t.sf_stride = sf.data_ptr(), sf.stride(0)
    t.ids, t.ids_stride = ids.data_ptr(), 4 * ids.stride(0)
    t.weights, t.weights_stride = w.data_ptr(), 4 * w.stride(0)
    t.scale, t.scale_stride = scale.data_ptr(), 4 * scale.stride(0) if scale.numel() > 1 else 0
    return t


def test_expand_kernels_bitexact(cuda_device):
    """pack -> records view -> expand, against the same steps in PyTorch:
    every record byte, the per-expert counts, each route's row holding exactly
    that token's bytes and decode scale, and -1 for absent and remote routes."""
    from ratchet_b200 import _lib

    L = _lib.lib()
    dev = cuda_device
    st = torch.cuda.current_stream().cuda_stream
    T, k, topk, Ex, world, rank = 300, 512, 8, 64, 4, 1
    g = torch.Generator(device=dev).manual_seed(3)
    codes = torch.randint(0, 256, (T, k // 2), dtype=torch.uint8, device=dev, generator=g)
    sf = torch.randint(0, 256, (T, k // 16), dtype=torch.uint8, device=dev, generator=g)
    ids_np, w_np = moe.zipf_routing(T, Ex, topk, seed=4)
    ids_np[7, :] = -1
    ids = torch.from_numpy(ids_np).to(dev)
    w = torch.from_numpy(w_np).to(dev)
    scale = torch.rand(T, device=dev, generator=g)
    src = _tok_view(codes, sf, ids, w, scale)
    rb = L.fgg_moe_record_bytes(k, topk)
    rec = torch.empty((T, rb), dtype=torch.uint8, device=dev)
    _lib.check(L.fgg_moe_pack_tokens(src, rec.data_ptr(), st), "pack")
    kh, ks = k // 2, k // 16
    assert torch.equal(rec[:, :kh], codes) and torch.equal(rec[:, kh:kh + ks], sf)
    assert torch.equal(rec[:, kh + ks:kh + ks + 4 * topk].contiguous().view(torch.int32), ids)
    assert torch.equal(rec[:, kh + ks + 4 * topk:kh + ks + 8 * topk].contiguous().view(torch.float32), w)
    assert torch.equal(rec[:, kh + ks + 8 * topk:kh + ks + 8 * topk + 4].contiguous().view(torch.float32)[:, 0], scale)
    view = _lib.FggMoeTokens()
    _lib.check(L.fgg_moe_records_view(rec.data_ptr(), T, k, topk, view), "view")
    owner, slot = moe.place_experts(moe.expert_popularity(Ex, seed=5), world)
    loc = Ex // world
    R = T * topk
    counts = torch.full((2 * loc,), 99, dtype=torch.int32, device=dev)   # zeroed by the call
    offsets = torch.empty(loc + 1, dtype=torch.int32, device=dev)
    route_row = torch.empty(T * topk, dtype=torch.int32, device=dev)
    src_tok = torch.full((R,), -7, dtype=torch.int32, device=dev)
    rscale = torch.empty(R, dtype=torch.float32, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    o_d, s_d = torch.from_numpy(owner).to(dev), torch.from_numpy(slot).to(dev)
    a = torch.empty((R, kh), dtype=torch.uint8, device=dev)
    a_sf = torch.empty((R, ks), dtype=torch.uint8, device=dev)
    _lib.check(L.fgg_moe_expand(view, o_d.data_ptr(), s_d.data_ptr(), Ex, rank, loc, R,
                                counts.data_ptr(), offsets.data_ptr(), route_row.data_ptr(),
                                src_tok.data_ptr(), rscale.data_ptr(), a.data_ptr(),
                                a_sf.data_ptr(), bad.data_ptr(), st), "expand")
    torch.cuda.synchronize()
    assert int(bad.item()) == 0
    flat = ids_np.reshape(-1)
    is_local = (flat >= 0) & (owner[np.maximum(flat, 0)] == rank)
    cnt = np.bincount(slot[flat[is_local]], minlength=loc)
    off = offsets.cpu().numpy()
    assert off[0] == 0 and np.array_equal(np.diff(off), cnt)
    rr = route_row.cpu().numpy()
    assert (rr[~is_local] == -1).all()
    rows = rr[is_local]
    assert np.array_equal(np.sort(rows), np.arange(cnt.sum()))        # a permutation
    tok = np.flatnonzero(is_local) // topk
    for e_slot in range(loc):                                          # each row in its expert's range
        sel = slot[flat[is_local]] == e_slot
        assert ((rows[sel] >= off[e_slot]) & (rows[sel] < off[e_slot + 1])).all()
    assert np.array_equal(src_tok.cpu().numpy()[rows], tok)
    rows_t = torch.from_numpy(rows).to(dev).long()
    tok_t = torch.from_numpy(tok).to(dev).long()
    assert torch.equal(a[rows_t], codes[tok_t]) and torch.equal(a_sf[rows_t], sf[tok_t])
    assert torch.equal(rscale[rows_t], scale[tok_t])


def test_reduce_and_sum_partials_match_fp32(cuda_device):
    """fgg_moe_reduce: sum_k w[t,k] * rows[route_row[t,k]] over the routes with
    a row (fp32, one bf16 rounding; zeros for a token without one);
    fgg_moe_sum_partials: the fp32 sum of the partial rows of every source."""
    from ratchet_b200 import _lib

    L = _lib.lib()
    dev = cuda_device
    st = torch.cuda.current_stream().cuda_stream
    T, topk, n, R = 129, 8, 512, 700
    g = torch.Generator(device=dev).manual_seed(8)
    rows = torch.randn((R, n), generator=g, device=dev).to(torch.bfloat16)
    rr = torch.randint(0, R, (T, topk), generator=g, device=dev, dtype=torch.int32)
    rr[torch.rand((T, topk), generator=g, device=dev) < 0.4] = -1
    rr[5] = -1                                           # a token with no local route
    w = torch.rand((T, topk), generator=g, device=dev)
    ids = torch.zeros((T, topk), dtype=torch.int32, device=dev)
    codes = torch.zeros((T, 32), dtype=torch.uint8, device=dev)
    sf = torch.zeros((T, 4), dtype=torch.uint8, device=dev)
    scale = torch.ones(1, device=dev)
    view = _tok_view(codes, sf, ids, w, scale)
    out = torch.full((T, n), float("nan"), dtype=torch.bfloat16, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(L.fgg_moe_reduce(rows.data_ptr(), R, rr.data_ptr(), view, n, out.data_ptr(),
                                bad.data_ptr(), st), "reduce")
    valid = (rr >= 0).float()[..., None]
    want = (rows.float()[rr.clamp_min(0).long()] * w[..., None] * valid).sum(1)
    err = (out.float() - want).abs()
    assert (err <= want.abs() * 2.0 ** -7 + 1e-6).all()
    assert (out[5].float() == 0).all() and int(bad.item()) == 0
    world, per = 3, 150
    parts = torch.randn((world * per, n), generator=g, device=dev).to(torch.bfloat16)
    summed = torch.empty((T, n), dtype=torch.bfloat16, device=dev)
    _lib.check(L.fgg_moe_sum_partials(parts.data_ptr(), world, per, T, n, summed.data_ptr(), st),
               "sum")
    p3 = parts.float().view(world, per, n)[:, :T]
    want = (p3[0] + p3[1]) + p3[2]                       # the kernel's order, fp32
    assert torch.equal(summed, want.to(torch.bfloat16))
