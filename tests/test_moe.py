"""Host logic of the expert-parallel MoE layer (ratchet_b200/moe.py) on CPU:
routing, placement, the dispatch plan, and a full forward at world size 1
and over two gloo ranks.  The expert GEMM is the CPU oracle here (the layer
accepts a stand-in GEMM for exactly this purpose); the GPU tests run the
same forward with the tcgen05 kernel.

Expected output of token t: the router-weighted sum of its routes,
    bf16( sum_k w[t,k] * bf16( x_scale * w_scale[e] * deq(x_t) . deq(W_e)^T ) )
(weights of 1 when none are given), compared within the operator tolerance
(the oracle GEMM sums a chunk of rows at once, the expected value one row at
a time).
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ref
from ratchet_b200 import moe


def test_zipf_routing_distinct_and_deterministic():
    ids, w = moe.zipf_routing(512, 16, 4, s=1.1, seed=3)
    assert ids.shape == (512, 4) and ids.dtype == np.int32
    assert all(len(set(row)) == 4 for row in ids.tolist())
    assert np.allclose(w.sum(1), 1.0, atol=1e-6) and (w > 0).all()
    ids2, w2 = moe.zipf_routing(512, 16, 4, s=1.1, seed=3)
    assert np.array_equal(ids, ids2) and np.array_equal(w, w2)
    counts = np.bincount(ids.ravel(), minlength=16)
    pop = moe.expert_popularity(16, s=1.1, seed=3)
    assert counts.max() <= 512
    assert np.argmax(counts) == np.argmax(pop)  # the most popular expert gets the most rows


def test_place_experts_equal_counts_and_spread():
    pop = moe.expert_popularity(64, seed=0)
    for world in (1, 2, 4, 8):
        owner, slot = moe.place_experts(pop, world)
        assert np.array_equal(np.bincount(owner, minlength=world), np.full(world, 64 // world))
        for r in range(world):
            assert sorted(slot[owner == r].tolist()) == list(range(64 // world))
        load = np.bincount(owner, weights=pop, minlength=world)
        assert load.max() - load.min() <= pop.max() + 1e-12
    with pytest.raises(ValueError):
        moe.place_experts(pop, 3)


def _weights(E, n, k, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(E):
        c, s, g = ref.nvfp4_quantize(rng.standard_normal((n, k), dtype=np.float32))
        out.append((c, s, np.float32(g)))
    return out


def _tokens(T, k, seed):
    rng = np.random.default_rng(seed)
    return ref.nvfp4_quantize(rng.standard_normal((T, k), dtype=np.float32))


def _oracle_gemm(local_w):
    deq = [ref.nvfp4_dequantize(c, s) for c, s, _ in local_w]

    def fn(a_list, sf_list, b_index, alpha, out):
        r = 0
        for g, (a, s) in enumerate(zip(a_list, sf_list)):
            m = int(a.shape[0])
            if m:
                A = ref.nvfp4_dequantize(a.numpy(), s.view(torch.uint8).numpy())
                y = (A @ deq[b_index[g]].T) * np.float32(alpha[g].item())
                out[r:r + m] = torch.from_numpy(y).to(torch.bfloat16)
            r += m
    return fn


def _expected(xc, xs, xg, ids, weights_all, w=None):
    """Router-weighted sum per token: bf16(sum_k w[t,k] * bf16(route output))
    (weights of 1 when w is None); ids < 0 are absent routes."""
    X = ref.nvfp4_dequantize(xc, xs)
    T, K = ids.shape
    n = weights_all[0][0].shape[0]
    out = np.zeros((T, n), dtype=np.float32)
    for t in range(T):
        for k in range(K):
            if ids[t, k] < 0:
                continue
            c, s, g = weights_all[ids[t, k]]
            y = (X[t:t + 1] @ ref.nvfp4_dequantize(c, s).T)[0] * np.float32(xg * g)
            y = torch.from_numpy(y).to(torch.bfloat16).float().numpy()
            out[t] += (1.0 if w is None else w[t, k]) * y
    return torch.from_numpy(out).to(torch.bfloat16)


def _build_layer(weights_all, owner, slot, rank, max_tokens=None):
    mine = [weights_all[e] for e in np.flatnonzero(owner == rank)]
    mine = [mine[i] for i in np.argsort([slot[e] for e in np.flatnonzero(owner == rank)])]
    return moe.ExpertParallelMoE([torch.from_numpy(c) for c, _, _ in mine],
                                 [torch.from_numpy(s) for _, s, _ in mine],
                                 [float(g) for _, _, g in mine], owner, slot,
                                 gemm_fn=_oracle_gemm(mine), max_tokens=max_tokens)


def test_forward_world1_matches_oracle():
    E, n, k, T, topk = 8, 32, 64, 45, 3
    weights_all = _weights(E, n, k, seed=1)
    owner, slot = moe.place_experts(moe.expert_popularity(E, seed=2), 1)
    layer = _build_layer(weights_all, owner, slot, 0)
    ids, w = moe.zipf_routing(T, E, topk, seed=2)
    ids[5, 1] = -1                        # an absent route
    xc, xs, xg = _tokens(T, k, seed=4)
    got = layer.forward(torch.from_numpy(xc), torch.from_numpy(xs), float(xg), torch.from_numpy(ids))
    ok, st = ref.check_close(got.float(), _expected(xc, xs, xg, ids, weights_all).float())
    assert ok, st
    summed = layer.forward(torch.from_numpy(xc), torch.from_numpy(xs), float(xg),
                           torch.from_numpy(ids), torch.from_numpy(w))
    ok, st = ref.check_close(summed.float(), _expected(xc, xs, xg, ids, weights_all, w).float())
    assert ok, st


def test_capacity_is_enforced():
    E, n, k = 4, 16, 64
    weights_all = _weights(E, n, k, seed=5)
    owner, slot = moe.place_experts(np.ones(E), 1)
    layer = _build_layer(weights_all, owner, slot, 0, max_tokens=8)
    xc, xs, xg = _tokens(9, k, seed=6)
    ids, _ = moe.zipf_routing(9, E, 2, seed=7)
    with pytest.raises(ValueError):
        layer.forward(torch.from_numpy(xc), torch.from_numpy(xs), float(xg), torch.from_numpy(ids))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, n, k, T, topk = 8, 32, 64, 37 + 11 * rank, 3
        weights_all = _weights(E, n, k, seed=1)           # the same experts on every rank
        owner, slot = moe.place_experts(moe.expert_popularity(E, seed=2), world)
        # ranks pass different token counts under one dispatch capacity
        layer = _build_layer(weights_all, owner, slot, rank, max_tokens=64)
        ids, w = moe.zipf_routing(T, E, topk, seed=10 + rank)
        xc, xs, xg = _tokens(T, k, seed=20 + rank)         # each rank its own tokens and scale
        got = layer.forward(torch.from_numpy(xc), torch.from_numpy(xs), float(xg),
                            torch.from_numpy(ids))
        ok, st = ref.check_close(got.float(), _expected(xc, xs, xg, ids, weights_all).float())
        summed = layer.forward(torch.from_numpy(xc), torch.from_numpy(xs), float(xg),
                               torch.from_numpy(ids), torch.from_numpy(w))
        ok2, st2 = ref.check_close(summed.float(),
                                   _expected(xc, xs, xg, ids, weights_all, w).float())
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{int(ok and ok2)} {st} {st2}\n")
    finally:
        dist.destroy_process_group()


def test_forward_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        line = (tmp_path / f"rank{r}.txt").read_text()
        assert line.startswith("1 "), f"rank {r}: {line}"


def test_routed_load_is_topk_inclusion():
    """Expected rows per token: sums to topk, never above 1 per expert, ranks
    the experts like their popularity, and balances a placement of a sampled
    batch far better than the raw popularity at two and four ranks."""
    E, topk = 64, 8
    load = moe.routed_load(E, topk, samples=16384)
    assert abs(load.sum() - topk) < 1e-9 and (load <= 1.0).all()
    pop = moe.expert_popularity(E)
    top = np.argsort(-pop)[:8]
    assert np.array_equal(np.argsort(-load)[:8], top)   # the popular experts, in order
    ids, _ = moe.zipf_routing(4096, E, topk, seed=0)
    cnt = np.bincount(ids.ravel(), minlength=E)
    for world in (2, 4):
        by_load = [cnt[moe.place_experts(load, world)[0] == r].sum() for r in range(world)]
        by_pop = [cnt[moe.place_experts(pop, world)[0] == r].sum() for r in range(world)]
        assert max(by_load) / np.mean(by_load) < 1.03 < max(by_pop) / np.mean(by_pop)


def test_layer_options_validated():
    """Bad transport, combine or wait limit names are refused up front."""
    E, n, k = 4, 16, 64
    weights_all = _weights(E, n, k, seed=8)
    owner, slot = moe.place_experts(np.ones(E), 1)
    mine = [weights_all[e] for e in range(E)]
    args = ([torch.from_numpy(c) for c, _, _ in mine], [torch.from_numpy(s) for _, s, _ in mine],
            [float(g) for _, _, g in mine], owner, slot)
    with pytest.raises(ValueError):
        moe.ExpertParallelMoE(*args, gemm_fn=_oracle_gemm(mine), transport="shm")
    with pytest.raises(ValueError):
        moe.ExpertParallelMoE(*args, gemm_fn=_oracle_gemm(mine), combine="allreduce")
    with pytest.raises(ValueError):
        moe.ExpertParallelMoE(*args, gemm_fn=_oracle_gemm(mine), transport="p2p", wait_ms=-1)
    layer = moe.ExpertParallelMoE(*args, gemm_fn=_oracle_gemm(mine), transport="p2p", wait_ms=250)
    assert layer.wait_ms == 250 and layer.transport == "p2p"
