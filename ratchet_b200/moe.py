"""Expert-parallel NVFP4 MoE layer: route -> dispatch -> grouped GEMM -> combine.

The single-GPU analogue in the reference is `_moe_forward`
(tasks/muse_prefill_boundary/reference/submission.py:843-895): a gather plan
puts the routed token rows of each expert together, one grouped GEMM runs
every expert, and a combine weights the rows and sums them back per token.
Here the experts are sharded over the ranks of a process group (one process
per GPU) and the tokens travel between ranks.

No size ever reaches the host, so a forward never synchronises it (and can be
captured in a CUDA graph).  That fixes the exchange buffers' shapes: a
dispatch that can never overflow gives every (source, destination) pair room
for all of the source's tokens (`max_tokens`, the per-rank capacity), and at
that capacity the dispatch moves exactly the bytes of an all-gather of the
tokens.  So a forward is:

  1. pack       each token becomes one record (NVFP4 codes and scales, its
                top-k expert ids and router weights, its rank's decode
                scale); slots past the rank's tokens carry no route
  2. dispatch   NCCL all-gather of the records (one NVLink crossing per token
                and rank)
  3. expand     every rank plans the routes of its own experts (expert by
                expert) and gathers their token rows into one buffer
  4. GEMM       one grouped GEMM over the expanded rows with the plan's device
                offsets (fgg_nvfp4_grouped_gemm_rows); each row carries its
                source's decode scale as a row factor
  5. combine    each rank sums every token's local routes with their router
                weights into one partial row per token, an equal-split NCCL
                all-to-all returns each source its tokens' partial rows, and
                the source sums them in fp32

At world size 1 steps 1, 2 and the exchange of step 5 drop out: the expand
reads the caller's tensors and the weighted sum is the output.

Collectives go through torch.distributed (NCCL on GPUs, gloo for the CPU
tests of the host logic).  `gemm_fn` replaces the device path with a host
emulation of the same steps (torch CPU ops around a stand-in GEMM), only to
test the host logic without a GPU.
"""
from __future__ import annotations

from typing import Callable, Sequence

import numpy as np
import torch

from . import _lib, ops


# ------------------------------------------------------------------ routing
def zipf_routing(num_tokens: int, num_experts: int, topk: int, s: float = 1.1, seed: int = 0):
    """Seeded top-k routing with Zipf(s) expert popularity.

    A seeded permutation ranks the experts; expert with rank r (1-based) has
    weight r^-s.  Each token draws `topk` DISTINCT experts without
    replacement in proportion to those weights (Gumbel top-k), so no expert
    receives more than `num_tokens` rows.  Router weights are the drawn
    experts' popularity renormalised over the token's k routes.
    Returns (ids int32 [T, k], weights float32 [T, k]).
    """
    if not 0 < topk <= num_experts:
        raise ValueError(f"topk={topk} must be in [1, {num_experts}]")
    rng = np.random.default_rng(seed)
    rank_of = rng.permutation(num_experts)  # expert e has popularity rank rank_of[e]
    pop = (rank_of + 1.0) ** (-s)
    pop /= pop.sum()
    gumbel = -np.log(-np.log(rng.random((num_tokens, num_experts))))
    keys = np.log(pop)[None, :] + gumbel
    ids = np.argpartition(-keys, topk - 1, axis=1)[:, :topk]
    # order each token's routes by key (largest first) so the result is deterministic
    kk = np.take_along_axis(keys, ids, axis=1)
    ids = np.take_along_axis(ids, np.argsort(-kk, axis=1), axis=1).astype(np.int32)
    w = pop[ids]
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def expert_popularity(num_experts: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """The per-expert weights zipf_routing draws with (same seed, same order)."""
    rng = np.random.default_rng(seed)
    rank_of = rng.permutation(num_experts)
    pop = (rank_of + 1.0) ** (-s)
    return pop / pop.sum()


def routed_load(num_experts: int, topk: int, s: float = 1.1, seed: int = 0,
                samples: int = 65536, sample_seed: int = 12345) -> np.ndarray:
    """Expected rows per token of each expert under zipf_routing(seed):
    the probability that the expert is among a token's `topk` distinct
    draws.  Drawing without replacement flattens the popularity (an expert
    takes at most one route per token), so this, not the popularity itself,
    is the load a placement must balance.  Estimated from `samples` draws
    with their own seed, independent of any batch being served."""
    pop = expert_popularity(num_experts, s=s, seed=seed)
    rng = np.random.default_rng(sample_seed)
    counts = np.zeros(num_experts, dtype=np.int64)
    chunk = 8192
    for start in range(0, samples, chunk):
        m = min(chunk, samples - start)
        keys = np.log(pop)[None, :] - np.log(-np.log(rng.random((m, num_experts))))
        sel = np.argpartition(-keys, topk - 1, axis=1)[:, :topk]
        counts += np.bincount(sel.ravel(), minlength=num_experts)
    return counts / float(samples)


def place_experts(load: Sequence[float], world: int):
    """Static expert -> rank placement that spreads the expected load.

    Longest-processing-time first with equal expert counts per rank: experts
    in decreasing load go to the least-loaded rank that still has room
    (ties: lower rank).  Returns (owner int32 [E], slot int32 [E]) where
    slot is the expert's index among its owner's experts, in expert order.
    """
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    if world < 1 or E % world != 0:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    per = E // world
    owner = np.full(E, -1, dtype=np.int32)
    acc = np.zeros(world)
    cnt = np.zeros(world, dtype=np.int64)
    for e in sorted(range(E), key=lambda e: (-load[e], e)):
        room = [r for r in range(world) if cnt[r] < per]
        r = min(room, key=lambda r: (acc[r], r))
        owner[e] = r
        acc[r] += load[e]
        cnt[r] += 1
    slot = np.zeros(E, dtype=np.int32)
    for r in range(world):
        for i, e in enumerate(np.flatnonzero(owner == r)):
            slot[e] = i
    return owner, slot


# ------------------------------------------------------------------ layer
GemmFn = Callable[[list, list, list, torch.Tensor, torch.Tensor], None]

PHASES = ("pack", "dispatch", "expand", "gemm", "reduce", "combine", "sum")


class ExpertParallelMoE:
    """One expert-parallel MoE projection (e.g. the fused gate+up of every
    expert) over the ranks of `group`.

    w_codes / w_sf / w_scale: this rank's experts, in slot order: codes
    [N, K/2] uint8, E4M3 scales [N, K/16], fp32 decode scale (0-dim tensor
    or float).  owner / slot: the placement of every expert (place_experts).
    max_tokens: the dispatch capacity, the most tokens any rank passes to one
    forward (every rank must use the same value); default: the first
    forward's token count.  topk: routes per token (default: the first
    forward's).  combine: "a2a" returns the partial rows with an equal-split
    all-to-all and sums them in fp32 on the token's rank; "reduce_scatter"
    lets NCCL sum them on the way (bf16 additions, one rounding per step of
    its reduction).  transport: "nccl" moves the records and partial rows
    with NCCL collectives; "p2p" with the library's own kernels, which store
    them straight into the other ranks' buffers over NVLink (peer memory
    mapped through CUDA IPC, epoch-tagged arrival flags, bounded waits),
    fuse the exchange with the packing and the final sum, and move a
    token's record and partial row only to and from the ranks that own one
    of its experts; call release() before destroying the process group.
    wait_ms: the limit of each wait on the other ranks' flags (0: the
    library's default, 10 s); a wait that runs out makes check() raise.
    """

    def __init__(self, w_codes: Sequence[torch.Tensor], w_sf: Sequence[torch.Tensor],
                 w_scale: Sequence, owner: np.ndarray, slot: np.ndarray, group=None,
                 gemm_fn: GemmFn | None = None, max_tokens: int | None = None,
                 combine: str = "a2a", transport: str = "nccl", wait_ms: int = 0):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        owner = np.asarray(owner, dtype=np.int32)
        slot = np.asarray(slot, dtype=np.int32)
        if owner.max() >= self.world or owner.min() < 0:
            raise ValueError("owner names a rank outside the process group")
        self.num_experts = int(owner.shape[0])
        self.local = int((owner == self.rank).sum())
        if self.local != len(w_codes) or len(w_codes) != len(w_sf) or len(w_sf) != len(w_scale):
            raise ValueError(f"rank {self.rank} owns {self.local} experts, got {len(w_codes)} weights")
        counts = np.bincount(owner, minlength=self.world)
        if (counts != counts[0]).any():
            raise ValueError("every rank must own the same number of experts")
        self.w_codes = list(w_codes)
        self.w_sf = list(w_sf)
        self.n = int(self.w_codes[0].shape[0])
        self.k = int(self.w_codes[0].shape[1]) * 2
        dev = self.w_codes[0].device
        self.device = dev
        self.w_scale = torch.stack([torch.as_tensor(s, dtype=torch.float32, device=dev).reshape(())
                                    for s in w_scale]).contiguous()
        self.owner_np, self.slot_np = owner, slot
        self.gemm_fn = gemm_fn
        self.max_tokens = max_tokens
        if combine not in ("a2a", "reduce_scatter"):
            raise ValueError(f"combine={combine!r}: 'a2a' or 'reduce_scatter'")
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport={transport!r}: 'nccl' or 'p2p'")
        if transport == "p2p" and self.world > _lib.FGG_PEERS_MAX:
            raise ValueError(f"the peer exchange spans at most {_lib.FGG_PEERS_MAX} ranks")
        self.combine = combine
        self.transport = transport
        if wait_ms < 0:
            raise ValueError("wait_ms must be >= 0 (0: the library's default)")
        self.wait_ms = int(wait_ms)
        self._peer_own = []      # buffers this rank allocated (freed by release)
        self._peer_mapped = []   # other ranks' buffers mapped here (closed by release)
        self.topk = None
        self.bufs = None
        self.pack = None
        self.bad = None
        self._graph = None
        if gemm_fn is None:
            # the product path: weights packed once and reused by every
            # forward; the kernels raise this flag on a bad id or index
            self.pack = ops.pack_weights(self.w_codes, self.w_sf)
            self.bad = torch.zeros(1, dtype=torch.int32, device=dev)
            self.owner_d = torch.from_numpy(owner).to(dev)
            self.slot_d = torch.from_numpy(slot).to(dev)

    # ---------------------------------------------------------- buffers
    def _buffers(self, T: int, topk: int):
        """Device buffers of one forward geometry, made on first use."""
        if self.max_tokens is None:
            self.max_tokens = T
        if self.topk is None:
            self.topk = topk
        C, W, E = self.max_tokens, self.world, self.local
        if T > C:
            raise ValueError(f"{T} tokens exceed the layer's dispatch capacity max_tokens={C}")
        if topk != self.topk:
            raise ValueError(f"topk={topk}, the layer was set up for {self.topk}")
        if self.bufs is not None:
            return self.bufs
        L = _lib.lib()
        dev, kh, ks, n = self.device, self.k // 2, self.k // 16, self.n
        NT = W * C if W > 1 else C           # tokens the expand plan walks
        R = NT * min(topk, E)                # local routes at most
        b = {"NT": NT, "R": R}
        if self.transport == "p2p":
            self._peer_setup(b, C, topk)
        elif W > 1:
            rb = int(L.fgg_moe_record_bytes(self.k, topk))
            b["rb"] = rb
            b["records"] = torch.empty((C, rb), dtype=torch.uint8, device=dev)
            b["gathered"] = torch.empty((W * C, rb), dtype=torch.uint8, device=dev)
            b["partial"] = torch.empty((W * C, n), dtype=torch.bfloat16, device=dev)
            b["recv"] = torch.empty((W * C, n), dtype=torch.bfloat16, device=dev)
            toks = _lib.FggMoeTokens()
            _lib.check(L.fgg_moe_records_view(b["gathered"].data_ptr(), W * C, self.k, topk, toks),
                       "fgg_moe_records_view")
            b["gathered_view"] = toks
        b["counts"] = torch.empty(2 * E, dtype=torch.int32, device=dev)
        b["offsets"] = torch.empty(E + 1, dtype=torch.int32, device=dev)
        b["route_row"] = torch.empty(NT * topk, dtype=torch.int32, device=dev)
        b["src_token"] = torch.empty(R, dtype=torch.int32, device=dev)
        b["row_scale"] = torch.empty(R, dtype=torch.float32, device=dev)
        b["a"] = torch.empty((R, kh), dtype=torch.uint8, device=dev)
        b["a_sf"] = torch.empty((R, ks), dtype=torch.uint8, device=dev)
        b["y"] = torch.empty((R, n), dtype=torch.bfloat16, device=dev)
        prob = _lib.FggNvfp4RowsProblem(E, n, self.k, R, b["offsets"].data_ptr(), b["a"].data_ptr(),
                                        b["a_sf"].data_ptr(), self.w_scale.data_ptr(),
                                        b["y"].data_ptr(), b["row_scale"].data_ptr(), None, E, 0)
        nbytes = int(L.fgg_nvfp4_rows_workspace_bytes(prob))
        if nbytes == 0:
            _lib.check(L.fgg_nvfp4_grouped_gemm_rows(prob, None, None, 0, None), "grouped GEMM")
        b["prob"] = prob
        b["ws"] = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.bufs = b
        return b

    def _peer_setup(self, b: dict, C: int, topk: int) -> None:
        """Allocate this rank's exchange buffers, map every other rank's
        (CUDA IPC handles swapped through the process group), and describe
        them in an FggMoePeers struct.  Collective: every rank calls it."""
        import ctypes

        import torch.distributed as dist

        L = _lib.lib()
        W, n, dev = self.world, self.n, self.device
        rb = int(L.fgg_moe_record_bytes(self.k, topk))
        # records (two halves), partial rows (one), arrival flags
        sizes = (2 * W * C * rb, W * C * n * 2, 2 * _lib.FGG_PEERS_MAX * 8)
        own = []
        hb = int(L.fgg_peer_handle_bytes())
        handles = []
        try:
            with torch.cuda.device(dev):
                for nbytes in sizes:
                    p = ctypes.c_void_p()
                    _lib.check(L.fgg_peer_alloc(nbytes, ctypes.byref(p)), "fgg_peer_alloc")
                    own.append(p.value)
                    self._peer_own.append(p.value)
                    h = ctypes.create_string_buffer(hb)
                    _lib.check(L.fgg_peer_export(p.value, h), "fgg_peer_export")
                    handles.append(h.raw)
            everyone = [handles]
            if W > 1:
                everyone = [None] * W
                dist.all_gather_object(everyone, handles, group=self.group)
            ptrs = [[0] * W for _ in sizes]
            with torch.cuda.device(dev):
                for r in range(W):
                    for i in range(len(sizes)):
                        if r == self.rank:
                            ptrs[i][r] = own[i]
                            continue
                        q = ctypes.c_void_p()
                        _lib.check(L.fgg_peer_import(everyone[r][i], ctypes.byref(q)),
                                   "fgg_peer_import")
                        self._peer_mapped.append(q.value)
                        ptrs[i][r] = q.value
        except Exception:
            # give back what this rank holds (no collective: the others may be
            # failing too, and their process group ends their part)
            with torch.cuda.device(dev):
                for q in self._peer_mapped:
                    L.fgg_peer_close(q)
                for q in self._peer_own:
                    L.fgg_peer_free(q)
            self._peer_mapped, self._peer_own = [], []
            raise
        # this rank's own state: epoch (int64), three block counters, status
        b["pstate"] = torch.zeros(4, dtype=torch.int64, device=dev)
        base = b["pstate"].data_ptr()
        peers = _lib.FggMoePeers()
        peers.world, peers.rank, peers.capacity, peers.n = W, self.rank, C, n
        peers.epoch, peers.counters, peers.status = base, base + 8, base + 20
        for r in range(W):
            peers.gathered[r] = ptrs[0][r]
            peers.recv[r] = ptrs[1][r]
            peers.flags[r] = ptrs[2][r]
        # each token's destination ranks, from the dispatch to the sum
        b["routes"] = torch.zeros(C, dtype=torch.int32, device=dev)
        peers.owner, peers.num_experts = self.owner_d.data_ptr(), self.num_experts
        peers.routes = b["routes"].data_ptr()
        peers.wait_ms = self.wait_ms
        b["peers"] = peers
        b["rb"] = rb
        toks = _lib.FggMoeTokens()
        _lib.check(L.fgg_moe_records_view(own[0], W * C, self.k, topk, toks), "fgg_moe_records_view")
        toks.epoch, toks.parity_bytes = base, W * C * rb   # this forward's half
        b["gathered_view"] = toks
        if W > 1:
            dist.barrier(group=self.group)

    def _tokens_view(self, x_u8, s_u8, ids32, w32, xs):
        T, topk = int(ids32.shape[0]), int(ids32.shape[1])
        t = _lib.FggMoeTokens()
        t.num_tokens, t.topk, t.k = T, topk, self.k
        t.codes, t.codes_stride = x_u8.data_ptr(), x_u8.stride(0)
        t.sf, t.sf_stride = s_u8.data_ptr(), s_u8.stride(0)
        t.ids, t.ids_stride = ids32.data_ptr(), 4 * ids32.stride(0)
        t.weights, t.weights_stride = (w32.data_ptr(), 4 * w32.stride(0)) if w32 is not None else (None, 0)
        t.scale, t.scale_stride = xs.data_ptr(), 0
        return t

    def _a2a(self, out, inp):
        import torch.distributed as dist

        if inp.dtype == torch.bfloat16:  # rows as bytes: bit-exact on every backend
            out, inp = out.view(torch.uint8), inp.view(torch.uint8)
        dist.all_to_all_single(out, inp, group=self.group)

    # ---------------------------------------------------------- forward
    def forward(self, x_codes: torch.Tensor, x_sf: torch.Tensor, x_scale, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor | None = None, events: dict | None = None) -> torch.Tensor:
        """x_codes [T, K/2] uint8 and x_sf [T, K/16] E4M3: this rank's tokens,
        quantised with decode scale x_scale.  topk_ids [T, k] expert ids (an
        id < 0 is an absent route).  Returns [T, N] bf16, the router-weighted
        sum over each token's routes (topk_weights [T, k]; None = weights of 1).
        events: optional dict; CUDA events (start of each of PHASES, and "end")
        are recorded into it on the current stream, for a per-phase breakdown."""
        T, topk = int(topk_ids.shape[0]), int(topk_ids.shape[1])
        kh, ks = self.k // 2, self.k // 16
        x_u8 = x_codes.view(torch.uint8)
        s_u8 = x_sf.view(torch.uint8)
        if x_u8.shape != (T, kh) or s_u8.shape != (T, ks):
            raise ValueError(f"x_codes {tuple(x_u8.shape)} / x_sf {tuple(s_u8.shape)} do not match "
                             f"T={T}, K={self.k}")
        if self.gemm_fn is not None:
            return self._forward_host(x_u8, s_u8, x_scale, topk_ids, topk_weights)
        b = self._buffers(T, topk)
        dev = self.device
        L = _lib.lib()
        stream = ops._stream_ptr(dev)
        W, E, n, C = self.world, self.local, self.n, self.max_tokens

        def mark(name):
            if events is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                events[name] = ev

        ids32 = topk_ids.to(device=dev, dtype=torch.int32).contiguous()
        w32 = None if topk_weights is None else topk_weights.to(device=dev, dtype=torch.float32).contiguous()
        xs = torch.as_tensor(x_scale, dtype=torch.float32, device=dev).reshape(1)
        mine = self._tokens_view(x_u8, s_u8, ids32, w32, xs)
        mark("pack")
        if self.transport == "p2p":
            return self._forward_peers(b, mine, T, mark, stream)
        if W > 1:
            if T < C:  # slots past this rank's tokens carry no route (expert id -1)
                b["records"][T:, kh + ks:kh + ks + 4 * topk].view(torch.int32).fill_(-1)
            _lib.check(L.fgg_moe_pack_tokens(mine, b["records"].data_ptr(), stream), "fgg_moe_pack_tokens")
            mark("dispatch")
            import torch.distributed as dist

            dist.all_gather_into_tensor(b["gathered"], b["records"], group=self.group)
            toks = b["gathered_view"]
        else:
            mark("dispatch")
            toks = mine
        mark("expand")
        _lib.check(L.fgg_moe_expand(toks, self.owner_d.data_ptr(), self.slot_d.data_ptr(),
                                    self.num_experts, self.rank, E, b["R"], b["counts"].data_ptr(),
                                    b["offsets"].data_ptr(), b["route_row"].data_ptr(),
                                    b["src_token"].data_ptr(), b["row_scale"].data_ptr(),
                                    b["a"].data_ptr(), b["a_sf"].data_ptr(), self.bad.data_ptr(),
                                    stream), "fgg_moe_expand")
        mark("gemm")
        _lib.check(L.fgg_nvfp4_grouped_gemm_rows(b["prob"], self.pack.buf.data_ptr(),
                                                 b["ws"].data_ptr(), b["ws"].numel(), stream),
                   "fgg_nvfp4_grouped_gemm_rows")
        ops._set_last_ws(b["ws"])
        mark("reduce")
        out = torch.empty((T, n), dtype=torch.bfloat16, device=dev)
        target = b["partial"] if W > 1 else out
        _lib.check(L.fgg_moe_reduce(b["y"].data_ptr(), b["R"], b["route_row"].data_ptr(), toks, n,
                                    target.data_ptr(), self.bad.data_ptr(), stream), "fgg_moe_reduce")
        mark("combine")
        if W > 1 and self.combine == "reduce_scatter":
            import torch.distributed as dist

            summed = torch.empty((C, n), dtype=torch.bfloat16, device=dev)
            dist.reduce_scatter_tensor(summed, b["partial"], group=self.group)
            mark("sum")
            mark("end")
            return summed[:T]
        if W > 1:
            self._a2a(b["recv"], b["partial"])
        mark("sum")
        if W > 1:
            _lib.check(L.fgg_moe_sum_partials(b["recv"].data_ptr(), W, C, T, n, out.data_ptr(), stream),
                       "fgg_moe_sum_partials")
        mark("end")
        return out

    def _forward_peers(self, b, mine, T, mark, stream):
        """Steps 1-6 over peer memory: the dispatch kernel stores each record
        in the ranks that own one of its experts, the reduce kernel writes the
        partial rows into this rank's own return buffer and the sum kernel
        reads a token's partial rows from the ranks that computed them, with
        bounded waits on the arrival flags between."""
        L = _lib.lib()
        E, n, dev = self.local, self.n, self.device
        peers, toks = b["peers"], b["gathered_view"]
        _lib.check(L.fgg_moe_dispatch_peers(mine, peers, stream), "fgg_moe_dispatch_peers")
        mark("dispatch")
        _lib.check(L.fgg_moe_wait_peers(peers, 0, stream), "fgg_moe_wait_peers")
        mark("expand")
        _lib.check(L.fgg_moe_expand(toks, self.owner_d.data_ptr(), self.slot_d.data_ptr(),
                                    self.num_experts, self.rank, E, b["R"], b["counts"].data_ptr(),
                                    b["offsets"].data_ptr(), b["route_row"].data_ptr(),
                                    b["src_token"].data_ptr(), b["row_scale"].data_ptr(),
                                    b["a"].data_ptr(), b["a_sf"].data_ptr(), self.bad.data_ptr(),
                                    stream), "fgg_moe_expand")
        mark("gemm")
        _lib.check(L.fgg_nvfp4_grouped_gemm_rows(b["prob"], self.pack.buf.data_ptr(),
                                                 b["ws"].data_ptr(), b["ws"].numel(), stream),
                   "fgg_nvfp4_grouped_gemm_rows")
        ops._set_last_ws(b["ws"])
        mark("reduce")
        _lib.check(L.fgg_moe_reduce_peers(b["y"].data_ptr(), b["R"], b["route_row"].data_ptr(), toks,
                                          peers, self.bad.data_ptr(), stream), "fgg_moe_reduce_peers")
        mark("combine")
        _lib.check(L.fgg_moe_wait_peers(peers, 1, stream), "fgg_moe_wait_peers")
        mark("sum")
        out = torch.empty((T, n), dtype=torch.bfloat16, device=dev)
        _lib.check(L.fgg_moe_sum_peers(peers, T, out.data_ptr(), stream), "fgg_moe_sum_peers")
        mark("end")
        return out

    def capture(self, x_codes: torch.Tensor, x_sf: torch.Tensor, x_scale, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor | None = None, warmup: int = 2):
        """Capture forward() on these input tensors into a CUDA graph and return
        (replay, out): replay() re-runs the whole layer -- every kernel and both
        collectives -- from one graph launch, reading whatever the input tensors
        hold at that moment, and leaves the result in `out` (the same tensor on
        every replay).  The host then issues one launch per forward instead of
        a dozen kernels and two collectives, so the device never waits for it.
        The warm-up forwards (outside the capture) set up the buffers and the
        collectives' communicators first."""
        if self.gemm_fn is not None:
            raise ValueError("capture needs the device path")
        for _ in range(warmup):
            self.forward(x_codes, x_sf, x_scale, topk_ids, topk_weights)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                out = self.forward(x_codes, x_sf, x_scale, topk_ids, topk_weights)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self._graph = g  # released with the layer (before any process-group teardown)
        return g.replay, out

    def release(self) -> None:
        """Drop a captured graph (it holds the collectives' captured work) and,
        for the peer transport, unmap the other ranks' buffers and free this
        rank's (collective: every rank calls it).  Call before destroying the
        process group."""
        self._graph = None
        if not (self._peer_own or self._peer_mapped):
            return
        import torch.distributed as dist

        L = _lib.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._peer_mapped:
                _lib.check(L.fgg_peer_close(p), "fgg_peer_close")
            self._peer_mapped = []
            if self.world > 1:
                dist.barrier(group=self.group)   # nobody maps a buffer that is freed below
            for p in self._peer_own:
                _lib.check(L.fgg_peer_free(p), "fgg_peer_free")
            self._peer_own = []
        self.bufs = None

    # ------------------------------------------------ host emulation (tests)
    def _forward_host(self, x_u8, s_u8, x_scale, topk_ids, topk_weights):
        """The same steps with torch CPU ops and the stand-in GEMM: records
        padded to the capacity, all-gathered, expanded per local expert (and
        per source, whose decode scale goes into that chunk's alpha), the
        router-weighted partial rows, the equal-split all-to-all, the fp32 sum."""
        import torch.distributed as dist

        T, topk = int(topk_ids.shape[0]), int(topk_ids.shape[1])
        if self.max_tokens is None:
            self.max_tokens = T
        C, W, E, n = self.max_tokens, self.world, self.local, self.n
        if T > C:
            raise ValueError(f"{T} tokens exceed the layer's dispatch capacity max_tokens={C}")
        ids = torch.full((C, topk), -1, dtype=torch.int32)
        ids[:T] = topk_ids.to(torch.int32)
        w = torch.zeros((C, topk), dtype=torch.float32)
        w[:T] = 1.0 if topk_weights is None else topk_weights.to(torch.float32)
        codes = torch.zeros((C, x_u8.shape[1]), dtype=torch.uint8)
        codes[:T] = x_u8
        sf = torch.zeros((C, s_u8.shape[1]), dtype=torch.uint8)
        sf[:T] = s_u8
        xs = torch.as_tensor(x_scale, dtype=torch.float32).reshape(1)
        if W > 1:
            def gather(t):
                out = torch.empty((W * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype)
                dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
                return out
            ids, w, codes, sf, scales = gather(ids), gather(w), gather(codes), gather(sf), gather(xs)
        else:
            scales = xs
        NT = ids.shape[0]
        owner = torch.from_numpy(self.owner_np.astype(np.int64))
        slot = torch.from_numpy(self.slot_np.astype(np.int64))
        flat = ids.reshape(-1).long()
        present = flat >= 0
        if bool((flat >= self.num_experts).any()):
            raise ValueError("an expert id is out of range")
        safe = flat.clamp_min(0)
        local = present & (owner[safe] == self.rank)
        route_idx = torch.nonzero(local).flatten()               # routes of local experts
        tok = route_idx // topk
        src = tok // C
        key = slot[safe[route_idx]] * W + src                    # chunk (expert, source)
        order = torch.argsort(key, stable=True)
        route_idx, tok, src, key = route_idx[order], tok[order], src[order], key[order]
        ms = torch.bincount(key, minlength=E * W).tolist()
        a_list = list(codes[tok].split(ms))
        sf_list = [s.view(torch.float8_e4m3fn) for s in sf[tok].split(ms)]
        b_index = [g // W for g in range(E * W)]
        alpha = (self.w_scale.cpu()[:, None] * scales[None, :]).reshape(-1)
        y = torch.empty((route_idx.numel(), n), dtype=torch.bfloat16)
        self.gemm_fn(a_list, sf_list, b_index, alpha, y)
        route_row = torch.full((NT * topk,), -1, dtype=torch.long)
        route_row[route_idx] = torch.arange(route_idx.numel())
        partial = torch.zeros((NT, n), dtype=torch.float32)
        rr = route_row.view(NT, topk)
        for k in range(topk):
            sel = torch.nonzero(rr[:, k] >= 0).flatten()
            partial[sel] += w[sel, k][:, None] * y[rr[sel, k]].float()
        partial = partial.to(torch.bfloat16)
        if W == 1:
            return partial[:T]
        recv = torch.empty_like(partial)
        self._a2a(recv, partial)
        return recv.view(W, C, n).float().sum(0)[:T].to(torch.bfloat16)

    def check(self) -> None:
        """Raise if a plan, expand or combine kernel met a bad expert id or
        index, or a bounded wait in the GEMM gave up (synchronises the device)."""
        if self.bufs is not None and "pstate" in self.bufs:
            # pstate bytes 20-23 (the high half of word 2) hold the status
            st = int(self.bufs["pstate"][2].item() >> 32) & 0xFFFFFFFF
            if st != 0:
                raise _lib.FggError(_lib.FGG_ETIMEOUT, "ExpertParallelMoE",
                                    f"a peer exchange wait gave up (status 0x{st:x})")
        if self.bad is not None:
            v = int(self.bad.item())
            if v != 0:
                raise _lib.FggError(_lib.FGG_EINVAL, "ExpertParallelMoE",
                                    "an expert id was out of range" if v == 1 else
                                    "more local routes than the expanded buffer holds")
        if self.bufs is not None:
            L = _lib.lib()
            _lib.check(L.fgg_read_device_status(self.bufs["ws"].data_ptr(),
                                                torch.cuda.current_stream(self.device).cuda_stream),
                       "grouped GEMM status")
