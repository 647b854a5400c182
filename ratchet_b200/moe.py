"""Expert-parallel NVFP4 MoE layer: route -> dispatch -> grouped GEMM -> combine.

The single-GPU analogue in the reference is `_moe_forward`
(tasks/muse_prefill_boundary/reference/submission.py:843-895): a gather plan
puts the routed token rows of each expert together, one grouped GEMM runs
every expert, and a combine weights the rows and sums them back per token.
Here the experts are sharded over the ranks of a process group (one process
per GPU) and the rows travel between ranks:

  1. plan      every (token, k) route gets its owner rank and the expert's
               slot on that rank; routes are ordered by (rank, slot) with one
               stable sort, and counted per (rank, slot)
  2. dispatch  all-to-all of the counts (with each rank's activation decode
               scale), then of the NVFP4 rows (codes and E4M3 scales) in that
               order
  3. GEMM      the received rows are source-major: the rows of one local
               expert arrive as one contiguous chunk per source rank.  Each
               (source, expert) chunk is one problem group of the grouped
               GEMM, pointing at the expert's packed weights through b_index,
               so nothing is permuted on the receiving side
  4. combine   all-to-all of the bf16 output rows back along the same splits,
               an index_copy_ that undoes the plan's order, and (with router
               weights) the weighted sum over each token's k routes

Collectives go through torch.distributed (NCCL on GPUs, gloo for the CPU
tests of this host logic).  The expert compute is the library's tcgen05
grouped GEMM; `gemm_fn` may replace it only to test the host logic without
a GPU.
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


class ExpertParallelMoE:
    """One expert-parallel MoE projection (e.g. the fused gate+up of every
    expert) over the ranks of `group`.

    w_codes / w_sf / w_scale: this rank's experts, in slot order: codes
    [N, K/2] uint8, E4M3 scales [N, K/16], fp32 decode scale (0-dim tensor
    or float).  owner / slot: the placement of every expert (place_experts).
    """

    def __init__(self, w_codes: Sequence[torch.Tensor], w_sf: Sequence[torch.Tensor],
                 w_scale: Sequence, owner: np.ndarray, slot: np.ndarray, group=None,
                 gemm_fn: GemmFn | None = None):
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
                                    for s in w_scale])
        self.owner_t = torch.from_numpy(owner).to(dev, torch.int64)
        self.slot_t = torch.from_numpy(slot).to(dev, torch.int64)
        self.gemm_fn = gemm_fn
        self.pack = None
        self.bad = None
        self.ws = None
        self._host_counts = None  # pinned landing buffer of the per-forward count exchange
        if gemm_fn is None:
            # the product path: weights packed once and reused by every
            # forward; the gather / combine kernels raise this flag on an
            # out-of-range row index (see check())
            self.pack = ops.pack_weights(self.w_codes, self.w_sf)
            self.bad = torch.zeros(1, dtype=torch.int32, device=dev)
            self.owner_i32 = torch.from_numpy(owner).to(dev)
            self.slot_i32 = torch.from_numpy(slot).to(dev)
            self.ws = torch.empty(0, dtype=torch.uint8, device=dev)  # GEMM workspace, grown on demand
        # problem group g = (source rank, local slot), source-major
        self.b_index = [e for _ in range(self.world) for e in range(self.local)]
        self.b_index_np = np.asarray(self.b_index, dtype=np.int32)

    # -------------------------------------------------------------- pieces
    def plan(self, topk_ids: torch.Tensor):
        """Order of the routes by (owner rank, slot) and their counts."""
        flat = topk_ids.reshape(-1).to(self.owner_t.device, torch.int64)
        key = self.owner_t[flat] * self.local + self.slot_t[flat]
        order = torch.argsort(key, stable=True)
        counts = torch.bincount(key, minlength=self.world * self.local).to(torch.int32)
        return order, counts

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        import torch.distributed as dist

        if inp.dtype == torch.bfloat16:  # rows as bytes: bit-exact on every backend
            out, inp = out.view(torch.uint8), inp.view(torch.uint8)
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x_codes: torch.Tensor, x_sf: torch.Tensor, x_scale, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor | None = None, gemm_events=None) -> torch.Tensor:
        """x_codes [T, K/2] uint8 and x_sf [T, K/16] E4M3: this rank's tokens,
        quantised with decode scale x_scale.  topk_ids [T, k] expert ids.
        Returns [T, k, N] bf16 per-route outputs, or [T, N] bf16 (the
        weighted sum over k) when topk_weights [T, k] is given.
        gemm_events: optional (start, end) CUDA events recorded around the
        grouped GEMM on the current stream (for timing the kernel alone)."""
        T, topk = int(topk_ids.shape[0]), int(topk_ids.shape[1])
        kh, ks = self.k // 2, self.k // 16
        x_u8 = x_codes.view(torch.uint8)
        s_u8 = x_sf.view(torch.uint8)
        if x_u8.shape != (T, kh) or s_u8.shape != (T, ks):
            raise ValueError(f"x_codes {tuple(x_u8.shape)} / x_sf {tuple(s_u8.shape)} do not match "
                             f"T={T}, K={self.k}")
        dev = x_u8.device
        W, E = self.world, self.local
        S = T * topk
        L = _lib.lib() if self.gemm_fn is None else None
        stream = ops._stream_ptr(dev) if L is not None else None
        # 1. plan
        if L is not None:
            ids32 = topk_ids.to(dev, torch.int32).contiguous()
            counts = torch.empty(W * E, dtype=torch.int32, device=dev)
            src_row = torch.empty(S, dtype=torch.int32, device=dev)
            route_pos = torch.empty(S, dtype=torch.int32, device=dev)
            _lib.check(L.fgg_moe_plan(ids32.data_ptr(), T, topk, self.owner_i32.data_ptr(),
                                      self.slot_i32.data_ptr(), self.num_experts, W, E,
                                      counts.data_ptr(), src_row.data_ptr(), route_pos.data_ptr(),
                                      self.bad.data_ptr(), stream), "fgg_moe_plan")
        else:  # host-logic tests without a GPU
            order, counts = self.plan(topk_ids)
        # 2. to every rank: the counts of the routes it gets from here and
        #    this rank's activation decode scale (its bits after the counts)
        xs = torch.as_tensor(x_scale, dtype=torch.float32, device=dev).reshape(1)
        info = torch.empty((W, E + 1), dtype=torch.int32, device=dev)
        info[:, :E] = counts.view(W, E)
        info[:, E] = xs.view(torch.int32)
        if W == 1:
            recv_info = info
        else:
            recv_info = torch.empty_like(info)
            self._a2a(recv_info, info)
        # the counts travel to the host ahead of the row gather: the host waits
        # for this copy alone (one host sync per forward) and plans the GEMM
        # while the device still gathers
        both_d = torch.stack([info, recv_info])
        counts_ready = None
        if both_d.is_cuda:
            if self._host_counts is None or self._host_counts.shape != both_d.shape:
                self._host_counts = torch.empty(both_d.shape, dtype=torch.int32, pin_memory=True)
            both = self._host_counts
            both.copy_(both_d, non_blocking=True)
            counts_ready = torch.cuda.Event()
            counts_ready.record()
        else:
            both = both_d
        # 3. the rows in (owner, slot) order
        if L is not None:
            send_codes = torch.empty((S, kh), dtype=torch.uint8, device=dev)
            send_sf = torch.empty((S, ks), dtype=torch.uint8, device=dev)
            _lib.check(L.fgg_moe_gather_rows(
                x_u8.data_ptr(), s_u8.data_ptr(), T, kh, ks, src_row.data_ptr(), S,
                send_codes.data_ptr(), send_sf.data_ptr(), self.bad.data_ptr(), stream),
                "fgg_moe_gather_rows")
        else:
            rows = order // topk
            send_codes = x_u8.index_select(0, rows)
            send_sf = s_u8.index_select(0, rows)
        # alpha of problem group (source, slot) = source's activation scale x
        # the slot's weight scale: device work, queued before the host waits
        src_scale = recv_info[:, E].contiguous().view(torch.float32)
        alpha = (src_scale[:, None] * self.w_scale[None, :]).reshape(-1).contiguous()
        # on one rank every route stays: the GEMM output size is known up front
        out = torch.empty((S, self.n), dtype=torch.bfloat16, device=dev) if W == 1 else None
        if counts_ready is not None:
            counts_ready.synchronize()
        send_ce, recv_ce = both[0, :, :E], both[1, :, :E]
        send_splits = send_ce.sum(1).tolist()
        recv_splits = recv_ce.sum(1).tolist()
        R = int(sum(recv_splits))
        if W == 1:  # nothing leaves the rank
            recv_codes, recv_sf = send_codes, send_sf
        else:
            recv_codes = torch.empty((R, kh), dtype=torch.uint8, device=dev)
            recv_sf = torch.empty((R, ks), dtype=torch.uint8, device=dev)
            self._a2a(recv_codes, send_codes, recv_splits, send_splits)
            self._a2a(recv_sf, send_sf, recv_splits, send_splits)
        # 4. grouped GEMM over the (source, slot) chunks
        if out is None:
            out = torch.empty((R, self.n), dtype=torch.bfloat16, device=dev)
        if gemm_events is not None:
            gemm_events[0].record()
        if L is not None:
            if R > 0:
                self._gemm(L, recv_ce, recv_codes, recv_sf, alpha, out, stream)
        else:
            ms = recv_ce.reshape(-1).tolist()
            a_list = list(recv_codes.split(ms))
            sf_list = [t.view(torch.float8_e4m3fn) for t in recv_sf.split(ms)]
            self.gemm_fn(a_list, sf_list, self.b_index, alpha, out)
        if gemm_events is not None:
            gemm_events[1].record()
        # 5. combine: rows go back along the dispatch splits, then to route order
        if W == 1:
            back = out
        else:
            back = torch.empty((T * topk, self.n), dtype=torch.bfloat16, device=dev)
            self._a2a(back, out, send_splits, recv_splits)
        if L is not None:
            if topk_weights is None:
                return back.index_select(0, route_pos.long()).view(T, topk, self.n)
            # one pass: each token reads its k rows where the dispatch order
            # left them and writes the weighted sum
            w = topk_weights.to(dev, torch.float32).contiguous()
            res = torch.empty((T, self.n), dtype=torch.bfloat16, device=dev)
            _lib.check(L.fgg_moe_combine(back.data_ptr(), S, route_pos.data_ptr(), w.data_ptr(), T,
                                         topk, self.n, res.data_ptr(), self.bad.data_ptr(),
                                         stream), "fgg_moe_combine")
            return res
        res = torch.empty_like(back)
        res.index_copy_(0, order, back)
        res = res.view(T, topk, self.n)
        if topk_weights is None:
            return res
        w = topk_weights.to(dev, torch.float32).view(T, topk, 1)
        return (res.float() * w).sum(1).to(torch.bfloat16)

    def _gemm(self, L, recv_ce, recv_codes, recv_sf, alpha, out, stream):
        """The grouped GEMM through the C ABI directly: the group pointers are
        offsets into the two receive buffers, so no per-group tensor views."""
        kh, ks = self.k // 2, self.k // 16
        ms = recv_ce.reshape(-1).numpy().astype(np.int32)
        offs = np.zeros_like(ms, dtype=np.uint64)
        offs[1:] = np.cumsum(ms[:-1], dtype=np.uint64)
        a_ptrs = np.uint64(recv_codes.data_ptr()) + offs * np.uint64(kh)
        sf_ptrs = np.uint64(recv_sf.data_ptr()) + offs * np.uint64(ks)
        prob = _lib.FggNvfp4Problem(len(ms), self.n, self.k, ms.ctypes.data, a_ptrs.ctypes.data,
                                    sf_ptrs.ctypes.data, alpha.data_ptr(), out.data_ptr(),
                                    self.b_index_np.ctypes.data, self.local)
        nbytes = int(L.fgg_nvfp4_workspace_bytes(prob))
        if nbytes == 0:
            _lib.check(L.fgg_nvfp4_grouped_gemm(prob, None, None, 0, None), "grouped GEMM")
        if self.ws.numel() < nbytes:
            self.ws = torch.empty(nbytes, dtype=torch.uint8, device=out.device)
        _lib.check(L.fgg_nvfp4_grouped_gemm(prob, self.pack.buf.data_ptr(), self.ws.data_ptr(),
                                            self.ws.numel(), stream), "grouped GEMM")

    def check(self) -> None:
        """Raise if a plan, gather or combine kernel met an out-of-range index,
        or a bounded wait in the GEMM gave up (synchronises the device)."""
        if self.bad is not None and int(self.bad.item()) != 0:
            raise _lib.FggError(_lib.FGG_EINVAL, "ExpertParallelMoE",
                                "an expert id or a dispatch / combine row index was out of range")
        if self.ws is not None and self.ws.numel():
            L = _lib.lib()
            _lib.check(L.fgg_read_device_status(self.ws.data_ptr(),
                                                torch.cuda.current_stream(self.device).cuda_stream),
                       "grouped GEMM status")
