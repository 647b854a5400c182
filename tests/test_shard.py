"""The multi-GPU partitionings of the benchmark configurations, on two gloo
ranks (CPU): config 4 splits the weight rows (output columns) with the
activations replicated, config 5 places whole groups by longest-processing-
time on their weight bytes.  Each rank computes its part with the CPU oracle;
the parts, gathered, must cover the problem exactly once and equal the
whole problem computed on one rank, bit for bit (the same arithmetic per
output column and per group).  The GPU runs the same partitioning through
bench.py under torchrun."""
import os
import socket

import numpy as np
import pytest
import torch

import bench
from oracle import nvfp4 as ref


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


DENSE = dict(name="dense", desc="small dense", m=[96], n=1024, k=256, w_std=1.0, bound="tensor")
DECODE = dict(name="decode", desc="small decode", m=[3, 1, 16, 7, 0, 9, 12, 2, 5, 16, 4, 8, 1],
              n=256, k=512, w_std=0.02, bound="hbm")


def _group_data(g, m, n, k, w_std):
    rng = np.random.default_rng(1000 + g)
    qa, sa, ga = ref.nvfp4_quantize(rng.standard_normal((max(m, 1), k), dtype=np.float32)[:m]) \
        if m else (np.zeros((0, k // 2), np.uint8), np.zeros((0, k // 16), np.uint8), np.float32(1))
    qb, sb, gb = ref.nvfp4_quantize(rng.standard_normal((n, k), dtype=np.float32) * np.float32(w_std))
    return qa, sa, qb, sb, np.float32(ga * gb)


def _dense_part(sub):
    qa, sa, qb, sb, al = _group_data(0, sub["m"][0], DENSE["n"], DENSE["k"], 1.0)
    r0, r1 = sub["w_rows"]
    return ref.grouped_gemm([qa], [sa], [qb[r0:r1]], [sb[r0:r1]], [al])[0]


def _decode_part(sub):
    out = {}
    for g, m in zip(sub["groups"], sub["m"]):
        qa, sa, qb, sb, al = _group_data(g, m, DECODE["n"], DECODE["k"], DECODE["w_std"])
        out[g] = ref.grouped_gemm([qa], [sa], [qb], [sb], [al])[0]
    return out


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ok = True
        msgs = []
        # config 4: column slices
        sub = bench.shard(DENSE, world, rank)
        part = _dense_part(sub)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        whole = _dense_part(bench.shard(DENSE, 1, 0))
        if not torch.equal(torch.cat(parts, dim=1), whole):
            ok = False
            msgs.append("dense: the column slices differ from the whole product")
        # config 5: whole groups, each on exactly one rank
        sub = bench.shard(DECODE, world, rank)
        mine = _decode_part(sub)
        got = [None] * world
        dist.all_gather_object(got, mine)
        seen = sorted(g for d in got for g in d)
        if seen != list(range(len(DECODE["m"]))):
            ok = False
            msgs.append(f"decode: groups covered {seen}")
        full = _decode_part(bench.shard(DECODE, 1, 0))
        for d in got:
            for g, t in d.items():
                if not torch.equal(t, full[g]):
                    ok = False
                    msgs.append(f"decode: group {g} differs")
        sizes = [len(d) for d in got]
        if max(sizes) - min(sizes) > 1:
            ok = False
            msgs.append(f"decode: unbalanced group counts {sizes}")
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{int(ok)} {msgs}\n")
    finally:
        dist.destroy_process_group()


def test_partitionings_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        line = (tmp_path / f"rank{r}.txt").read_text()
        assert line.startswith("1 "), f"rank {r}: {line}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_covers_every_column_and_group(world):
    dense = bench.workload("dense")
    cols = [bench.shard(dense, world, r)["w_rows"] for r in range(world)]
    assert cols[0][0] == 0 and cols[-1][1] == dense["n"]
    assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
    decode = bench.workload("decode")
    groups = sorted(g for r in range(world) for g in bench.shard(decode, world, r)["groups"])
    assert groups == list(range(len(decode["m"])))
