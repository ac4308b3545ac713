"""Multi-rank partitioning of batched decode, on the CPU: world_size-2 gloo
process groups, the oracle standing in for each rank's kernel.

* sequence sharding: LPT split, per-rank attention of its own sequences,
  reassembly equals the single-process batch;
* kv-head sharding: per-rank attention over its kv heads' slice of the pool,
  gather_heads equals the single-process batch.
"""
import math
import os
import socket

import numpy as np
import pytest

from conftest import ROOT

B, NQ, NKV, D, PS = 5, 8, 4, 64, 16
LENS = [40, 17, 70, 33, 1]
SCALE = 0.125


def make_case():
    rng = np.random.default_rng(11)
    need = [max(1, math.ceil(n / PS)) for n in LENS]
    total = sum(need) + 2
    perm = rng.permutation(total)
    bt = np.zeros((B, max(need)), np.int32)
    k = 0
    for b, m in enumerate(need):
        bt[b, :m] = perm[k:k + m]
        k += m
    Kp = rng.standard_normal((total, NKV, PS, D)).astype(np.float32)
    Vp = rng.standard_normal((total, NKV, PS, D)).astype(np.float32)
    Q = rng.standard_normal((B, NQ, D)).astype(np.float32)
    return Q, Kp, Vp, bt


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    import oracle
    from molot_b200 import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        Q, Kp, Vp, bt = make_case()
        if mode == "seq":
            mine = shard.lpt_partition(LENS, world)[rank]
            o = oracle.attn_decode_paged(Q[mine], Kp, Vp, bt[mine], [LENS[i] for i in mine],
                                         None, len(mine), NQ, NKV, D, PS, SCALE, 0)
            got = [None] * world
            dist.all_gather_object(got, (mine, o))
            full = np.full((B, NQ, D), np.nan, np.float32)
            for idx, part in got:
                full[idx] = part
        else:
            g0, g1 = shard.head_shard(NKV, world, rank)
            G = NQ // NKV
            ql = np.ascontiguousarray(Q[:, g0 * G:g1 * G])
            kl = np.ascontiguousarray(Kp[:, g0:g1])
            vl = np.ascontiguousarray(Vp[:, g0:g1])
            o = oracle.attn_decode_paged(ql, kl, vl, bt, LENS, None, B, (g1 - g0) * G, g1 - g0,
                                         D, PS, SCALE, 0)
            full = shard.gather_heads(torch.from_numpy(o)).numpy()
        np.save(os.path.join(out_dir, f"{mode}_{rank}.npy"), full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["seq", "head"])
def test_two_rank_sharding_matches_single_process(mode, tmp_path):
    import torch.multiprocessing as tmp
    import oracle
    tmp.start_processes(_worker, args=(2, free_port(), mode, str(tmp_path)), nprocs=2,
                        join=True, start_method="spawn")
    Q, Kp, Vp, bt = make_case()
    want = oracle.attn_decode_paged(Q, Kp, Vp, bt, LENS, None, B, NQ, NKV, D, PS, SCALE, 0)
    for r in range(2):
        got = np.load(tmp_path / f"{mode}_{r}.npy")
        # the same per-sequence / per-head arithmetic in every layout
        assert np.array_equal(got.view(np.int32), want.view(np.int32)), (mode, r)


def test_lpt_partition_balance_and_cover():
    from molot_b200 import shard
    rng = np.random.default_rng(3)
    lens = rng.integers(512, 32769, size=64)
    for world in (1, 2, 4, 8):
        parts = shard.lpt_partition(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [int(lens[p].sum()) for p in parts]
        # LPT bound: max load <= (4/3 - 1/(3w)) * optimum <= that of the mean
        assert max(loads) <= (4 / 3) * (lens.sum() / world) + lens.max()
        assert max(loads) - min(loads) <= lens.max()
    assert shard.lpt_partition([5, 5, 5], 2) == [[0, 2], [1]]


def test_head_shard_ranges():
    from molot_b200 import shard
    assert [shard.head_shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        shard.head_shard(8, 3, 0)
