"""Peer gather of kv-head-sharded decode (molot_comm_* and
molot_paged_decode_gather): each rank's paged decode writes its heads'
outputs into every rank's gathered buffer over NVLink, its last CTA raises
its epoch flag there, and molot_comm_wait waits for every rank's flag.

With one rank the gather is the identity: the gathered buffer must equal
molot_paged_decode's output bit for bit.  With two GPUs (skipped on fewer)
two processes each decode half the kv heads and both gathered buffers must
equal the oracle's full [B][nq][d].  The reference has no multi-device path;
its per-head independence (attn.h:125-177 computes every q head from its
own kv head only) is what makes head sharding exact."""
import os
import sys
import time

import numpy as np
import pytest

from conftest import PARITY_TOL, ROOT
from test_paged_gpu import make_pool, oracle_parallel

pytestmark = pytest.mark.gpu


def test_one_rank_gather_is_identity(mb, torch_cuda, orc):
    torch = torch_cuda
    lens = [4097, 333, 16385, 17]
    nq, nkv, d, ps = 16, 2, 128, 16
    B = len(lens)
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=61)
    Q = np.random.default_rng(62).standard_normal((B, nq, d)).astype(np.float32)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    dQ, dK, dV, dbt = cu(Q), cu(Kp), cu(Vp), cu(bt)
    layers = 3
    per = B * nq * d
    comm = mb.Comm(1, 0, 4 * layers * per)
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, None, 0)
        ref = torch.empty((B, nq, d), device="cuda")
        plan.decode(dQ, ref, dK, dV, dbt, ps, d ** -0.5)
        buf = comm.buffer((layers, B, nq, d))
        buf.fill_(float("nan"))
        for layer in range(layers):  # epochs advance with every pair
            plan.decode_gather(comm, dQ, layer * per, dK, dV, dbt, ps, d ** -0.5)
            comm.wait()
        comm.check()
        plan.check()
        got = buf.cpu().numpy()
        want_dev = ref.cpu().numpy()
    finally:
        plan.close()
        comm.close()
    for layer in range(layers):
        assert np.array_equal(got[layer], want_dev), layer
    want = orc.attn_decode_paged(Q, Kp, Vp, bt, lens, None, B, nq, nkv, d, ps, d ** -0.5, 0)
    assert orc.rel_err(got[0], want) <= PARITY_TOL


def test_gather_rejects_bad_offsets(mb, torch_cuda):
    torch = torch_cuda
    lens = [100, 40]
    nq, nkv, d, ps = 8, 2, 64, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=3)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    comm = mb.Comm(1, 0, 4 * len(lens) * nq * d)
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, None, 0)
        Q = torch.zeros((2, nq, d), device="cuda")
        with pytest.raises(mb.MolotError) as ei:  # one float past the end
            plan.decode_gather(comm, Q, 4, cu(Kp), cu(Vp), cu(bt), ps, 1.0)
        assert ei.value.status == mb.ERR_INVALID
        plan.build(nq, nkv, d, [100, 0], None, 0)  # a sequence attending nothing
        with pytest.raises(mb.MolotError):
            plan.decode_gather(comm, Q, 0, cu(Kp), cu(Vp), cu(bt), ps, 1.0)
    finally:
        plan.close()
        comm.close()


def test_wait_without_peer_runs_out(mb, torch_cuda):
    """A wait whose flag nothing raises (no decode_gather before it) gives up
    after its bound, records the timeout for molot_comm_check and leaves the
    GPU usable."""
    torch = torch_cuda
    comm = mb.Comm(1, 0, 1024)
    try:
        t0 = time.time()
        comm.wait()
        with pytest.raises(mb.MolotError) as ei:
            comm.check()
        assert ei.value.status == mb.ERR_TIMEOUT
        assert time.time() - t0 < 30
        comm.check()  # reported once, then cleared
    finally:
        comm.close()
    x = torch.ones(16, device="cuda")
    assert float(x.sum()) == 16.0


def _rank_main(rank, world, handles_q, open_q, result_q, case):
    """One rank of the two-GPU test (a spawned process)."""
    sys.path.insert(0, ROOT)
    import torch

    import molot_b200 as mb
    torch.cuda.set_device(rank)
    lens, nq, nkv, d, ps, seed = (case[k] for k in ("lens", "nq", "nkv", "d", "ps", "seed"))
    B = len(lens)
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=seed)
    Q = np.random.default_rng(seed + 1).standard_normal((B, nq, d)).astype(np.float32)
    nkv_l, nq_l = nkv // world, nq // world
    g0 = rank * nkv_l
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    dK = cu(Kp[:, g0:g0 + nkv_l])
    dV = cu(Vp[:, g0:g0 + nkv_l])
    dQ = cu(Q[:, rank * nq_l:(rank + 1) * nq_l])
    comm = mb.Comm(world, rank, 4 * B * nq * d)
    handles_q.put((rank, comm.ipc_handle()))
    handles = open_q.get(timeout=120)
    comm.open(handles)
    plan = mb.PagedPlan()
    plan.build(nq_l, nkv_l, d, lens, None, 0)
    buf = comm.buffer((B, nq, d))
    for _ in range(3):
        plan.decode_gather(comm, dQ, 0, dK, dV, cu(bt), ps, d ** -0.5)
        comm.wait()
    comm.check()
    plan.check()
    result_q.put((rank, buf.cpu().numpy()))
    torch.cuda.synchronize()
    # every rank has read its buffer before any rank unmaps or frees it
    open_q.get(timeout=120)
    plan.close()
    comm.close()


def test_two_gpu_head_sharded_gather(mb, torch_cuda, orc):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    case = dict(lens=[20001, 4097, 131, 9000], nq=16, nkv=2, d=128, ps=16, seed=71)
    world = 2
    ctx = mp.get_context("spawn")
    handles_q, result_q = ctx.Queue(), ctx.Queue()
    open_qs = [ctx.Queue() for _ in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, handles_q, open_qs[r], result_q, case))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        hs = dict(handles_q.get(timeout=300) for _ in range(world))
        for q in open_qs:
            q.put([hs[r] for r in range(world)])
        outs = dict(result_q.get(timeout=300) for _ in range(world))
        for q in open_qs:
            q.put(None)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    lens, nq, nkv, d, ps = (case[k] for k in ("lens", "nq", "nkv", "d", "ps"))
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=case["seed"])
    Q = np.random.default_rng(case["seed"] + 1).standard_normal(
        (len(lens), nq, d)).astype(np.float32)
    want = oracle_parallel(orc, Q, Kp, Vp, bt, lens, nq, nkv, d, ps, d ** -0.5, 0)
    assert np.array_equal(outs[0], outs[1])
    for b in range(len(lens)):
        assert orc.rel_err(outs[0][b], want[b]) <= PARITY_TOL, b
