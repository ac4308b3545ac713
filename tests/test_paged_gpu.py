"""GPU parity of the paged, batched decode (continuous batching) and of the
batched append, against per-sequence calls of the oracle on gathered pages."""
import math
import os

import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def make_pool(lens, nkv, d, page_size, seed, spare=5):
    """K/V pools [pages][nkv][page_size][d] and a shuffled block table."""
    rng = np.random.default_rng(seed)
    need = [max(1, math.ceil(n / page_size)) for n in lens]
    total = sum(need) + spare
    perm = rng.permutation(total)
    max_pages = max(need)
    bt = np.zeros((len(lens), max_pages), np.int32)
    k = 0
    for b, m in enumerate(need):
        bt[b, :m] = perm[k:k + m]
        k += m
    Kp = rng.standard_normal((total, nkv, page_size, d)).astype(np.float32)
    Vp = rng.standard_normal((total, nkv, page_size, d)).astype(np.float32)
    return Kp, Vp, bt


def run_paged(mb, torch, Q, Kp, Vp, bt, lens, positions, nq, nkv, d, page_size, scale, window):
    B = len(lens)
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, positions, window)
        dO = torch.full((B, nq, d), float("nan"), device="cuda")
        plan.decode(torch.from_numpy(Q).cuda(), dO, torch.from_numpy(Kp).cuda(),
                    torch.from_numpy(Vp).cuda(), torch.from_numpy(bt).cuda(), page_size, scale)
        plan.check()
        return dO.cpu().numpy()
    finally:
        plan.close()


def check_against_oracle(orc, got, Q, Kp, Vp, bt, lens, positions, nq, nkv, d, page_size, scale,
                         window):
    B = len(lens)
    want = orc.attn_decode_paged(Q, Kp, Vp, bt, lens, positions, B, nq, nkv, d, page_size, scale,
                                 window)
    for b in range(B):
        n = lens[b]
        pos = positions[b] if positions is not None else n - 1
        t0 = pos - window + 1 if window > 0 and pos - window + 1 > 0 else 0
        if n <= t0:
            assert not np.any(got[b]), b
            assert not np.any(want[b]), b
        else:
            assert orc.rel_err(got[b], want[b]) <= PARITY_TOL, (b, n)


@pytest.mark.parametrize("case", [
    dict(lens=[1, 15, 16, 17, 100, 1000, 3333, 0], nq=32, nkv=8, d=128, ps=16, window=0),
    dict(lens=[4097, 2, 700, 16385], nq=32, nkv=8, d=128, ps=16, window=0),
    dict(lens=[5000, 1200, 77, 3000, 1], nq=8, nkv=4, d=256, ps=16, window=1024),
    dict(lens=[900, 129, 4000], nq=8, nkv=1, d=128, ps=32, window=0),
    dict(lens=[300, 64, 65, 1023], nq=16, nkv=2, d=64, ps=16, window=50),
], ids=["ragged_llama", "long_mixed", "gemma_swa", "g8_ps32", "d64_window"])
def test_paged_ragged(mb, torch_cuda, orc, case):
    lens = case["lens"]
    nq, nkv, d, ps, window = case["nq"], case["nkv"], case["d"], case["ps"], case["window"]
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=sum(lens))
    rng = np.random.default_rng(len(lens))
    Q = rng.standard_normal((len(lens), nq, d)).astype(np.float32)
    scale = d ** -0.5
    got = run_paged(mb, torch_cuda, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, scale, window)
    check_against_oracle(orc, got, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, scale, window)


def test_paged_batch64_llama8b(mb, torch_cuda, orc):
    """cfg4 shape (Llama-3-8B heads, 16-token pages, shuffled block table),
    batch 64 with lengths drawn from [512, 4096] to keep the oracle quick."""
    rng = np.random.default_rng(4)
    lens = [int(x) for x in rng.integers(512, 4097, size=64)]
    nq, nkv, d, ps = 32, 8, 128, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=44)
    Q = rng.standard_normal((64, nq, d)).astype(np.float32)
    got = run_paged(mb, torch_cuda, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, d ** -0.5, 0)
    check_against_oracle(orc, got, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, d ** -0.5, 0)


def oracle_parallel(orc, Q, Kp, Vp, bt, lens, nq, nkv, d, ps, scale, window):
    """The oracle per sequence, sequences on threads (the C checker releases
    the GIL), for the long-context cases."""
    from concurrent.futures import ThreadPoolExecutor

    def one(b):
        return orc.attn_decode_paged(Q[b:b + 1], Kp, Vp, bt[b:b + 1], [lens[b]], None, 1, nq,
                                     nkv, d, ps, scale, window)[0]

    with ThreadPoolExecutor(max_workers=min(len(lens), os.cpu_count() or 1)) as ex:
        return np.stack(list(ex.map(one, range(len(lens)))))


def test_paged_cfg4_full_lengths(mb, torch_cuda, orc):
    """cfg4 as configured: lengths from its own seeded U[512, 32768] draw
    (the bench's draw, always including its longest sequence), Llama-3-8B
    heads, 16-slot pages, a shuffled block table; 8 of its 64 sequences."""
    rng = np.random.default_rng(4)
    draw = [int(x) for x in rng.integers(512, 32769, size=64)]
    longest = int(np.argmax(draw))
    pick = [longest] + [i for i in range(64) if i != longest][:7]
    lens = [draw[i] + 1 for i in pick]  # cached slots + the new token's
    nq, nkv, d, ps = 32, 8, 128, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=404)
    Q = np.random.default_rng(405).standard_normal((len(lens), nq, d)).astype(np.float32)
    got = run_paged(mb, torch_cuda, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, d ** -0.5, 0)
    want = oracle_parallel(orc, Q, Kp, Vp, bt, lens, nq, nkv, d, ps, d ** -0.5, 0)
    for b in range(len(lens)):
        assert orc.rel_err(got[b], want[b]) <= PARITY_TOL, (b, lens[b])


def test_paged_cfg5_one_rank(mb, torch_cuda, orc):
    """cfg5 as one of 8 ranks sees it: one kv head and its 8 query heads
    (G = 8), 16-slot pages, sequences of ~131k, ~40k and 8k slots plus a
    short one.  The stream-K partition spreads the 131k-slot segment over
    ~100 CTAs, so its combine merges many partials in several batches."""
    lens = [131073, 40001, 8193, 37]
    nq, nkv, d, ps = 8, 1, 128, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=505)
    Q = np.random.default_rng(506).standard_normal((len(lens), nq, d)).astype(np.float32)
    got = run_paged(mb, torch_cuda, Q, Kp, Vp, bt, lens, None, nq, nkv, d, ps, d ** -0.5, 0)
    want = oracle_parallel(orc, Q, Kp, Vp, bt, lens, nq, nkv, d, ps, d ** -0.5, 0)
    for b in range(len(lens)):
        assert orc.rel_err(got[b], want[b]) <= PARITY_TOL, (b, lens[b])


def test_paged_explicit_positions(mb, torch_cuda, orc):
    lens = [500, 800, 120]
    positions = [499, 650, 300]  # window start taken from pos, attention ends at n
    nq, nkv, d, ps = 8, 2, 128, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=8)
    Q = np.random.default_rng(3).standard_normal((3, nq, d)).astype(np.float32)
    got = run_paged(mb, torch_cuda, Q, Kp, Vp, bt, lens, positions, nq, nkv, d, ps, 0.1, 200)
    check_against_oracle(orc, got, Q, Kp, Vp, bt, lens, positions, nq, nkv, d, ps, 0.1, 200)


def test_paged_plan_reuse_across_layers(mb, torch_cuda, orc):
    """One plan serves every layer of a step (the bench pattern)."""
    torch = torch_cuda
    lens = [1000, 37, 2500]
    nq, nkv, d, ps = 32, 8, 128, 16
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, None, 0)
        for layer in range(3):
            Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=100 + layer)
            Q = np.random.default_rng(layer).standard_normal((3, nq, d)).astype(np.float32)
            dO = torch.empty((3, nq, d), device="cuda")
            plan.decode(torch.from_numpy(Q).cuda(), dO, torch.from_numpy(Kp).cuda(),
                        torch.from_numpy(Vp).cuda(), torch.from_numpy(bt).cuda(), ps, 0.088)
            plan.check()
            check_against_oracle(orc, dO.cpu().numpy(), Q, Kp, Vp, bt, lens, None, nq, nkv, d,
                                 ps, 0.088, 0)
    finally:
        plan.close()


def test_paged_append_then_decode(mb, torch_cuda, orc):
    """molot_paged_append writes each sequence's new k/v at slot n-1 of its
    pages (QK-norm, V-norm, RoPE as forward.h:554-575), then decode reads them."""
    torch = torch_cuda
    lens = [33, 16, 1, 400]
    nq, nkv, d, ps = 8, 4, 256, 16
    B = len(lens)
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=77)
    rng = np.random.default_rng(78)
    q = rng.standard_normal((B, nq * d)).astype(np.float32)
    k = rng.standard_normal((B, nkv * d)).astype(np.float32)
    v = rng.standard_normal((B, nkv * d)).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    freq = orc.rope_inv_freq(1e4, d)
    dK, dV = torch.from_numpy(Kp).cuda(), torch.from_numpy(Vp).cuda()
    dbt = torch.from_numpy(bt).cuda()
    q_rot = torch.empty((B, nq * d), device="cuda")
    dO = torch.empty((B, nq, d), device="cuda")
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, None, 0)
        cu = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        plan.append(cu(q), cu(k), cu(v), q_rot, dK, dV, dbt, ps, cu(qn), cu(kn), True, 1e-6,
                    cu(freq))
        plan.decode(q_rot, dO, dK, dV, dbt, ps, 1.0)
        plan.check()
    finally:
        plan.close()
    # oracle: per sequence, prologue on host then the same pages
    Kp2, Vp2 = Kp.copy(), Vp.copy()
    q_ref = np.zeros_like(q)
    for b in range(B):
        n = lens[b]
        pos = n - 1
        qh = q[b].reshape(nq, d).copy()
        for h in range(nq):
            qh[h] = orc.rope_apply(orc.rmsnorm(qh[h], qn, 1e-6), d, pos, freq)
        q_ref[b] = qh.reshape(-1)
        kh = k[b].reshape(nkv, d)
        vv = orc.rmsnorm_plain(v[b], 1e-6).reshape(nkv, d)
        page, off = bt[b, pos // ps], pos % ps
        for g in range(nkv):
            Kp2[page, g, off] = orc.rope_apply(orc.rmsnorm(kh[g], kn, 1e-6), d, pos, freq)
            Vp2[page, g, off] = vv[g]
    assert orc.rel_err(q_rot.cpu().numpy(), q_ref) < 1e-6
    assert orc.rel_err(dK.cpu().numpy(), Kp2) < 1e-6
    assert orc.rel_err(dV.cpu().numpy(), Vp2) < 1e-6
    want = orc.attn_decode_paged(q_ref.reshape(B, nq, d), Kp2, Vp2, bt, lens, None, B, nq, nkv, d,
                                 ps, 1.0, 0)
    assert orc.rel_err(dO.cpu().numpy(), want) <= PARITY_TOL
