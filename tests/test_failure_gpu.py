"""Failure detection on the GPU, without a fault: every wait of the decode
kernel is bounded; one that runs out records a status code, the launch
stops waiting and exits, and the host reports MOLOT_ERR_TIMEOUT on its next
check.  The test hook molot_debug_withhold_next makes the next launch's
producer issue no copy at all, so the consumers' first wait for a stage runs
out with nothing in flight (the wait is on a barrier that nothing will
complete).  After the report the same handle must serve a normal call with
full parity: the check cleared the status word and the tickets the
abandoned launch left behind."""
import numpy as np
import pytest

from conftest import PARITY_TOL
from test_paged_gpu import make_pool

pytestmark = pytest.mark.gpu

LIMIT_NS = 2_000_000  # 2 ms


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("nq,nkv,d,n", [(32, 8, 128, 16385), (8, 4, 256, 3000)])
def test_kv_handle_wait_runs_out_then_recovers(mb, torch_cuda, orc, nq, nkv, d, n):
    torch = torch_cuda
    rng = np.random.default_rng(n)
    K = rng.standard_normal((n, nkv * d)).astype(np.float32)
    V = rng.standard_normal((n, nkv * d)).astype(np.float32)
    q = rng.standard_normal(nq * d).astype(np.float32)
    kv = mb.KVCache(1, nkv, d, n)
    try:
        kv.write(0, 0, cu(torch, K), cu(torch, V))
        kv.set_length(0, n)
        o = torch.empty(nq * d, device="cuda")
        kv.decode(0, cu(torch, q), o, d ** -0.5, n - 1)  # sizes the workspace
        kv.check()
        mb.debug_withhold_next(LIMIT_NS)
        kv.decode(0, cu(torch, q), o, d ** -0.5, n - 1)
        with pytest.raises(mb.MolotError) as ei:
            kv.check()
        assert ei.value.status == mb.ERR_TIMEOUT
        kv.check()  # reported once, then cleared
        o.fill_(float("nan"))
        kv.decode(0, cu(torch, q), o, d ** -0.5, n - 1)
        kv.check()
        want = orc.attn_decode_gqa_cache(q, K, V, nq, nkv, n, d, d ** -0.5, n - 1, 0)
        assert orc.rel_err(o.cpu().numpy().reshape(nq, d), want) <= PARITY_TOL
    finally:
        kv.close()


def test_paged_plan_wait_runs_out_then_recovers(mb, torch_cuda, orc):
    torch = torch_cuda
    lens = [9000, 130, 2049]
    nq, nkv, d, ps = 32, 8, 128, 16
    Kp, Vp, bt = make_pool(lens, nkv, d, ps, seed=90)
    Q = np.random.default_rng(91).standard_normal((3, nq, d)).astype(np.float32)
    dQ, dK, dV, dbt = cu(torch, Q), cu(torch, Kp), cu(torch, Vp), cu(torch, bt)
    plan = mb.PagedPlan()
    try:
        plan.build(nq, nkv, d, lens, None, 0)
        O = torch.empty((3, nq, d), device="cuda")
        mb.debug_withhold_next(LIMIT_NS)
        plan.decode(dQ, O, dK, dV, dbt, ps, d ** -0.5)
        with pytest.raises(mb.MolotError) as ei:
            plan.check()
        assert ei.value.status == mb.ERR_TIMEOUT
        O.fill_(float("nan"))
        plan.decode(dQ, O, dK, dV, dbt, ps, d ** -0.5)
        plan.check()
        want = orc.attn_decode_paged(Q, Kp, Vp, bt, lens, None, 3, nq, nkv, d, ps, d ** -0.5, 0)
        assert orc.rel_err(O.cpu().numpy(), want) <= PARITY_TOL
    finally:
        plan.close()


def test_default_workspace_reports_through_device_status(mb, torch_cuda, orc):
    torch = torch_cuda
    nq, nkv, d, n = 16, 4, 128, 5000
    rng = np.random.default_rng(5)
    K = cu(torch, rng.standard_normal((n, nkv * d)).astype(np.float32))
    V = cu(torch, rng.standard_normal((n, nkv * d)).astype(np.float32))
    q = cu(torch, rng.standard_normal((nq, d)).astype(np.float32))
    o = torch.empty((nq, d), device="cuda")
    assert mb.device_status() == mb.OK
    mb.debug_withhold_next(LIMIT_NS)
    mb.decode_strided(q, K, V, o, nq, nkv, n, d, nkv * d, d, d ** -0.5, n - 1, 0)
    assert mb.device_status(clear=False) == mb.ERR_TIMEOUT
    assert mb.device_status(clear=True) == mb.ERR_TIMEOUT
    assert mb.device_status() == mb.OK
    mb.decode_strided(q, K, V, o, nq, nkv, n, d, nkv * d, d, d ** -0.5, n - 1, 0)
    assert mb.device_status() == mb.OK
    want = orc.attn_decode_gqa_cache(q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(), nq, nkv,
                                     n, d, d ** -0.5, n - 1, 0)
    assert orc.rel_err(o.cpu().numpy(), want) <= PARITY_TOL


def test_withhold_request_is_cancelled_by_zero(mb, torch_cuda, orc):
    torch = torch_cuda
    nq, nkv, d, n = 8, 2, 64, 700
    rng = np.random.default_rng(6)
    K = cu(torch, rng.standard_normal((n, nkv * d)).astype(np.float32))
    V = cu(torch, rng.standard_normal((n, nkv * d)).astype(np.float32))
    q = cu(torch, rng.standard_normal((nq, d)).astype(np.float32))
    o = torch.empty((nq, d), device="cuda")
    mb.debug_withhold_next(LIMIT_NS)
    mb.debug_withhold_next(0)
    mb.decode_strided(q, K, V, o, nq, nkv, n, d, nkv * d, d, d ** -0.5, n - 1, 0)
    assert mb.device_status() == mb.OK
