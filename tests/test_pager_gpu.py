"""Continuous batching through the page manager: sequences join and leave
between decode steps, pages are reused, and every step's batched append +
paged decode matches the oracle per sequence (forward.h:554-590 on each
sequence's own cache).  Pools of every storage type: FP32 (bit-exact scores),
BF16 (the oracle on bf16-rounded rows) and Q8 (the oracle on dequantized
rows)."""
import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def bf16(x):
    """Round float32 values to bf16 (nearest even), returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


class Store:
    """How rows of one kv head ([..., d] float32) look in a pool and what
    values the kernels read back from them."""

    def __init__(self, mb, orc, dtype, d):
        self.mb, self.orc, self.dtype, self.d = mb, orc, dtype, d

    def readback(self, rows):
        if self.dtype == "bf16":
            return bf16(rows)
        if self.dtype == "q8":
            q, s = self.orc.quantize_q8_blocks(rows)
            return self.orc.dequantize_q8_blocks(q, s)
        return np.asarray(rows, np.float32)

    def encode(self, torch, rows):
        """Pool representation of rows [nkv][d] as a device tensor."""
        t = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).cuda()
        if self.dtype == "bf16":
            return t.to(torch.bfloat16)
        if self.dtype == "q8":
            d, rb = self.d, self.mb.q8_row_bytes(self.d)
            q, s = self.orc.quantize_q8_blocks(rows)
            out = np.zeros(rows.shape[:-1] + (rb,), np.uint8)
            out[..., :d] = q.view(np.uint8)
            out[..., d:d + d // 8] = np.ascontiguousarray(s).view(np.uint8)
            return torch.from_numpy(out).cuda()
        return t


@pytest.mark.parametrize("dtype", ["f32", "bf16", "q8"])
def test_continuous_batching_steps(mb, torch_cuda, orc, dtype):
    torch = torch_cuda
    L, nq, nkv, d, ps = 2, 8, 2, 128, 16
    scale = d ** -0.5
    rng = np.random.default_rng(42)
    st = Store(mb, orc, dtype, d)
    pager = mb.Pager(L, nkv, d, ps, num_pages=48, max_seqs=4, max_pages_per_seq=12, dtype=dtype)
    plan = mb.PagedPlan(dtype)
    host = {}  # seq -> per layer (K, V) [n][nkv*d] values the kernels read back
    pools = [pager.layer_pools(l) for l in range(L)]

    def add(prompt):
        s = pager.add(prompt)
        bt, _ = pager.tables([s])
        host[s] = []
        for l in range(L):
            k = rng.standard_normal((prompt, nkv, d)).astype(np.float32)
            v = rng.standard_normal((prompt, nkv, d)).astype(np.float32)
            for t in range(prompt):  # scatter the prompt rows into its pages
                page, off = bt[0, t // ps], t % ps
                pools[l][0][page, :, off] = st.encode(torch, k[t])
                pools[l][1][page, :, off] = st.encode(torch, v[t])
            host[s].append((st.readback(k).reshape(prompt, -1),
                            st.readback(v).reshape(prompt, -1)))
        return s

    try:
        live = [add(20), add(35), add(7)]
        for step in range(10):
            if step == 4:
                pager.free(live[1])
                del host[live[1]]
                live.pop(1)
            if step == 5:
                live.append(add(50))  # takes the freed pages first
            for s in live:
                pager.grow(s, 1)
            bt, lens = pager.tables(live)
            B = len(live)
            plan.build(nq, nkv, d, lens)
            bt_dev = torch.from_numpy(bt).cuda()
            for l in range(L):
                q = rng.standard_normal((B, nq, d)).astype(np.float32)
                k = rng.standard_normal((B, nkv, d)).astype(np.float32)
                v = rng.standard_normal((B, nkv, d)).astype(np.float32)
                q_out = torch.empty((B, nq, d), device="cuda")
                O = torch.full((B, nq, d), float("nan"), device="cuda")
                kp, vp = pools[l]
                plan.append(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                            torch.from_numpy(v).cuda(), q_out, kp, vp, bt_dev, ps)
                plan.decode(q_out, O, kp, vp, bt_dev, ps, scale)
                plan.check()
                got = O.cpu().numpy()
                for b, s in enumerate(live):
                    K, V = host[s][l]
                    K = np.vstack([K, st.readback(k[b]).reshape(1, -1)])
                    V = np.vstack([V, st.readback(v[b]).reshape(1, -1)])
                    host[s][l] = (K, V)
                    assert K.shape[0] == lens[b]
                    want = orc.attn_decode_gqa_cache(q[b].reshape(-1), K, V, nq, nkv, lens[b], d,
                                                     scale, lens[b] - 1, 0)
                    assert orc.rel_err(got[b], want) <= PARITY_TOL, (step, l, s)
        assert pager.free_pages() == 48 - sum(-(-pager.length(s) // ps) for s in live)
    finally:
        plan.close()
        pager.close()
