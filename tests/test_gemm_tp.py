"""The fused TP-training GEMM (csrc/gemm_tp.cu) on one GPU: all ranks of a TP
group run as one cooperative launch (rank y = blockIdx.y), each rank's
buffers standing in for its peers' symmetric memory. Every mode is checked
against an fp32 PyTorch reference over several calls, so both ring slots are
used twice and the flags' use counts advance as they do in training."""
import pytest
import torch

from aether_b200 import _ext
from aether_b200.ops import functional as F

pytestmark = pytest.mark.gpu

BM = 128


def _C():
    return _ext.C()


class Group:
    """Per-rank gather / receive rings of one emulated TP group."""

    def __init__(self, tp, Ml, d, dev):
        M = tp * Ml
        mt = Ml // BM
        nn = (d + 255) // 256
        self.tp, self.Ml, self.d = tp, Ml, d
        self.ag = [[torch.zeros(M, d, dtype=torch.bfloat16, device=dev) for _ in range(tp)] for _ in range(2)]
        self.agf = [[torch.zeros(tp * mt, dtype=torch.int32, device=dev) for _ in range(tp)] for _ in range(2)]
        self.rs = [[torch.zeros(tp * Ml * d, dtype=torch.bfloat16, device=dev) for _ in range(tp)] for _ in range(2)]
        self.rsf = [[torch.zeros(mt * nn * 4, dtype=torch.int32, device=dev) for _ in range(tp)] for _ in range(2)]
        self.n_ag = self.n_rs = 0

    def next_ag(self):
        s, e = self.n_ag & 1, (self.n_ag >> 1) + 1
        self.n_ag += 1
        return s, e

    def next_rs(self):
        s, e = self.n_rs & 1, (self.n_rs >> 1) + 1
        self.n_rs += 1
        return s, e

    def call(self, a_local, a_ag, b, out, residual, push_src, b_mn, ag_mode, rs, local_copy, ag_slot=0, ag_ep=0,
             rs_slot=0, rs_ep=0):
        ptr = lambda ts: [t.data_ptr() for t in ts]
        F.gemm_tp(a_local, a_ag, b, out, residual, push_src, list(range(self.tp)), self.tp, self.Ml, b_mn, ag_mode,
                     rs, local_copy, ptr(self.ag[ag_slot]) if ag_mode else [], ptr(self.agf[ag_slot]) if ag_mode else [],
                     0, ptr(self.rs[rs_slot]) if rs else [], ptr(self.rsf[rs_slot]) if rs else [], ag_ep, rs_ep, 2.0)


def _rand(*shape, gen):
    return (torch.randn(*shape, generator=gen) * 0.5).to(torch.bfloat16).cuda()


def _close(got, want, what):
    err = float((got.float() - want).norm() / want.norm().clamp(min=1e-6))
    assert err < 1e-2, (what, err)


def _status_ok():
    torch.cuda.synchronize()
    assert _ext.check_status() == 0


@pytest.mark.parametrize("tp,Ml,K,N", [(2, 256, 200, 320), (2, 384, 512, 768), (4, 128, 256, 512)])
def test_allgather_gemm(tp, Ml, K, N):
    g = torch.Generator().manual_seed(1)
    grp = Group(tp, Ml, K, "cuda")
    for call in range(4):
        h = [_rand(Ml, K, gen=g) for _ in range(tp)]
        w = [_rand(N, K, gen=g) for _ in range(tp)]
        y = [torch.empty(tp * Ml, N, dtype=torch.bfloat16, device="cuda") for _ in range(tp)]
        slot, ep = grp.next_ag()
        grp.call(h, grp.ag[slot], w, y, [], h, False, 1, False, False, ag_slot=slot, ag_ep=ep)
        hf = torch.cat([x.float() for x in h])
        for r in range(tp):
            _close(y[r], hf @ w[r].float().t(), f"call {call} rank {r}")
    _status_ok()


@pytest.mark.parametrize("tp,Ml,K,N", [(2, 256, 192, 256), (2, 256, 512, 320), (4, 256, 256, 512)])
def test_gemm_reduce_scatter(tp, Ml, K, N):
    g = torch.Generator().manual_seed(2)
    grp = Group(tp, Ml, N, "cuda")
    M = tp * Ml
    for call in range(4):
        o = [_rand(M, K, gen=g) for _ in range(tp)]
        w = [_rand(N, K, gen=g) for _ in range(tp)]
        res = [_rand(Ml, N, gen=g) for _ in range(tp)] if call % 2 == 0 else []
        x = [torch.empty(Ml, N, dtype=torch.bfloat16, device="cuda") for _ in range(tp)]
        slot, ep = grp.next_rs()
        grp.call(o, [], w, x, res, [], False, 0, True, False, rs_slot=slot, rs_ep=ep)
        tot = sum(o[s].float() @ w[s].float().t() for s in range(tp))
        for r in range(tp):
            want = tot[r * Ml : (r + 1) * Ml] + (res[r].float() if res else 0.0)
            _close(x[r], want, f"call {call} rank {r}")
    _status_ok()


@pytest.mark.parametrize("tp,Ml,n,d", [(2, 256, 384, 256), (4, 128, 256, 512)])
def test_backward_modes(tp, Ml, n, d):
    """Column backward (dgrad reduce-scatter + rows gathered alongside) and row
    backward (gathered A rows, own rows copied in for the weight gradient),
    interleaved as in a layer's backward."""
    g = torch.Generator().manual_seed(3)
    grp = Group(tp, Ml, d, "cuda")
    M = tp * Ml
    for call in range(3):
        # column: dh = RS(dy . w), w [n, d] (b_mn); h gathered alongside
        dy = [_rand(M, n, gen=g) for _ in range(tp)]
        w = [_rand(n, d, gen=g) for _ in range(tp)]
        h = [_rand(Ml, d, gen=g) for _ in range(tp)]
        dh = [torch.empty(Ml, d, dtype=torch.bfloat16, device="cuda") for _ in range(tp)]
        a_slot, a_ep = grp.next_ag()
        r_slot, r_ep = grp.next_rs()
        grp.call(dy, [], w, dh, [], h, True, 2, True, True, ag_slot=a_slot, ag_ep=a_ep, rs_slot=r_slot, rs_ep=r_ep)
        tot = sum(dy[s].float() @ w[s].float() for s in range(tp))
        hf = torch.cat(h)
        for r in range(tp):
            _close(dh[r], tot[r * Ml : (r + 1) * Ml], f"column dgrad call {call} rank {r}")
            assert torch.equal(grp.ag[a_slot][r], hf), f"gathered rows call {call} rank {r}"
        # row: do = AG(dx) . w, w [d, n] (b_mn); dx rows gathered (own rows copied in)
        dx = [_rand(Ml, d, gen=g) for _ in range(tp)]
        w2 = [_rand(d, n, gen=g) for _ in range(tp)]
        do = [torch.empty(M, n, dtype=torch.bfloat16, device="cuda") for _ in range(tp)]
        slot, ep = grp.next_ag()
        grp.call(dx, grp.ag[slot], w2, do, [], dx, True, 1, False, True, ag_slot=slot, ag_ep=ep)
        dxf = torch.cat(dx)
        for r in range(tp):
            _close(do[r], dxf.float() @ w2[r].float(), f"row dgrad call {call} rank {r}")
            assert torch.equal(grp.ag[slot][r], dxf), f"gathered dY call {call} rank {r}"
    _status_ok()


@pytest.mark.parametrize("world,b_mn", [(2, False), (2, True), (4, False)])
def test_param_gather_gemm(world, b_mn):
    """ZeRO-3 form: the weight lives in a flat parameter unit sharded over the
    ranks; one kernel gathers the unit into every rank's buffer and multiplies
    with the weight as its chunks arrive. Two calls (updated parameters): the
    flags' use count and the chunk-ticket reset both carry over."""
    g = torch.Generator().manual_seed(4)
    chunk, M, N, K = 2048, 256, 384, 256
    off = 1024  # the weight's element offset inside the unit (another tensor before it)
    S = -(-(off + N * K + 1000) // (world * chunk)) * chunk
    units = [torch.zeros(world * S, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    flags = [torch.zeros(world * (S // chunk), dtype=torch.int32, device="cuda") for _ in range(world)]
    ctr = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(world)]
    ready = [torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]
    for epoch in (1, 2):
        full = (torch.randn(world * S, generator=g) * 0.5).to(torch.bfloat16)
        shards = [full[r * S : (r + 1) * S].contiguous().cuda() for r in range(world)]
        a = [_rand(M, K, gen=g) for _ in range(world)]
        shape = (K, N) if b_mn else (N, K)
        views = [u[off : off + N * K].view(*shape) for u in units]
        out = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        F.gemm_param_gather(a, views, out, shards, ctr, list(range(world)), world, chunk, b_mn,
                               [u.data_ptr() for u in units], [f.data_ptr() for f in flags],
                               [x.data_ptr() for x in ready], 0, epoch, 2.0)
        w = full[off : off + N * K].float().view(*shape).cuda()
        for r in range(world):
            want = a[r].float() @ (w if b_mn else w.t())
            _close(out[r], want, f"epoch {epoch} rank {r}")
            assert torch.equal(units[r].cpu(), full), f"unit gathered on rank {r}"
            assert int(ctr[r].abs().sum()) == 0
    _status_ok()
