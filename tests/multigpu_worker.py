"""Worker for the multi-GPU tests (launched by torchrun from tests/test_multigpu.py).

Checks, on N ranks over NVLink:
  * team barrier + NVLS / P2P all-reduce (bf16 and fp32) against the plain sum;
  * fused data-parallel step (reduce + AdamW + broadcast kernel) against the
    NCCL reduce-scatter / AdamW / all-gather path from identical gradients;
  * the backward-overlapped bucketed DP engine against the NCCL engine;
  * Qwen TP decode (push-reduce or multicast-reduce GEMM, vocabulary-parallel
    LM head) and prefill against TP=1 tokens.
Prints "OK <name>" lines; any mismatch raises (non-zero exit).
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from aether_b200 import _ext  # noqa: E402
from aether_b200.parallel import dist as D  # noqa: E402


def check_allreduce(team, info):
    from aether_b200.parallel.symm import SymmTeam  # noqa: F401

    for dtype in (torch.bfloat16, torch.float32):
        n = 1 << 16
        buf = team.alloc(n, dtype)
        g = torch.Generator(device=info.device).manual_seed(100 + team.rank)
        x = torch.randn(n, generator=g, device=info.device).to(dtype)
        buf.tensor.copy_(x)
        allx = [torch.empty_like(x) for _ in range(team.world)]
        dist.all_gather(allx, x)
        ref = torch.stack([a.float() for a in allx]).sum(0)
        team.all_reduce_(buf)
        torch.cuda.synchronize()
        err = float((buf.tensor.float() - ref).norm() / ref.norm())
        assert err < (1e-2 if dtype == torch.bfloat16 else 1e-6), (dtype, err)
    print(f"OK allreduce mc={team.has_multicast}", flush=True)


def check_fused_dp(info):
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.dp import DataParallel, FusedDataParallel, team_alloc
    from aether_b200.parallel.symm import SymmTeam

    cfg = GPTConfig(vocab=512, d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=128)
    team = SymmTeam(info)
    m1 = GPT(cfg, device=info.device, seed=5, pad_multiple=info.world, alloc=team_alloc(team))
    m2 = GPT(cfg, device=info.device, seed=5, pad_multiple=info.world)
    fused = FusedDataParallel(m1.arena, team, lr=1e-3)
    base = DataParallel(m2.arena, info, lr=1e-3)
    toks = torch.randint(0, 512, (2, 129), device=info.device,
                         generator=torch.Generator(device=info.device).manual_seed(info.rank))
    for step in range(3):
        m1.arena.zero_grad()
        m1.loss(toks[:, :-1].contiguous(), toks[:, 1:].contiguous()).backward()
        m2.arena.grad.copy_(m1.arena.grad)  # both optimisers see the same gradient
        fused.step()
        base.step()
        torch.cuda.synchronize()
        d = float((m1.arena.bf16.float() - m2.arena.bf16.float()).abs().max())
        dm = float((m1.arena.master[fused.start:fused.end] - m2.arena.master[base.start:base.end]).abs().max())
        assert dm < 1e-5 and d < 1e-2, (step, d, dm)
        m2.arena.bf16.copy_(m1.arena.bf16)  # keep both forwards identical
    assert _ext.check_status() == 0
    print(f"OK fused_dp mc={team.has_multicast}", flush=True)


def check_overlap_dp(info):
    """Backward-overlapped bucketed DP (through Trainer, two micro-batches per
    step) against the NCCL DataParallel engine from the same weights and data."""
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.dp import DataParallel, OverlappedDataParallel, team_alloc
    from aether_b200.parallel.symm import SymmTeam
    from aether_b200.train import Trainer

    cfg = GPTConfig(vocab=512, d_model=256, n_layers=3, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=128)
    team = SymmTeam(info)
    m1 = GPT(cfg, device=info.device, seed=5, pad_multiple=info.world, alloc=team_alloc(team))
    m2 = GPT(cfg, device=info.device, seed=5, pad_multiple=info.world)
    t1 = Trainer(m1, info, lr=1e-3, micro_batch=2, dp=OverlappedDataParallel(m1.arena, team, lr=1e-3))
    t2 = Trainer(m2, info, lr=1e-3, micro_batch=2, dp=DataParallel(m2.arena, info, lr=1e-3))
    toks = torch.randint(0, 512, (4, 129), device=info.device,
                         generator=torch.Generator(device=info.device).manual_seed(info.rank))
    for step in range(3):
        l1 = float(t1.train_step(toks))
        l2 = float(t2.train_step(toks))
        torch.cuda.synchronize()
        d = float((m1.arena.bf16.float() - m2.arena.bf16.float()).abs().max())
        same = float((m1.arena.bf16.view(torch.int16) == m2.arena.bf16.view(torch.int16)).float().mean())
        # two ranks sum in the same order as NCCL (a + b == b + a); more ranks sum in a
        # different order, and AdamW amplifies those last-bit differences where a
        # gradient is ~0, so a few bf16 parameters move by one unit in the last place
        assert abs(l1 - l2) < 1e-3 * abs(l2) and d < 1e-2 and same > (0.99 if info.world == 2 else 0.9), \
            (step, l1, l2, d, same)
    assert _ext.check_status() == 0
    print(f"OK overlap_dp mc={team.has_multicast} same={same:.4f}", flush=True)


def check_tp_qwen(info):
    from aether_b200.models.qwen import QwenConfig, QwenModel
    from aether_b200.parallel.tp import TensorParallel

    cfg = QwenConfig(vocab=2048, d_model=1024, n_layers=2, n_heads=8, n_kv_heads=2, d_ff=2048, max_seq=512,
                     init_std=0.05)
    tp = TensorParallel(info)
    mt = QwenModel(cfg, device=info.device, seed=3, max_batch=4, max_seq=512, tp=tp)
    m1 = QwenModel(cfg, device=info.device, seed=3, max_batch=4, max_seq=512)
    prompts = torch.randint(0, cfg.vocab, (3, 33), device=info.device, generator=torch.Generator(device=info.device).manual_seed(9))
    out_t = mt.generate(prompts, 8, use_graph=True)
    out_1 = m1.generate(prompts, 8, use_graph=False)
    agree = float((out_t == out_1).float().mean())
    assert agree > 0.9, (agree, out_t, out_1)
    assert _ext.check_status() == 0
    print(f"OK tp_qwen agree={agree:.3f} mc={tp.team.has_multicast}", flush=True)


def check_tp_mega(info):
    """The one-kernel TP decode step (multimem reductions + flag barriers inside
    the kernel) against the TP kernel chain: per-rank vocabulary-slice logits
    and merged greedy tokens, batch buckets 1 / 2 / 4, teacher-forced."""
    from aether_b200.models.qwen import QwenConfig, QwenModel
    from aether_b200.parallel.tp import TensorParallel

    cfg = QwenConfig(vocab=2048, d_model=1024, n_layers=3, n_heads=8, n_kv_heads=2, d_ff=2048, max_seq=512,
                     init_std=0.05)
    tp = TensorParallel(info)
    ma = QwenModel(cfg, device=info.device, seed=5, max_batch=4, max_seq=512, tp=tp)
    mb = QwenModel(cfg, device=info.device, seed=5, max_batch=4, max_seq=512, tp=tp)
    ma.mega_batches = {1, 2, 4}
    mb.mega = False
    if not ma.mega:
        print("OK tp_mega skipped: no multicast reduction buffers", flush=True)
        return
    w = ma.w
    agree = []
    for B in (1, 2, 4):
        g = torch.Generator(device=info.device).manual_seed(20 + B)
        prompts = torch.randint(0, cfg.vocab, (B, 130), device=info.device, generator=g)
        tok = mb.prefill(prompts)
        ma.prefill(prompts)
        pos = torch.full((B,), 130, dtype=torch.int32, device=info.device)
        for step in range(4):
            b = ma.buf
            b["tok"][:B].copy_(tok)
            b["pos"][:B].copy_(pos)
            b["seqlen"][:B].copy_(pos + 1)
            b["slot"][:B].copy_(torch.arange(B, dtype=torch.int32, device=info.device))
            loc = torch.zeros(B, w.vocab_per, device=info.device)
            ma._decode_mega(B, loc)
            na = b["next"][:B].clone()
            nb = mb.decode_step(tok, pos, use_graph=step % 2 == 1, want_logits=True).clone()
            full = mb.buf["logits"][:B, w.vocab_col0 : w.vocab_col0 + w.vocab_n]
            err = float((loc[:, : w.vocab_n] - full).abs().max())
            assert err <= 2e-2 * float(full.abs().max()) + 1e-5, (B, step, err)
            agree.append(float((na == nb).float().mean()))
            tok, pos = nb, pos + 1
    assert sum(agree) / len(agree) > 0.9, agree
    assert _ext.check_status() == 0
    print(f"OK tp_mega agree={sum(agree) / len(agree):.3f}", flush=True)


def check_pp(info):
    """1F1B pipeline over NCCL p2p (one stage per rank) against one GPU."""
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.optim import FlatAdamW
    from aether_b200.parallel.pp import GPTPipelineStage, run_1f1b

    cfg = GPTConfig(vocab=512, d_model=256, n_layers=2 * info.world, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=128)
    st = GPTPipelineStage(cfg, info.rank, info.world, info.device, seed=11, lr=1e-3, weight_decay=0.0)
    g = torch.Generator().manual_seed(5)
    toks = torch.randint(0, 512, (4, 2, 129), generator=g)
    batches = [(t[:, :-1].contiguous(), t[:, 1:].contiguous()) for t in toks]
    losses = []
    for _ in range(2):
        st.zero_grad()
        loss = run_1f1b(st, batches)
        st.step()
        if loss is not None:
            losses.append(float(loss))
    t = torch.tensor(losses or [0.0, 0.0], device=info.device)
    dist.broadcast(t, src=info.world - 1)
    if info.rank == 0:
        ref = GPT(cfg, device=info.device, seed=11)
        opt = FlatAdamW(ref.arena, lr=1e-3, weight_decay=0.0)
        n_tok = sum(tg.numel() for _, tg in batches)
        for step in range(2):
            ref.arena.zero_grad()
            tot = 0.0
            for ids, tg in batches:
                l = ref.loss(ids.to(info.device), tg.to(info.device), 1.0 / n_tok)
                l.backward()
                tot += float(l)
            opt.step()
            assert abs(tot - float(t[step])) < 2e-2 * abs(tot), (step, tot, float(t[step]))
    dist.barrier()
    print(f"OK pp losses={[round(float(x), 4) for x in t]}", flush=True)


def check_tp_train(info, sp=False, fused=False):
    """Megatron TP over all ranks (in-kernel symmetric-memory all-reduce; with
    sp, NCCL reduce-scatter / all-gather around a token-split residual; with
    fused, every projection one gemm_tp kernel with its all-gather /
    reduce-scatter inside) against one GPU."""
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.tp_train import make_mesh, shard_tensor

    w = info.world
    cfg = GPTConfig(vocab=512, d_model=128 * w, n_layers=2, n_heads=w, n_kv_heads=w, d_ff=256 * w, max_seq=128)
    mesh = make_mesh(w, use_symm=not fused, sequence_parallel=sp, fused=fused)
    m = GPT(cfg, device=info.device, seed=13, tp=mesh.tp)
    ref = GPT(cfg, device=info.device, seed=13)
    # fused: 256 token rows per rank (a multiple of the kernel's 128-row tiles)
    toks = torch.randint(0, 512, (2 * w if fused else 2, 129), generator=torch.Generator().manual_seed(2))
    ids, tg = toks[:, :-1].contiguous().to(info.device), toks[:, 1:].contiguous().to(info.device)
    lt = m.loss(ids, tg)
    lt.backward()
    m.finish_grads()
    lr = ref.loss(ids, tg)
    lr.backward()
    assert abs(float(lt.detach()) - float(lr.detach())) < 1e-2 * abs(float(lr.detach()))
    for n, s in m.arena.slots.items():
        g = m.arena.grad[s.offset : s.offset + s.numel].view(s.shape)
        rs = ref.arena.slots[n]
        want = shard_tensor(cfg, n, ref.arena.grad[rs.offset : rs.offset + rs.numel].view(rs.shape), mesh.tp.rank, w)
        err = float((g - want).norm() / want.norm().clamp(min=1e-12))
        assert err < 5e-2, (n, err)
    torch.cuda.synchronize()
    assert _ext.check_status() == 0
    if fused:
        assert all(r.n_ag > 0 and r.n_rs > 0 for r in mesh.tp.fused.rings.values()), "fused path not taken"
    print(f"OK tp_train{'_sp' if sp else ''}{'_fused' if fused else ''} loss={float(lt.detach()):.4f}", flush=True)


def check_fsdp(info):
    """ZeRO-2 and ZeRO-3 over all ranks: the gathered gradient shards equal the
    all-reduced gradients of the flat arena, and one step keeps the loss finite."""
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.fsdp import ShardedDataParallel, ShardSpec

    w, r = info.world, info.rank
    cfg = GPTConfig(vocab=512, d_model=256, n_layers=3, n_heads=4, n_kv_heads=4, d_ff=512, max_seq=128)
    g = torch.Generator().manual_seed(40 + r)
    toks = [torch.randint(0, 512, (2, 129), generator=g).to(info.device) for _ in range(2)]
    ref = GPT(cfg, device=info.device, seed=5)
    for t in toks:
        ref.loss(t[:, :-1].contiguous(), t[:, 1:].contiguous()).backward()
    dist.all_reduce(ref.arena.grad)
    from aether_b200.parallel.symm import SymmTeam

    ref_l0 = float(GPT(cfg, device=info.device, seed=5).loss(toks[0][:, :-1].contiguous(),
                                                              toks[0][:, 1:].contiguous()).detach())
    stages = [s for s in os.environ.get("AETHER_FSDP_CHECK", "2,3,3-fused").split(",")]
    after = {}  # stage -> this rank's loss after one optimizer step
    for stage in [int(s) if s.isdigit() else s for s in stages]:
        # 3-fused: every layer's parameter all-gather inside its first consuming GEMM
        spec = ShardSpec(r, w, 3, fused=SymmTeam(info)) if stage == "3-fused" else ShardSpec(r, w, stage)
        m = GPT(cfg, device=info.device, seed=5, shard=spec)
        for j, t in enumerate(toks):
            lj = m.loss(t[:, :-1].contiguous(), t[:, 1:].contiguous())
            if j == 0:  # the forward alone (parameter gathers) against the unsharded model
                l0 = float(lj.detach())
                assert abs(l0 - ref_l0) < 1e-3 * abs(ref_l0), (stage, "forward loss", l0, ref_l0)
            lj.backward()
        a = m.arena
        a._finish_grads()
        for u, unit in a.units.items():
            full = torch.empty(unit.numel, dtype=torch.float32, device=info.device)
            a._all_gather(full, a._shard_of(u, a.grad).contiguous(), False)
            for n, s in unit.slots.items():
                o = ref.arena.slots[n].offset
                want = ref.arena.grad[o : o + s.numel]
                err = float((full[s.offset : s.offset + s.numel] - want).norm() / want.norm().clamp(min=1e-12))
                assert err < 1e-4, (stage, n, err)
        eng = ShardedDataParallel(a, lr=1e-3)
        eng.step()
        loss = m.loss(toks[0][:, :-1].contiguous(), toks[0][:, 1:].contiguous())
        assert torch.isfinite(loss)
        after[stage] = float(loss.detach())
        if stage == "3-fused":
            loss.backward()  # a second backward on the same slots (flags' use counts advance)
            a._finish_grads()
            assert sum(a._puses) >= 2 * cfg.n_layers, a._puses  # gathers ran inside the GEMMs
            if 3 in after:  # same data, same step: the NCCL-gathering engine's loss
                assert abs(after[3] - after[stage]) < 1e-3 * abs(after[3]), after
            assert _ext.check_status() == 0
    torch.cuda.synchronize()
    print(f"OK fsdp stages=2,3,3-fused world={w}", flush=True)


def check_cp(info):
    """Context parallelism over all ranks (K/V all-gather) against the whole sequence on one GPU."""
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.cp import CPGroup, shard_sequence

    w, r = info.world, info.rank
    S = 128 * w
    cfg = GPTConfig(vocab=512, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=512, max_seq=S)
    toks = torch.randint(0, 512, (2, S + 1), generator=torch.Generator().manual_seed(9)).to(info.device)
    cp = CPGroup(r, w, None)
    m = GPT(cfg, device=info.device, seed=8, cp=cp)
    ids, tg = shard_sequence(toks, cp)
    lc = m.loss(ids, tg)
    lc.backward()
    dist.all_reduce(m.arena.grad)
    m.arena.grad /= w
    lsum = lc.detach().clone()
    dist.all_reduce(lsum)
    ref = GPT(cfg, device=info.device, seed=8)
    lr = ref.loss(toks[:, :-1].contiguous(), toks[:, 1:].contiguous())
    lr.backward()
    assert abs(float(lsum) / w - float(lr.detach())) < 1e-2 * abs(float(lr.detach()))
    err = float((m.arena.grad - ref.arena.grad).norm() / ref.arena.grad.norm())
    assert err < 5e-2, err
    torch.cuda.synchronize()
    print(f"OK cp world={w} grad_err={err:.2e}", flush=True)


def check_ep(info):
    """MoE with experts partitioned over all ranks (attention and shared expert TP-sharded) against one GPU."""
    from aether_b200.models.moe import MoEConfig, MoEQwenModel
    from aether_b200.parallel.tp import TensorParallel

    w = info.world
    cfg = MoEConfig(vocab=512, d_model=256, n_layers=2, n_heads=2 * w, n_kv_heads=w, d_ff=8, max_seq=64,
                    init_std=0.05, n_experts=4 * w, top_k=2, d_expert=128, shared_ff=128 * w)
    tp = TensorParallel(info)
    m = MoEQwenModel(cfg, device=info.device, seed=1, max_batch=2, max_seq=64, tp=tp)
    ref = MoEQwenModel(cfg, device=info.device, seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 512, (2, 16), generator=torch.Generator().manual_seed(2)).to(info.device)
    _, lt = m.prefill(toks, return_logits=True)
    _, lr = ref.prefill(toks, return_logits=True)
    err = float((lt - lr).norm() / lr.norm())
    assert err < 3e-2, err
    torch.cuda.synchronize()
    tp.close()
    print(f"OK ep world={w} err={err:.2e}", flush=True)


def check_mla_tp(info):
    """DeepSeek-V2-family MLA model with heads, experts and FFNs split over all ranks against one GPU."""
    from aether_b200.models.deepseek import DeepSeekConfig, DeepSeekModel
    from aether_b200.parallel.tp import TensorParallel

    w = info.world
    cfg = DeepSeekConfig(vocab=512, d_model=256, n_layers=2, n_heads=4 * w, d_ff=256 * w, first_dense=1,
                         n_experts=4 * w, top_k=2, d_expert=64, n_shared=w, max_seq=64, init_std=0.05)
    tp = TensorParallel(info)
    m = DeepSeekModel(cfg, device=info.device, seed=1, max_batch=2, max_seq=64, tp=tp)
    ref = DeepSeekModel(cfg, device=info.device, seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 512, (2, 16), generator=torch.Generator().manual_seed(2)).to(info.device)
    _, lt = m.prefill(toks, return_logits=True)
    _, lr = ref.prefill(toks, return_logits=True)
    err = float((lt - lr).norm() / lr.norm())
    assert err < 3e-2, err
    torch.cuda.synchronize()
    tp.close()
    print(f"OK mla_tp world={w} err={err:.2e}", flush=True)


def main():
    info = D.init(timeout_s=120)
    from aether_b200.parallel.symm import SymmTeam

    team = SymmTeam(info)
    which = sys.argv[1:] or ["allreduce", "dp", "overlap_dp", "tp", "tp_mega", "pp", "tp_train", "fsdp", "cp", "ep",
                             "mla_tp"]
    if "allreduce" in which:
        check_allreduce(team, info)
    if "dp" in which:
        check_fused_dp(info)
    if "overlap_dp" in which:
        check_overlap_dp(info)
    if "tp" in which:
        check_tp_qwen(info)
    if "tp_mega" in which:
        check_tp_mega(info)
    if "pp" in which:
        check_pp(info)
    if "tp_train" in which:
        check_tp_train(info)
        check_tp_train(info, sp=True)
        check_tp_train(info, sp=True, fused=True)
    if "fsdp" in which:
        check_fsdp(info)
    if "cp" in which:
        check_cp(info)
    if "ep" in which:
        check_ep(info)
    if "mla_tp" in which:
        check_mla_tp(info)
    torch.cuda.synchronize()
    dist.barrier()
    D.shutdown()


if __name__ == "__main__":
    main()
