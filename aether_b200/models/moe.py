"""Mixture-of-experts decoder (Qwen2-MoE / Mixtral family) for serving.

Attention, KV cache (contiguous or paged), prefill and CUDA-graph decode are
the Qwen2 model's; every FFN is a sparse MoE block:
    logits = h Wr^T                        router (tcgen05 GEMM, fp32 out)
    (ids, w) = top-k(softmax(logits))      moe_route, one warp per token
    sort the T*k (token, expert) pairs by expert into 128-row segments
    Y = SwiGLU(X Wgu[e]^T) Wd[e]^T         two grouped tcgen05 GEMMs, each
                                           128-row tile picks its expert's weights
    out = x + sum_j w_j Y[row(t, j)] (+ sigmoid(h Wsg^T) * shared_expert(h))
Qwen2-MoE routes with softmax over all experts then top-k (not renormalised)
and adds a gated shared expert; Mixtral takes softmax over the top-k logits
and has no shared expert.

Expert parallelism: under tensor parallelism the token rows are replicated on
every rank, so the experts are partitioned over the same ranks (rank r holds
experts [r E / w, (r+1) E / w)) and need no all-to-all. Each rank routes all
tokens, permutes only the pairs routed to its experts (the others get row -1),
runs its grouped GEMMs and combines its share together with its TP slice of
the shared expert; one all-reduce of that partial sum finishes the block, the
same reduction as a dense row-parallel FFN.

Reference: the MoE fields of the serving ModelConfig
(runtime/src/serving.rs:459-900), host-side top-k routing (serving.rs:2335)
and one expert GEMV per (token, expert)
(fused_*_expert_matmul_seq1, runtime/src/cuda.rs:5666-6135); MoE is
replicated under the reference's TP plan (runtime/src/tensor_parallel.rs:21-22).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import functional as F
from .qwen import QwenConfig, QwenModel, QwenWeights


@dataclass
class MoEConfig(QwenConfig):
    n_experts: int = 8
    top_k: int = 2
    d_expert: int = 1408
    shared_ff: int = 0  # 0: no shared expert
    router_softmax_all: bool = True
    norm_topk: bool = False

    @staticmethod
    def qwen2_moe_a2_7b(**kw) -> "MoEConfig":
        base = dict(vocab=151936, d_model=2048, n_layers=24, n_heads=16, n_kv_heads=16, d_ff=5632, n_experts=60,
                    top_k=4, d_expert=1408, shared_ff=5632, tie_embeddings=False, qkv_bias=True)
        base.update(kw)
        return MoEConfig(**base)

    @staticmethod
    def mixtral_8x7b(**kw) -> "MoEConfig":
        base = dict(vocab=32000, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, d_ff=8, n_experts=8, top_k=2,
                    d_expert=14336, shared_ff=0, router_softmax_all=False, norm_topk=False, tie_embeddings=False,
                    qkv_bias=False, rope_theta=1e6)
        base.update(kw)
        return MoEConfig(**base)


def expert_range(E: int, rank: int, world: int) -> tuple[int, int]:
    """Experts [e0, e1) of rank ``rank`` out of ``world`` (sizes differ by at most one)."""
    return rank * E // world, (rank + 1) * E // world


class MoEWeights:
    """Router [E, d], experts gate|up [E, 2F, d] and down [E, d, F], and the
    shared expert's gate vector [1, d] (its MLP is the dense FFN of the base
    weights, with d_ff = shared_ff)."""

    def __init__(self, cfg: MoEConfig, device, seed: int = 0, ep_rank: int = 0, ep_size: int = 1):
        """ep_rank / ep_size: keep only this rank's experts [e0, e1) (same
        values as the matching slice of the unpartitioned weights)."""
        dev = torch.device(device)
        E, F_, d = cfg.n_experts, cfg.d_expert, cfg.d_model
        self.e0, self.e1 = expert_range(E, ep_rank, ep_size)

        def rnd(idx, *shape, std=cfg.init_std):
            g = torch.Generator(device=dev).manual_seed(seed * 7919 + 104729 + idx)
            return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

        self.router, self.wgu, self.wd, self.shared_gate = [], [], [], []
        Ep = (E + 7) // 8 * 8  # router rows padded with zeros for the GEMM's N % 8 rule
        for i in range(cfg.n_layers):
            r = torch.zeros(Ep, d, dtype=torch.bfloat16, device=dev)
            r[:E] = rnd(4 * i, E, d)
            self.router.append(r)
            self.wgu.append(rnd(4 * i + 1, E, 2 * F_, d)[self.e0 : self.e1].contiguous())
            self.wd.append(rnd(4 * i + 2, E, d, F_)[self.e0 : self.e1].contiguous())
            self.shared_gate.append(rnd(4 * i + 3, 8, d) if cfg.shared_ff else None)  # row 0 used; 8 rows for the GEMM


class MoEQwenModel(QwenModel):
    def __init__(self, cfg: MoEConfig, device="cuda", seed: int = 0, max_batch: int = 64, max_seq: int | None = None,
                 kv_pages: int = 0, page_size: int = 64, moe_weights: MoEWeights | None = None, tp=None):
        """tp: tensor-parallel group (``all_reduce_``, ``rank``, ``world``):
        attention and the shared expert are TP-sharded, the routed experts
        are partitioned over the same ranks (expert parallelism)."""
        import dataclasses

        r, w = (tp.rank, tp.world) if tp is not None else (0, 1)
        dense = dataclasses.replace(cfg, d_ff=cfg.shared_ff or 8 * w)  # the shared expert is the dense FFN
        weights = QwenWeights(dense, device, seed, r, w)
        super().__init__(cfg, device=device, seed=seed, max_batch=max_batch, max_seq=max_seq, weights=weights,
                         kv_pages=kv_pages, page_size=page_size, tp=tp)
        self.fused_decode = False  # decode runs the MoE block through the generic path
        self.moe = moe_weights or MoEWeights(cfg, device, seed, r, w)

    def _moe(self, i: int, h: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        cfg, m = self.cfg, self.moe
        logits = F.gemm(h, m.router[i], out_dtype=torch.float32)[:, : cfg.n_experts]
        idx, wt = F.moe_route(logits, cfg.top_k, cfg.router_softmax_all, cfg.norm_topk)
        row_of, src_row, tile_group = F.moe_permute(idx, m.e1 - m.e0, m.e0)
        X = F.moe_gather(h, src_row)
        act = F.swiglu(F.gemm_grouped(X, m.wgu[i], tile_group))
        Y = F.gemm_grouped(act, m.wd[i], tile_group)
        extra = None
        if cfg.shared_ff:  # under TP: this rank's slice of the shared expert (a partial sum)
            g = F.gemm(h, m.shared_gate[i], out_dtype=torch.float32)[:, :1]
            s = F.gemm(F.swiglu(F.gemm(h, self.w.wgu[i])), self.w.wd[i])
            extra = (torch.sigmoid(g) * s.float()).to(torch.bfloat16)
        if self.tp is None:
            return F.moe_combine(Y, row_of, wt, res=x, extra=extra)
        y = F.moe_combine(Y, row_of, wt, extra=extra)  # this rank's experts + shared slice
        self.tp.all_reduce_(y)
        return x + y

    def _ffn(self, i, h, x):
        return self._moe(i, h, x)

    def _decode_ffn(self, i, h, x2, x, act, acc) -> None:
        x.copy_(self._moe(i, h, x2))

    def _reference_ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        """fp32 per-token loop over the selected experts (numerics oracle; one rank)."""
        cfg, m = self.cfg, self.moe
        assert m.e0 == 0 and m.e1 == cfg.n_experts, "the oracle needs every expert"
        shp = h.shape
        h2 = h.reshape(-1, shp[-1])
        logits = h2 @ m.router[i][: cfg.n_experts].float().t()
        if cfg.router_softmax_all:
            wt, idx = torch.topk(torch.softmax(logits, -1), cfg.top_k, dim=-1)
            if cfg.norm_topk:
                wt = wt / wt.sum(-1, keepdim=True)
        else:
            top, idx = torch.topk(logits, cfg.top_k, dim=-1)
            wt = torch.softmax(top, -1)
        out = torch.zeros_like(h2)
        for t in range(h2.shape[0]):
            for j in range(cfg.top_k):
                e = int(idx[t, j])
                g, u = (h2[t] @ m.wgu[i][e].float().t()).chunk(2, -1)
                out[t] += wt[t, j] * ((torch.nn.functional.silu(g) * u) @ m.wd[i][e].float().t())
        if cfg.shared_ff:
            gate = torch.sigmoid(h2 @ m.shared_gate[i][0].float())
            out += gate.unsqueeze(-1) * super()._reference_ffn(i, h2)
        return out.view(shp)
