"""Tensor-parallel serving on gloo ranks (CPU): rank 0 runs the engine on a
BroadcastModel, rank 1 replays every call; greedy outputs match the
single-rank model."""
import os
import socket

import pytest
import torch

TINY = dict(vocab=512, d_model=128, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=256, max_seq=64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _GlooTP:
    """The TensorParallel contract on gloo: in-place all-reduce, and the
    reducing GEMM (fp32 sum over ranks of x @ w^T) of the decode path."""

    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def all_reduce_(self, t):
        import torch.distributed as dist

        f = t.float()
        dist.all_reduce(f)
        t.copy_(f)
        return t

    def reduce_gemm(self, x, w, which):
        import torch.distributed as dist

        acc = x.float() @ w.float().t()
        dist.all_reduce(acc)
        return acc

    def finalize_wait(self):
        return None

    def vocab_argmax(self, logits, n_loc, col0, out=None):
        import torch.distributed as dist

        loc = logits[:, :n_loc].float()
        best, idx = loc.max(-1)
        cand = torch.stack([best, (idx + col0).float()], -1)
        allc = [torch.empty_like(cand) for _ in range(self.world)]
        dist.all_gather(allc, cand)
        allc = torch.stack(allc)  # [world, rows, 2]; ties go to the lowest rank = lowest index
        r = allc[..., 0].argmax(0)
        res = allc[r, torch.arange(allc.shape[1]), 1].long()
        if out is None:
            return res
        out.copy_(res)
        return out

    def gather_vocab(self, logits, n_loc, col0, V, out=None):
        import torch.distributed as dist

        per = logits[:, :n_loc].float().contiguous()
        sizes = [None] * self.world
        dist.all_gather_object(sizes, per.shape[1])
        parts = [torch.empty(per.shape[0], n, dtype=torch.float32) for n in sizes]
        dist.all_gather(parts, per)
        full = torch.cat(parts, 1)[:, :V]
        if out is None:
            return full
        out.copy_(full)
        return out


def _worker(rank, world, port, q, tie=True):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from aether_b200.models.qwen import QwenConfig, QwenModel
    from aether_b200.serving.tp_serve import BroadcastModel, follow

    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctrl = dist.new_group(backend="gloo")
    model = QwenModel(QwenConfig(**TINY, tie_embeddings=tie), device="cpu", seed=4, max_batch=2, max_seq=64,
                      tp=_GlooTP(rank, world))
    if rank == 0:
        from aether_b200.serving.engine import Engine
        from aether_b200.serving.sampling import SamplingParams
        from aether_b200.serving.tokenizer import ByteTokenizer

        bm = BroadcastModel(model, ctrl)
        eng = Engine(bm, ByteTokenizer(), max_concurrent=2, use_graph=False)
        rs = [eng.submit(list(b"hello world"), SamplingParams(max_tokens=5)),
              eng.submit(list(b"tensor parallel"), SamplingParams(max_tokens=4))]
        outs = []
        for r in rs:
            while r.out.get(timeout=120) is not None:
                pass
            outs.append(list(r.tokens))
        eng.shutdown()
        bm.stop()
        q.put(("outs", outs))
    else:
        q.put(("replayed", follow(model, ctrl)))
    dist.destroy_process_group()


@pytest.mark.parametrize("tie", [True, False])
def test_tp_serving_matches_one_rank(tie):
    """Tied head: the shard is a slice of the embedding; untied: each rank
    keeps only its vocabulary slice of the head (vocabulary-parallel LM head)."""
    import multiprocessing as mp

    from aether_b200.models.qwen import QwenConfig, QwenModel

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, tie)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got["replayed"] >= 2  # prefills and decode steps reached rank 1
    ref = QwenModel(QwenConfig(**TINY, tie_embeddings=tie), device="cpu", seed=4, max_batch=2, max_seq=64)
    for prompt, n, out in ((b"hello world", 5, got["outs"][0]), (b"tensor parallel", 4, got["outs"][1])):
        want = ref.generate(torch.tensor([list(prompt)]), n, use_graph=False)[0].tolist()
        assert out == want, (prompt, out, want)
