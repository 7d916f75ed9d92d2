"""BERT and ViT encoders against independent fp32 statements of the same
architectures (CPU), and the GPU kernels against the CPU path."""
import math

import pytest
import torch
import torch.nn.functional as tF

from aether_b200.models.encoders import BertConfig, BertEncoder, VitConfig, VitEncoder
from aether_b200.ops import reference as ref

BERT = BertConfig(vocab=500, d_model=128, n_layers=2, n_heads=2, d_ff=256, max_pos=64)
VIT = VitConfig(d=128, n_layers=2, n_heads=2, d_ff=256, patch=8, img=32, n_reg=4)


def bert_ref(m, ids):
    c = m.cfg
    f = lambda t: t.float()  # noqa: E731
    x = f(m.word)[ids] + f(m.pos)[: len(ids)] + f(m.typ)[0]
    x = tF.layer_norm(x, (c.d_model,), f(m.emb_g), f(m.emb_b), c.eps)
    H, D = c.n_heads, c.d_model // c.n_heads
    for L in m.layers:
        qkv = x @ f(L["wqkv"]).t() + f(L["bqkv"])
        q, k, v = (qkv[:, i * c.d_model : (i + 1) * c.d_model].view(-1, H, D).transpose(0, 1) for i in range(3))
        a = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(D), -1) @ v
        y = a.transpose(0, 1).reshape(-1, c.d_model) @ f(L["wo"]).t() + f(L["bo"])
        x = tF.layer_norm(x + y, (c.d_model,), f(L["ln1_g"]), f(L["ln1_b"]), c.eps)
        hh = ref.gelu_tanh(x @ f(L["w1"]).t() + f(L["b1"]))
        x = tF.layer_norm(x + hh @ f(L["w2"]).t() + f(L["b2"]), (c.d_model,), f(L["ln2_g"]), f(L["ln2_b"]), c.eps)
    return x


def vit_ref(m, img):
    c = m.cfg
    f = lambda t: t.float()  # noqa: E731
    x = torch.cat([f(m.cls), f(m.reg), m.patchify(img).float() @ f(m.patch_w).t() + f(m.patch_b)])
    H, D = c.n_heads, c.d // c.n_heads
    npre = 1 + c.n_reg
    for L in m.layers:
        h = tF.layer_norm(x, (c.d,), f(L["n1_g"]), f(L["n1_b"]), c.eps)
        qkv = h @ f(L["wqkv"]).t()
        qkv[npre:] = ref.rope(qkv[npre:], m.patch_pos, m.cos, m.sin, 2 * H, D)
        q, k, v = (qkv[:, i * c.d : (i + 1) * c.d].view(-1, H, D).transpose(0, 1) for i in range(3))
        a = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(D), -1) @ v
        x = x + a.transpose(0, 1).reshape(-1, c.d) @ f(L["wo"]).t() + f(L["bo"])
        h = tF.layer_norm(x, (c.d,), f(L["n2_g"]), f(L["n2_b"]), c.eps)
        x = x + ref.gelu_tanh(h @ f(L["w1"]).t() + f(L["b1"])) @ f(L["w2"]).t() + f(L["b2"])
    return tF.layer_norm(x, (c.d,), f(m.norm_g), f(m.norm_b), c.eps)


def cos(a, b):
    return float(tF.cosine_similarity(a.float().reshape(-1), b.float().reshape(-1), dim=0))


def test_bert_cpu_matches_reference():
    m = BertEncoder(BERT, device="cpu", seed=1)
    ids = torch.randint(0, 500, (20,), generator=torch.Generator().manual_seed(0))
    assert cos(m.hidden(ids), bert_ref(m, ids)) > 0.999
    e = m.embed(ids)
    assert abs(float(e.norm()) - 1.0) < 1e-4


def test_vit_cpu_matches_reference():
    m = VitEncoder(VIT, device="cpu", seed=2)
    img = torch.randn(3, 32, 32, generator=torch.Generator().manual_seed(0))
    assert m.forward(img).shape == (VIT.seq, VIT.d)
    assert cos(m.forward(img), vit_ref(m, img)) > 0.999


@pytest.mark.gpu
def test_encoders_gpu_match_cpu():
    ids = torch.randint(0, 500, (40,), generator=torch.Generator().manual_seed(3))
    bg, bc = BertEncoder(BERT, device="cuda", seed=4), BertEncoder(BERT, device="cpu", seed=4)
    assert cos(bg.hidden(ids).cpu(), bc.hidden(ids)) > 0.995
    img = torch.randn(3, 32, 32, generator=torch.Generator().manual_seed(5))
    vg, vc = VitEncoder(VIT, device="cuda", seed=6), VitEncoder(VIT, device="cpu", seed=6)
    assert cos(vg.forward(img).cpu(), vc.forward(img)) > 0.995
