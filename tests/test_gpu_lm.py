"""GPU checks of the LM training step (BASELINE config 4's model).

The fused kernels of csrc/lm_ops.cu against the plain torch forms of the same
formulas (the reference LM template's RMSNorm and RoPE, tasks/lm.py:45-60,
plus SwiGLU and cross-entropy), forward and gradients; the whole model fused
against plain; and a short training run whose loss must fall.  bf16
tolerances are relative to each tensor's largest entry (both sides round to
bf16 at different points).
"""

import math

import pytest
import torch
import torch.nn.functional as F

from smat_attention_b200 import lm_ops
from smat_attention_b200.attention import check_device_errors
from smat_attention_b200.lm import LM, LMConfig, MasterAdamW, Rotary, train_step

pytestmark = pytest.mark.gpu


def _close(a, b, rel, name):
    scale = b.float().abs().max().item() + 1e-6
    err = (a.float() - b.float()).abs().max().item()
    assert err <= rel * scale, (name, err, scale)


def _rand(*shape, device, seed, scale=1.0, grad=True):
    g = torch.Generator().manual_seed(seed)
    t = (torch.randn(*shape, generator=g) * scale).to(device=device, dtype=torch.bfloat16)
    return t.requires_grad_(grad)


@pytest.mark.parametrize("shape", [(4, 100, 768), (3, 256), (2, 7, 1536), (5, 512)])
def test_rms_norm(cuda_device, shape):
    d = shape[-1]
    x = _rand(*shape, device=cuda_device, seed=d)
    w = _rand(d, device=cuda_device, seed=d + 1)
    dy = _rand(*shape, device=cuda_device, seed=d + 2, grad=False)
    y = lm_ops.rms_norm(x, w, 1e-5)
    (y.float() * dy.float()).sum().backward()
    gx, gw = x.grad.clone(), w.grad.clone()
    x.grad = w.grad = None
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    (ref * dy.float()).sum().backward()
    _close(y, ref, 1e-2, "y")
    _close(gx, x.grad, 2e-2, "dx")
    _close(gw, w.grad, 2e-2, "dw")


@pytest.mark.parametrize("shape", [(4, 100, 768), (5, 512)])
def test_add_rms_norm(cuda_device, shape):
    d = shape[-1]
    x = _rand(*shape, device=cuda_device, seed=d)
    r = _rand(*shape, device=cuda_device, seed=d + 1)
    w = _rand(d, device=cuda_device, seed=d + 2)
    dh = _rand(*shape, device=cuda_device, seed=d + 3, grad=False)
    dy = _rand(*shape, device=cuda_device, seed=d + 4, grad=False)
    h, y = lm_ops.add_rms_norm(x, r, w, 1e-5)
    ((h.float() * dh.float()).sum() + (y.float() * dy.float()).sum()).backward()
    got = [t.grad.clone() for t in (x, r, w)]
    for t in (x, r, w):
        t.grad = None
    hr = x + r
    hf = hr.float()
    yr = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    ((hr.float() * dh.float()).sum() + (yr * dy.float()).sum()).backward()
    assert torch.equal(h, hr)
    _close(y, yr, 1e-2, "y")
    for g, t, n in zip(got, (x, r, w), "xrw"):
        _close(g, t.grad, 2e-2, "d" + n)


@pytest.mark.parametrize("B,T,H,D", [(2, 256, 4, 64), (1, 100, 3, 128), (2, 64, 12, 64)])
def test_rope_split(cuda_device, B, T, H, D):
    qkv = _rand(B, T, 3, H, D, device=cuda_device, seed=T)
    rot = Rotary(D)
    cos, sin = rot.tables(T, cuda_device)
    q, k, v = lm_ops.rope_split(qkv, cos, sin)
    grads = [_rand(B, H, T, D, device=cuda_device, seed=T + i, grad=False) for i in range(3)]
    sum((a.float() * g.float()).sum() for a, g in zip((q, k, v), grads)).backward()
    gq = qkv.grad.clone()
    qkv.grad = None
    rq, rk, rv = qkv.permute(2, 0, 3, 1, 4)
    rq, rk = Rotary.rotate(rq, cos, sin), Rotary.rotate(rk, cos, sin)
    sum((a.float() * g.float()).sum() for a, g in zip((rq, rk, rv), grads)).backward()
    for a, b, n in ((q, rq, "q"), (k, rk, "k"), (v, rv, "v")):
        assert a.shape == (B, H, T, D) and a.is_contiguous()
        _close(a, b, 1e-2, n)
    assert torch.equal(v, rv)
    _close(gq, qkv.grad, 1e-2, "dqkv")


@pytest.mark.parametrize("rows,hidden", [(1000, 2048), (37, 64)])
def test_swiglu(cuda_device, rows, hidden):
    a = _rand(rows, 2 * hidden, device=cuda_device, seed=rows, scale=2.0)
    dg = _rand(rows, hidden, device=cuda_device, seed=rows + 1, grad=False)
    g = lm_ops.swiglu(a)
    (g.float() * dg.float()).sum().backward()
    ga = a.grad.clone()
    a.grad = None
    a1, a3 = a.float().chunk(2, dim=-1)
    ref = F.silu(a1) * a3
    (ref * dg.float()).sum().backward()
    _close(g, ref, 1e-2, "g")
    _close(ga, a.grad, 1e-2, "da")


@pytest.mark.parametrize("N,d,V", [(512, 256, 32000), (300, 768, 1000)])
def test_linear_cross_entropy(cuda_device, N, d, V):
    h = _rand(N, d, device=cuda_device, seed=N)
    W = _rand(V, d, device=cuda_device, seed=N + 1, scale=0.05)
    g = torch.Generator().manual_seed(N + 2)
    tgt = torch.randint(0, V, (N,), generator=g).to(cuda_device)
    loss = lm_ops.linear_cross_entropy(h, W, tgt)
    loss.backward()
    gh, gW = h.grad.clone(), W.grad.clone()
    h.grad = W.grad = None
    ref = F.cross_entropy((h @ W.t()).float(), tgt)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 2e-3 * abs(ref.item())
    _close(gh, h.grad, 2e-2, "dh")
    _close(gW, W.grad, 2e-2, "dW")
    torch.cuda.synchronize()
    assert check_device_errors() == 0


SMALL = LMConfig(vocab=2048, d_model=256, n_layers=2, n_heads=4, mlp_hidden=512, seq_len=1024,
                 block=64, window=4, stride=8, n_sink=1)


def _tokens(cfg, B, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab, (B, cfg.seq_len + 1), generator=g).to(device)


def test_model_fused_matches_plain(cuda_device):
    fused = LM(SMALL, device=cuda_device, seed=0, fused=True)
    plain = LM(SMALL, device=cuda_device, seed=0, fused=False)
    tok = _tokens(SMALL, 2, 1, cuda_device)
    lf = fused.loss(tok[:, :-1], tok[:, 1:])
    lp = plain.loss(tok[:, :-1], tok[:, 1:])
    lf.backward()
    lp.backward()
    assert abs(lf.item() - lp.item()) < 1e-2, (lf.item(), lp.item())
    assert abs(lf.item() - math.log(SMALL.vocab)) < 0.1       # N(0, 0.02) init: near uniform
    for (n, a), (_, b) in zip(fused.named_parameters(), plain.named_parameters()):
        _close(a.grad, b.grad, 5e-2, n)


def test_master_adamw_matches_torch(cuda_device):
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(64, 32, device=cuda_device).to(torch.bfloat16))
    s = torch.nn.Parameter(torch.ones(32, device=cuda_device, dtype=torch.bfloat16))
    opt = MasterAdamW([p, s], lr=1e-2, clip=None)
    ref_p = p.detach().float().clone().requires_grad_(True)
    ref_s = s.detach().float().clone().requires_grad_(True)
    ref = torch.optim.AdamW([{"params": [ref_p], "weight_decay": 0.1},
                             {"params": [ref_s], "weight_decay": 0.0}],
                            lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    for i in range(5):
        gp = torch.randn(64, 32, device=cuda_device).to(torch.bfloat16)
        gs = torch.randn(32, device=cuda_device).to(torch.bfloat16)
        p.grad, s.grad = gp.clone(), gs.clone()
        ref_p.grad, ref_s.grad = gp.float(), gs.float()
        opt.step()
        ref.step()
        assert torch.allclose(opt.master[0], ref_p, atol=1e-6)
        assert torch.allclose(opt.master[1], ref_s, atol=1e-6)
        assert torch.equal(p.detach(), ref_p.detach().to(torch.bfloat16))
        assert p.grad is None


def test_training_reduces_loss(cuda_device):
    model = LM(SMALL, device=cuda_device, seed=0)
    opt = MasterAdamW(model.parameters(), lr=3e-3)
    tok = _tokens(SMALL, 2, 5, cuda_device)
    losses = [train_step(model, opt, tok).item() for _ in range(30)]
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    assert all(math.isfinite(x) for x in losses)
    assert losses[-1] < losses[0] - 1.0, losses
