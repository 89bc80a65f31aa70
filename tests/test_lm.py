"""The LM of BASELINE config 4 without a GPU: its parameter count and shapes,
and the fp32-master AdamW against torch's AdamW on fp32 copies (the fused
kernels and the attention op need a GPU and are covered by test_gpu_lm.py)."""

import torch

from smat_attention_b200.lm import C4, LM, LMConfig, MasterAdamW, Rotary
from smat_attention_b200.mask import block_layout_stats


def test_c4_shapes():
    cfg = C4
    assert (cfg.vocab, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.head_dim, cfg.mlp_hidden,
            cfg.seq_len) == (32000, 768, 12, 12, 64, 2048, 8192)
    spec = cfg.mask()
    assert (spec.block, spec.window, spec.stride, spec.n_sink) == (64, 8, 16, 1)
    # BASELINE: 6,406,144 unmasked pairs per head and layer
    assert block_layout_stats(spec)["pairs"] == 6406144


def test_param_count_matches_modules():
    cfg = LMConfig(vocab=1000, d_model=256, n_layers=3, n_heads=4, mlp_hidden=512, seq_len=256)
    model = LM(cfg, device="cpu")
    assert sum(p.numel() for p in model.parameters()) == cfg.n_params()
    assert all(p.dtype == torch.bfloat16 for p in model.parameters())
    # init N(0, 0.02) on matrices, ones on the norm scales
    w = model.blocks[0].attn.qkv.weight.float()
    assert abs(w.std().item() - 0.02) < 2e-3
    assert torch.equal(model.norm.w.float(), torch.ones(256))


def test_rotary_tables():
    rot = Rotary(64)
    cos, sin = rot.tables(16, "cpu")
    assert cos.shape == (16, 32)
    t, i = 5, 3
    ang = t / 10000 ** (2 * i / 64)
    assert abs(cos[t, i].item() - torch.cos(torch.tensor(ang)).item()) < 1e-6
    # the rotation preserves pair norms and is undone by the negative angle
    x = torch.randn(2, 16, 64)
    y = Rotary.rotate(x, cos, sin)
    assert torch.allclose(Rotary.rotate(y, cos, -sin), x, atol=1e-5)
    assert torch.allclose(y.pow(2).sum(-1), x.pow(2).sum(-1), atol=1e-4)


def test_master_adamw_cpu():
    torch.manual_seed(0)
    p = torch.nn.Parameter(torch.randn(8, 4).to(torch.bfloat16))
    s = torch.nn.Parameter(torch.ones(4, dtype=torch.bfloat16))
    opt = MasterAdamW([p, s], lr=1e-2, clip=1.0)
    rp = p.detach().float().clone().requires_grad_(True)
    rs = s.detach().float().clone().requires_grad_(True)
    ref = torch.optim.AdamW([{"params": [rp], "weight_decay": 0.1},
                             {"params": [rs], "weight_decay": 0.0}], lr=1e-2, betas=(0.9, 0.95))
    for _ in range(4):
        gp, gs = torch.randn(8, 4).to(torch.bfloat16), torch.randn(4).to(torch.bfloat16)
        p.grad, s.grad = gp, gs
        rp.grad, rs.grad = gp.float(), gs.float()
        torch.nn.utils.clip_grad_norm_([rp, rs], 1.0)
        norm = opt.step()
        ref.step()
        assert norm.item() > 0
        assert torch.allclose(opt.master[0], rp, atol=1e-6)
        assert torch.allclose(opt.master[1], rs, atol=1e-6)
        assert torch.equal(p.detach(), rp.detach().to(torch.bfloat16))


def _dp_worker(rank, world, port):
    import datetime
    import os

    import torch.distributed as dist

    from smat_attention_b200.lm import allreduce_grads
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        m = torch.nn.Sequential(torch.nn.Linear(4, 3), torch.nn.Linear(3, 2, bias=False))
        for i, p in enumerate(m.parameters()):
            p.grad = torch.full_like(p, float(rank + 1) * (i + 1))
        allreduce_grads(m, dist)
        for i, p in enumerate(m.parameters()):
            want = (i + 1) * sum(r + 1 for r in range(world)) / world
            assert torch.allclose(p.grad, torch.full_like(p, want)), (i, p.grad)
    finally:
        dist.destroy_process_group()


def test_allreduce_grads_gloo():
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_dp_worker, args=(3, port), nprocs=3, join=True)
