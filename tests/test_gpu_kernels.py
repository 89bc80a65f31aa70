"""GPU parity of the sm_100a kernels against the oracle.

Every case draws seeded inputs on the CPU, runs the kernels through the C ABI
(smat_attention_b200.attention.fwd / bwd), and compares with the oracle's
dense-masked computation (oracle.dense_softmax.rowchunked_masked_softmax,
which visits every (i, j) pair) evaluated in fp32 on the same, already
rounded, inputs.  Tolerances (max-abs): bf16 outputs 2e-2 for O, dQ, dK, dV
and 1e-3 for the fp32 LSE; the fp32 path 1e-4 for everything.
"""

import math

import pytest
import torch

from oracle import layout as OL
from oracle.dense_softmax import rowchunked_masked_softmax
from smat_attention_b200.attention import bwd, check_device_errors, fwd, smat_softmax_attention
from smat_attention_b200.mask import build_block_mask

pytestmark = pytest.mark.gpu

TOL_BF16, TOL_BF16_LSE, TOL_F32 = 2e-2, 1e-3, 1e-4


def _inputs(B, H, T, D, dtype, seed, scale_in, device):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(B, H, T, D, generator=g) * scale_in).to(device=device, dtype=dtype)
            for _ in range(4)]


def _reference(q, k, v, do, lay, backward, rows=512):
    B, H, T, D = q.shape
    f = lambda x: x.float().reshape(B * H, T, D)
    out = rowchunked_masked_softmax(f(q), f(k), f(v), f(do),
                                    OL.block_mask_rows(T, *lay, device=q.device),
                                    1.0 / math.sqrt(D), rows=rows, backward=backward)
    shape = lambda x: None if x is None else x.reshape(B, H, T, -1).squeeze(-1)
    return [shape(x) for x in out]


def _maxerr(a, b):
    return (a.float() - b.float()).abs().max().item()


def _run_case(B, H, T, D, lay, dtype, seed=0, scale_in=1.0, backward=True, device="cuda"):
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(B, H, T, D, dtype, seed, scale_in, device)
    scale = 1.0 / math.sqrt(D)
    o, lse = fwd(q, k, v, spec, scale)
    grads = bwd(q, k, v, o, lse, do, spec, scale) if backward else None
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    ro, rlse, rdq, rdk, rdv = _reference(q, k, v, do, lay, backward)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    tol_lse = TOL_F32 if dtype == torch.float32 else TOL_BF16_LSE
    errs = {"o": _maxerr(o, ro), "lse": _maxerr(lse, rlse)}
    if backward:
        for name, got, ref in zip(("dq", "dk", "dv"), grads, (rdq, rdk, rdv)):
            errs[name] = _maxerr(got, ref)
    print(f"B={B} H={H} T={T} D={D} lay={lay} {dtype}: " +
          " ".join(f"{k}={v:.2e}" for k, v in errs.items()))
    for name, e in errs.items():
        assert e <= (tol_lse if name == "lse" else tol), (name, e, errs)
    for t in (o, lse) + (tuple(grads) if grads else ()):
        assert torch.isfinite(t).all()
    return errs


SMALL = [  # (T, (bs, W, S, sinks))
    (128, (64, 0, 0, 0)), (128, (128, 0, 0, 0)), (256, (64, 1, 0, 1)), (256, (128, 1, 0, 1)),
    (640, (64, 2, 3, 1)), (768, (128, 1, 2, 1)), (200, (64, 1, 2, 1)), (1000, (128, 2, 3, 2)),
    (1000, (64, 3, 5, 2)), (512, (64, 0, 1, 0)), (384, (64, 100, 0, 0)),
]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("T,lay", SMALL)
def test_bf16_small(cuda_device, D, T, lay):
    _run_case(2, 2, T, D, lay, torch.bfloat16, seed=T + D)


@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("T,lay", [(256, (16, 2, 3, 1)), (200, (32, 1, 2, 1)),
                                   (384, (64, 1, 0, 1)), (300, (128, 1, 1, 1)),
                                   (100, (7, 3, 4, 2))])
def test_fp32_small(cuda_device, D, T, lay):
    _run_case(2, 2, T, D, lay, torch.float32, seed=T + D)


def test_c1_fp32_full(cuda_device):
    """B=1 H=4 T=1024 D=64 bs=64, W=4, sink 1, fp32 fwd+bwd, seed 0."""
    _run_case(1, 4, 1024, 64, (64, 4, 0, 1), torch.float32, seed=0)


def test_c2_bf16_fwd_full(cuda_device):
    """B=8 H=16 T=4096 D=64 bs=64, W=8, S=16, sink 1, inputs 0.5 N(0,1)."""
    _run_case(8, 16, 4096, 64, (64, 8, 16, 1), torch.bfloat16, seed=1, scale_in=0.5,
              backward=False)


def test_c3_bf16_full(cuda_device):
    """B=4 H=32 T=16384 D=128 bs=128, W=4, S=8, 2 sinks, fwd+bwd."""
    _run_case(4, 32, 16384, 128, (128, 4, 8, 2), torch.bfloat16, seed=2)


def test_c5_bf16_head_slice(cuda_device):
    """BASELINE config 5 shapes on 2 of its 32 heads: T=131072 D=128 bs=128, W=8,
    S=32, 4 sinks, fwd+bwd."""
    _run_case(1, 2, 131072, 128, (128, 8, 32, 4), torch.bfloat16, seed=4)


def test_c4_attention_shapes(cuda_device):
    """BASELINE config 4's attention: batch 8 x 12 heads, T=8192, D=64, bs=64,
    W=8, S=16, sink 1 (on 2 of the 8 sequences)."""
    _run_case(2, 12, 8192, 64, (64, 8, 16, 1), torch.bfloat16, seed=3, scale_in=1.0)


@pytest.mark.parametrize("dtype,bs", [(torch.bfloat16, 64), (torch.bfloat16, 128),
                                      (torch.float32, 64)])
def test_exact_noninfluence(cuda_device, dtype, bs):
    """Perturbing a key/value the mask hides from row i leaves row i's O and
    LSE bit-identical (reference property test_smat.py:292-324)."""
    T, lay = 768, (bs, 1, 3, 1)
    spec = build_block_mask(T, *lay)
    M = torch.from_numpy(OL.dense_mask(T, *lay)).cuda().bool()
    q, k, v, _ = _inputs(1, 2, T, 64, dtype, 11, 1.0, "cuda")
    o0, l0 = fwd(q, k, v, spec, 0.125)
    g = torch.Generator().manual_seed(5)
    for j in (bs - 1, bs + 3, 3 * bs + 7, T - bs - 2):
        k2, v2 = k.clone(), v.clone()
        k2[:, :, j] = (torch.randn(2, 64, generator=g) * 3).to(k2)
        v2[:, :, j] = (torch.randn(2, 64, generator=g) * 3).to(v2)
        o1, l1 = fwd(q, k2, v2, spec, 0.125)
        excl = ~M[:, j]
        assert excl.any()
        assert torch.equal(o1[:, :, excl], o0[:, :, excl]), j
        assert torch.equal(l1[:, :, excl], l0[:, :, excl]), j
    assert check_device_errors() == 0


def test_autograd_matches_direct_calls(cuda_device):
    T, lay = 512, (64, 2, 3, 1)
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(2, 3, T, 64, torch.bfloat16, 21, 1.0, "cuda")
    qa, ka, va = (x.clone().requires_grad_(True) for x in (q, k, v))
    o, lse = smat_softmax_attention(qa, ka, va, spec)
    o.backward(do)
    o2, lse2 = fwd(q, k, v, spec, 1 / 8)
    dq, dk, dv = bwd(q, k, v, o2, lse2, do, spec, 1 / 8)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    assert torch.equal(qa.grad, dq) and torch.equal(ka.grad, dk) and torch.equal(va.grad, dv)
    assert not lse.requires_grad


def test_strided_views(cuda_device):
    """q/k/v as views of a fused [B, T, 3, H, D] projection and O written
    through a permuted view give the same result as contiguous tensors."""
    B, T, H, D = 2, 384, 4, 64
    spec = build_block_mask(T, 64, 2, 3, 1)
    g = torch.Generator().manual_seed(9)
    qkv = torch.randn(B, T, 3, H, D, generator=g).to("cuda", torch.bfloat16)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
    o_bthd = torch.empty(B, T, H, D, device="cuda", dtype=torch.bfloat16)
    o, lse = fwd(q, k, v, spec, 0.125, o=o_bthd.transpose(1, 2))
    oc, lc = fwd(q.contiguous(), k.contiguous(), v.contiguous(), spec, 0.125)
    assert torch.equal(o_bthd.transpose(1, 2), oc) and torch.equal(lse, lc)


def test_rejects_unsupported(cuda_device):
    spec = build_block_mask(256, 64, 1, 0, 1)
    q = torch.randn(1, 1, 256, 64, device="cuda", dtype=torch.float64)
    with pytest.raises(TypeError):
        fwd(q, q, q, spec, 0.125)          # fp64 is never routed to the kernels
    with pytest.raises(ValueError):
        fwd(q.float().cpu(), q.float().cpu(), q.float().cpu(), spec, 0.125)
    qb = torch.randn(1, 1, 256, 96, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        fwd(qb, qb, qb, spec, 0.1)          # D = 96 unsupported on the bf16 path
    with pytest.raises(ValueError):
        fwd(qb[..., :64].contiguous()[:, :, :128], qb[..., :64].contiguous()[:, :, :128],
            qb[..., :64].contiguous()[:, :, :128], spec, 0.125)   # T mismatch


def test_fp32_matches_reference_c1_head(cuda_device):
    """Config 1 in full size on the fp32 path against the reference's own
    dense-masked attention (tests/golden/softmax_c1_t1024.npz, one head,
    T = 1024, D = 64, bs 64, W 4, one sink): O, dQ, dK, dV within 1e-4."""
    import numpy as np
    from test_oracle import c1_fixture
    f, (q, k, v, do), _ = c1_fixture()
    spec = build_block_mask(1024, 64, 4, 0, 1)
    dev = [x.reshape(1, 1, 1024, 64).to(cuda_device) for x in (q, k, v, do)]
    o, lse = fwd(dev[0], dev[1], dev[2], spec, float(f["scale"]))
    dq, dk, dv = bwd(dev[0], dev[1], dev[2], o, lse, dev[3], spec, float(f["scale"]))
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    for got, key in ((o, "o"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        err = np.abs(got.reshape(1, 1024, 64).cpu().double().numpy() - f[key]).max()
        assert err <= TOL_F32, (key, err)
