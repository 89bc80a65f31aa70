"""GPU parity of decode (one query per (batch, head) against a KV cache).

Each case fills a cache with seeded keys and values for the whole sequence,
picks query positions (different ones per batch row), and compares
decode_attention with (a) the oracle's dense-masked softmax of that row in
fp32 under the same mask (oracle.layout for block layouts, the reference's
materialise for M^(d) specs) and (b) the row of the full-sequence forward
kernel.  Keys after the query position are present in the cache and must be
masked out.  Tolerance: bf16 2e-2 max-abs (1e-3 for the LSE), as for the
forward.
"""

import math

import numpy as np
import pytest
import torch

from oracle import layout as OL
from smat_attention_b200.attention import check_device_errors, fwd
from smat_attention_b200.decode import SmatSoftmaxDecoder, decode_attention
from smat_attention_b200.mask import build_block_mask, build_mask, materialise

pytestmark = pytest.mark.gpu


def _qkv(B, H, T, D, seed, device, token_major=False):
    g = torch.Generator().manual_seed(seed)
    if token_major:   # [B, T, H, D] memory seen as [B, H, T, D]: key rows H D apart
        return [torch.randn(B, T, H, D, generator=g).to(device=device, dtype=torch.bfloat16)
                .transpose(1, 2) for _ in range(3)]
    return [torch.randn(B, H, T, D, generator=g).to(device=device, dtype=torch.bfloat16)
            for _ in range(3)]


def _oracle_rows(q, k, v, rows_mask, pos, scale):
    """o, lse of query q[b, :, pos[b]] under mask rows rows_mask(t) -> [T] bool."""
    B, H, T, D = k.shape
    outs, lses = [], []
    for b in range(B):
        t = int(pos[b])
        keep = rows_mask(t).to(q.device)
        s = torch.einsum("hd,hsd->hs", q[b, :, t].float(), k[b].float()) * scale
        s = s.masked_fill(~keep, float("-inf"))
        lse = torch.logsumexp(s, -1)
        outs.append(torch.einsum("hs,hsd->hd", torch.exp(s - lse[:, None]), v[b].float()))
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def _check(spec, rows_mask, B, H, T, D, positions, seed, device, token_major=False):
    q, k, v = _qkv(B, H, T, D, seed, device, token_major)
    scale = 1.0 / math.sqrt(D)
    o_full, lse_full = fwd(q, k, v, spec, scale)
    pos = torch.tensor(positions, dtype=torch.int32, device=device)
    qt = torch.stack([q[b, :, positions[b]] for b in range(B)])
    o, lse = decode_attention(qt, k, v, pos, spec, scale)
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    ro, rlse = _oracle_rows(q, k, v, rows_mask, positions, scale)
    err = (o.float() - ro).abs().max().item()
    err_lse = (lse - rlse).abs().max().item()
    full = torch.stack([o_full[b, :, positions[b]] for b in range(B)]).float()
    err_full = (o.float() - full).abs().max().item()
    print(f"T={T} D={D} pos={positions}: vs oracle {err:.2e} (lse {err_lse:.2e}), "
          f"vs forward kernel {err_full:.2e}")
    assert err <= 2e-2 and err_lse <= 1e-3 and err_full <= 2e-2


@pytest.mark.parametrize("T,lay,D,positions", [
    (1024, (64, 4, 0, 1), 64, [0, 1023]),
    (1024, (64, 4, 0, 1), 128, [63, 64]),
    (4096, (64, 8, 16, 1), 64, [4095, 2500]),
    (16384, (128, 4, 8, 2), 128, [16383, 9000]),
    (1000, (128, 2, 3, 2), 128, [999, 500]),
])
def test_block_layout(cuda_device, T, lay, D, positions):
    spec = build_block_mask(T, *lay)
    rows = OL.block_mask_rows(T, *lay)       # the oracle's mask rows (naive tile rule)
    dense = lambda t: rows(t, t + 1)[0].cpu()
    _check(spec, dense, len(positions), 2, T, D, positions, seed=T + D, device=cuda_device)


@pytest.mark.parametrize("T,d,chunk,D,positions", [
    (2048, 3, 64, 64, [2047, 1100]),     # recent rows: long-range pattern
    (2048, 3, 64, 128, [300, 1023]),     # landmark rows
    (1024, 10, 64, 64, [1000, 511]),     # endpoint family
    (16384, 3, 128, 128, [16383, 8200]),
])
def test_md_mask(cuda_device, T, d, chunk, D, positions):
    spec = build_mask(T, d, chunk=chunk)
    M = materialise(spec, np.uint8)
    _check(spec, lambda t: torch.from_numpy(M[t].astype(bool)), len(positions), 2, T, D,
           positions, seed=T + d, device=cuda_device)


@pytest.mark.parametrize("D", [64, 128])
def test_token_major_cache(cuda_device, D):
    """Caches whose key rows are not contiguous (the copies go row by row)."""
    T, lay = 2048, (128, 4, 4, 1)
    spec = build_block_mask(T, *lay)
    rows = OL.block_mask_rows(T, *lay)
    dense = lambda t: rows(t, t + 1)[0].cpu()
    _check(spec, dense, 2, 3, T, D, [2047, 1300], seed=D, device=cuda_device, token_major=True)


def test_decoder_steps(cuda_device):
    """SmatSoftmaxDecoder: prefill then token by token equals the forward."""
    T, D, B, H = 512, 64, 2, 3
    spec = build_block_mask(T, 64, 2, 3, 1)
    q, k, v = _qkv(B, H, T, D, 7, cuda_device)
    o_full, _ = fwd(q, k, v, spec, 1 / 8)
    dec = SmatSoftmaxDecoder(spec, B, H, D, device=cuda_device)
    dec.prefill(k[:, :, :300], v[:, :, :300])
    for t in range(300, 340):
        o = dec.step(q[:, :, t], k[:, :, t], v[:, :, t])
        assert (o.float() - o_full[:, :, t].float()).abs().max().item() <= 2e-2, t
    assert dec.cache_words() == 2 * B * H * T * D
    torch.cuda.synchronize()
    assert check_device_errors() == 0


def test_bad_position_flagged(cuda_device):
    T, D = 256, 64
    spec = build_block_mask(T, 64, 2, 0, 1)
    q, k, v = _qkv(1, 1, T, D, 0, cuda_device)
    pos = torch.tensor([T], dtype=torch.int32, device=cuda_device)
    o, _ = decode_attention(q[:, :, 0], k, v, pos, spec)
    torch.cuda.synchronize()
    assert check_device_errors() & 8
    assert o.float().abs().max().item() == 0.0
