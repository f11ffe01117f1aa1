"""Fused GPU kernels for tgc's attention and normalisation analyses against the oracle's
restatements (which equal tgc's outputs bit for bit). Tolerances: attention 2e-5 of the
largest output (fp32 dot products and softmax sums in another order); normalisations rtol
1e-5, atol 1e-5 (row and column means in the kernels' declared orders, not ATen's)."""

from __future__ import annotations

import pytest
import torch

from oracle import analysis as oa
from tgcb import attention, normalisation
from tgcb.errors import ConfigError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("s,w,blk,seed,scale", [
    (256, 64, 128, 0, 1.0), (300, 32, 50, 1, 1.0), (192, 128, 64, 2, 1.0), (200, 16, 7, 3, 8.0),
    (1000, 64, 128, 4, 1.0), (33, 64, 128, 5, 4.0), (2048, 128, 128, 6, 1.0),
])
def test_streaming_attention(cuda, s, w, blk, seed, scale):
    q, k, v = oa.random_head(s, w, seed=seed, scale=scale)
    ref = oa.streaming_attention(q, k, v, blk)
    got = attention.streaming_attention(q.cuda(), k.cuda(), v.cuda(), blk).cpu()
    assert torch.isfinite(got).all()
    assert float((got - ref).abs().max()) <= 2e-5 * float(ref.abs().max())


@pytest.mark.parametrize("s,sk,w", [(1000, 777, 64), (96, 4099, 128), (33, 65, 64)])
def test_vector_attention_kernel_equals_the_scalar_one(cuda, s, sk, w):
    """Widths 64 and 128 run the 16-byte-operand kernel; an output buffer that is not 16-byte
    aligned takes the scalar kernel instead. Both add in the same order, so they agree bit for
    bit."""
    g = torch.Generator().manual_seed(s + sk)
    q, k, v = (torch.randn(n, w, generator=g).cuda() for n in (s, sk, sk))
    aligned = torch.empty(s, w, device="cuda")
    backing = torch.empty(s * w + 1, device="cuda")
    shifted = backing[1:].view(s, w)  # 4 bytes past a 16-byte boundary
    assert shifted.data_ptr() % 16 != 0
    attention.streaming_attention_into(q, k, v, aligned)
    attention.streaming_attention_into(q, k, v, shifted)
    torch.cuda.synchronize()
    assert torch.equal(aligned, shifted)
    ref = oa.naive_attention(q.cpu(), k.cpu(), v.cpu())
    assert float((aligned.cpu() - ref).abs().max()) <= 2e-5 * float(ref.abs().max())


def test_attention_with_other_key_count(cuda):
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(n, 32, generator=g) for n in (70, 500, 500))
    out = torch.empty(70, 32, device="cuda")
    attention.streaming_attention_into(q.cuda(), k.cuda(), v.cuda(), out)
    ref = oa.naive_attention(q, k, v)
    assert float((out.cpu() - ref).abs().max()) <= 2e-5 * float(ref.abs().max())


def test_attention_checks(cuda):
    x = torch.ones(8, 24, device="cuda")
    with pytest.raises(ConfigError, match="widths"):
        attention.streaming_attention(x, x, x)
    with pytest.raises(ConfigError, match="block"):
        attention.streaming_attention(x, x, x, block=0)


@pytest.mark.parametrize("rows,width,offset", [(48, 512, 0.5), (37, 300, 0.0), (4096, 1024, 0.0), (3, 5000, 2.0)])
def test_normalisations(cuda, rows, width, offset):
    x, _, _ = oa.random_rows(rows, width, seed=rows, offset=offset)
    g = torch.Generator().manual_seed(width)
    gain, shift = torch.rand(width, generator=g) + 0.5, torch.randn(width, generator=g)
    mean, var = torch.randn(width, generator=g), torch.rand(width, generator=g) + 0.1
    xc, gc, sc = x.cuda(), gain.cuda(), shift.cuda()
    tol = {"rtol": 1e-5, "atol": 1e-5}
    torch.testing.assert_close(normalisation.layer_norm(xc, gc, sc).cpu(), oa.layer_norm(x, gain, shift), **tol)
    torch.testing.assert_close(normalisation.rms_norm(xc, gc).cpu(), oa.rms_norm(x, gain), **tol)
    torch.testing.assert_close(normalisation.batch_norm(xc, gc, sc).cpu(), oa.batch_norm(x, gain, shift), **tol)
    torch.testing.assert_close(
        normalisation.batch_norm(xc, gc, sc, running=(mean.cuda(), var.cuda())).cpu(),
        oa.batch_norm(x, gain, shift, running=(mean, var)), **tol,
    )
