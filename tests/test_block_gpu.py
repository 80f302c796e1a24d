"""The layer kernels around the attention path (include/b2_block.h) against
the same operations written in torch, in the order of the model definition
(transformers modeling_lfm2.py: Lfm2RMSNorm 59-64, Lfm2MLP 135-152,
Lfm2ShortConv.slow_forward 356-387, the decoder layer's residual adds
413-442).  The RMSNorm is bit-exact against torch on the CPU (the
reference's path) for widths that are a multiple of 32 (its mean is summed
in torch's CPU order); other bf16 results within one bf16 ulp and at least
99 % bit-exact (exp and GPU reductions in other orders than torch's); the
convolution state bit-exact."""
import numpy as np
import pytest
import torch

from conftest import load_pkg
from test_kernels_gpu import ulp_diff

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _close(got, ref, name):
    d = ulp_diff(got, ref)
    assert d.max() <= 1, f"{name}: {d.max()} ulps"
    assert (d == 0).mean() >= 0.99, f"{name}: exact fraction {(d == 0).mean():.4f}"


def _rms_ref(s, gamma, eps):
    h = s.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return gamma * h.to(BF)


@pytest.mark.parametrize("rows,width", [(1, 1024), (37, 1024), (256, 1024), (3, 4096), (5, 8)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_add_rmsnorm(cuda, rows, width, with_residual):
    blk = load_pkg("block")
    g = torch.Generator(device=cuda).manual_seed(rows * 7 + width)
    x = torch.randn(rows, width, generator=g, device=cuda).to(BF)
    res = torch.randn(rows, width, generator=g, device=cuda).to(BF) if with_residual else None
    gamma = (1 + 0.1 * torch.randn(width, generator=g, device=cuda)).to(BF)
    s_ref = x + res if with_residual else x
    out = torch.empty_like(x)
    sum_out = torch.empty_like(x)
    blk.add_rmsnorm(x, res, gamma, 1e-5, out=out, sum_out=sum_out)
    torch.cuda.synchronize()
    assert torch.equal(sum_out, s_ref)
    ref = _rms_ref(s_ref.cpu(), gamma.cpu(), 1e-5)
    if width % 32 == 0:
        d = ulp_diff(out, ref)
        assert (d == 0).all(), f"rmsnorm: {(d != 0).sum()} of {d.size} elements differ from torch CPU"
    else:
        _close(out, ref, "rmsnorm")


def test_add_rmsnorm_in_place_on_the_residual(cuda):
    blk = load_pkg("block")
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(64, 1024, generator=g, device=cuda).to(BF)
    h = torch.randn(64, 1024, generator=g, device=cuda).to(BF)
    gamma = torch.ones(1024, dtype=BF, device=cuda)
    s_ref = x + h
    out = torch.empty_like(x)
    blk.add_rmsnorm(x, h, gamma, 1e-5, out=out, sum_out=h)
    torch.cuda.synchronize()
    assert torch.equal(h, s_ref)
    assert torch.equal(out.cpu(), _rms_ref(s_ref.cpu(), gamma.cpu(), 1e-5)), "rmsnorm in place"


@pytest.mark.parametrize("rows,ffn", [(1, 2560), (256, 2560), (3, 8)])
def test_swiglu(cuda, rows, ffn):
    blk = load_pkg("block")
    g = torch.Generator(device=cuda).manual_seed(rows + ffn)
    gu = (torch.randn(rows, 2 * ffn, generator=g, device=cuda) * 3).to(BF)
    out = torch.empty(rows, ffn, dtype=BF, device=cuda)
    blk.swiglu(gu, out=out)
    ref = torch.nn.functional.silu(gu[:, :ffn]) * gu[:, ffn:]
    torch.cuda.synchronize()
    _close(out, ref, "swiglu")


@pytest.mark.parametrize("rows", [1, 256])
def test_shortconv_step(cuda, rows):
    blk = load_pkg("block")
    hid = 1024
    g = torch.Generator(device=cuda).manual_seed(rows)
    bcx = torch.randn(rows, 3 * hid, generator=g, device=cuda).to(BF)
    state = torch.randn(rows, hid, 3, generator=g, device=cuda).to(BF)
    w = (0.5 * torch.randn(hid, 3, generator=g, device=cuda)).to(BF)
    bg, cg, xg = bcx.split(hid, dim=-1)
    st_ref = torch.cat([state[..., 1:], (bg * xg)[..., None]], dim=-1)
    ref = cg * torch.sum(st_ref * w, dim=-1)
    out = torch.empty(rows, hid, dtype=BF, device=cuda)
    blk.shortconv_step(bcx, state, w, out=out)
    torch.cuda.synchronize()
    assert torch.equal(state, st_ref)
    _close(out, ref, "shortconv")


def test_block_argument_errors(cuda):
    blk = load_pkg("block")
    x = torch.zeros(2, 1020, dtype=BF, device=cuda)
    with pytest.raises(Exception):
        blk.add_rmsnorm(x, None, torch.ones(1020, dtype=BF, device=cuda), 1e-5, out=torch.empty_like(x))
    with pytest.raises(ValueError):
        blk.swiglu(torch.zeros(2, 7, dtype=BF, device=cuda), out=torch.empty(2, 3, dtype=BF, device=cuda))
    with pytest.raises(ValueError):
        blk.shortconv_step(torch.zeros(2, 3072, dtype=BF, device=cuda), torch.zeros(2, 1024, 2, dtype=BF, device=cuda),
                           torch.zeros(1024, 3, dtype=BF, device=cuda), out=torch.empty(2, 1024, dtype=BF, device=cuda))


@pytest.mark.parametrize("rows,cols", [(1, 65536), (256, 65536), (3, 8), (2, 4096)])
def test_argmax_rows(cuda, rows, cols):
    blk = load_pkg("block")
    g = torch.Generator(device=cuda).manual_seed(rows + cols)
    logits = torch.randn(rows, cols, generator=g, device=cuda).to(BF)
    logits[0, cols // 3] = logits[0].max() + 1      # a clear winner
    if rows > 1:                                    # ties: the first index wins
        logits[1, :] = 0
        logits[1, 5] = logits[1, cols - 1] = 7.0
    if rows > 2:
        logits[2, 2] = float("nan")                 # NaN counts as the maximum
    out = torch.empty(rows, dtype=torch.int64, device=cuda)
    blk.argmax_rows(logits, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, torch.argmax(logits, dim=-1))
