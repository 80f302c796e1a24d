"""The decode layer's projection GEMM (b2_gemm: tcgen05 tensor cores, TMEM
accumulators, cluster split-K) against torch references.

The plain product accumulates in fp32 like cuBLAS does, so its bf16 result is
compared with the fp32 product of the same bf16 operands rounded once to
bf16: every element within 1 bf16 ulp, and all but a few exact (a different
fp32 summation order can move a value across a rounding boundary).  The
SwiGLU epilogue is compared with b2_swiglu applied to that rounded product.
"""
import numpy as np
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu


def _block():
    return load_pkg("block")


def _lib():
    return load_pkg("_lib")


def ulps(a: torch.Tensor, b: torch.Tensor) -> np.ndarray:
    """Distance in bf16 ulps (sign-magnitude order) between two bf16 tensors."""
    def key(t):
        u = t.contiguous().view(torch.int16).cpu().numpy().astype(np.int32) & 0xFFFF
        return np.where(u & 0x8000, 0x8000 - (u & 0x7FFF), 0x8000 + u)
    return np.abs(key(a) - key(b))


def operands(m, n, k, seed, dev, rows_w=None):
    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(rows_w or n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return a, w


def check_product(got, a, w, what, exact_frac=0.999):
    ref = (a.float() @ w.float().t()).to(torch.bfloat16)
    d = ulps(got, ref)
    assert d.max() <= 1, f"{what}: {int((d > 1).sum())} elements beyond 1 ulp (max {d.max()})"
    assert (d == 0).mean() >= exact_frac, f"{what}: only {(d == 0).mean():.5f} exact"


@pytest.mark.parametrize("m,n,k", [(256, 1024, 1024), (256, 2048, 1024), (256, 3072, 1024), (256, 1024, 2560),
                                   (1, 1024, 1024), (16, 2048, 1024), (100, 512, 256), (300, 256, 128),
                                   (256, 8192, 1024)])
def test_gemm_matches_fp32_product(cuda, m, n, k):
    blk = _block()
    a, w = operands(m, n, k, m + n + k, cuda)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    blk.gemm(a, w, out=out, dev_err=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    check_product(out, a, w, f"{m}x{n}x{k} plan {blk.gemm_plan(m, n, k)}")


@pytest.mark.parametrize("tile_n", [16, 32, 64, 128])
@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_gemm_tilings_agree(cuda, tile_n, splits):
    """Every tile width and K split gives a deterministic result within the
    fp32-product bound; 4 M tiles, the last one partial."""
    blk = _block()
    m, n, k = 450, 256, 1024
    a, w = operands(m, n, k, 7, cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = []
    for _ in range(2):
        out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        blk.gemm(a, w, out=out, dev_err=err, tile_n=tile_n, splits=splits)
        outs.append(out)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.equal(outs[0], outs[1])
    check_product(outs[0], a, w, f"tile_n {tile_n} splits {splits}")


@pytest.mark.parametrize("m,ffn", [(256, 2560), (7, 512), (256, 64)])
def test_gemm_swiglu_epilogue(cuda, m, ffn):
    blk = _block()
    k = 1024
    a, w13 = operands(m, ffn, k, 11 + m, cuda, rows_w=2 * ffn)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty(m, ffn, dtype=torch.bfloat16, device=cuda)
    blk.gemm(a, w13, out=out, dev_err=err, swiglu=True)
    gu = (a.float() @ w13.float().t()).to(torch.bfloat16)
    ref = torch.empty(m, ffn, dtype=torch.bfloat16, device=cuda)
    blk.swiglu(gu, out=ref)
    torch.cuda.synchronize()
    assert err.item() == 0
    d = ulps(out, ref)
    assert d.max() <= 2 and (d == 0).mean() >= 0.995, f"max {d.max()} ulps, exact {(d == 0).mean():.5f}"


def test_gemm_strided_rows_and_column_slices(cuda):
    """A row-strided A (columns of a wider buffer) and an output written into
    the left part of a wider buffer, as the runner slices its buffers."""
    blk = _block()
    m, n, k = 64, 512, 1024
    big_a, w = operands(m, n, 2 * k, 21, cuda, rows_w=n)
    a = big_a[:, k:]                       # row stride 2k
    w = w[:, :k].contiguous()
    wide = torch.zeros(m, n + 64, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    blk.gemm(a, w, out=wide[:, :n], dev_err=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    check_product(wide[:, :n], a, w, "strided")
    assert (wide[:, n:] == 0).all()


def test_gemm_refuses_bad_arguments(cuda):
    blk, lib = _block(), _lib()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    a, w = operands(8, 64, 96, 1, cuda)
    with pytest.raises(lib.B2Error):                                  # k not a multiple of 64
        blk.gemm(a, w, out=torch.empty(8, 64, dtype=torch.bfloat16, device=cuda), dev_err=err)
    a, w = operands(8, 64, 128, 1, cuda)
    with pytest.raises(lib.B2Error):                                  # tile_n not dividing n
        blk.gemm(a, w, out=torch.empty(8, 64, dtype=torch.bfloat16, device=cuda), dev_err=err, tile_n=48)
    with pytest.raises(lib.B2Error):                                  # splits not dividing k / 64
        blk.gemm(a, w, out=torch.empty(8, 64, dtype=torch.bfloat16, device=cuda), dev_err=err, splits=4)
    with pytest.raises(ValueError):
        blk.gemm(a, w, out=torch.empty(8, 32, dtype=torch.bfloat16, device=cuda), dev_err=err)
    torch.cuda.synchronize()
    assert err.item() == 0


def test_gemm_in_a_cuda_graph(cuda):
    """Captured with programmatic dependent launch after a kernel that writes
    A: the product sees the new A on every replay."""
    blk = _block()
    m, n, k = 256, 1024, 1024
    a, w = operands(m, n, k, 31, cuda)
    src = torch.zeros_like(a)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        a.copy_(src)
        blk.gemm(a, w, out=out, dev_err=err)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        a.copy_(src)
        blk.gemm(a, w, out=out, dev_err=err)
    for seed in (1, 2):
        src.copy_(torch.randn(m, k, generator=torch.Generator(device=cuda).manual_seed(seed), device=cuda))
        graph.replay()
        torch.cuda.synchronize()
        check_product(out, src, w, f"replay {seed}")
    assert err.item() == 0
