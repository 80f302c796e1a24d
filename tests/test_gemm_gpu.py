"""The decode layer's projection GEMM (b2_gemm: tcgen05 tensor cores, TMEM
accumulators, cluster split-K) against torch references.

The plain product accumulates in fp32 like cuBLAS does.  Every element of its
bf16 result lies within half a bf16 ulp of the exact (fp64) product plus an
fp32 summation bound, 2^-20 x sum |a_i w_i| (this term only matters where the
terms cancel and the result is small next to them), and all but a few equal
the exact product rounded once to bf16 (another fp32 summation order can move
a value across a rounding boundary).  The SwiGLU epilogue carries those
bounds on g = a w1^T and u = a w3^T through silu(g) * u (first-order error
propagation plus the roundings of silu(g) and of the result), and almost all
of it equals b2_swiglu applied to the fp32 products rounded to bf16.
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


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -126))) - 7)


def check_product(got, a, w, what, exact_frac=0.999):
    exact = a.double() @ w.double().t()
    scale = (a.double().abs() @ w.double().abs().t()).cpu().numpy()
    g, e = got.double().cpu().numpy(), exact.cpu().numpy()
    tol = 0.5 * bf16_ulp(np.maximum(np.abs(g), np.abs(e))) + 2.0 ** -20 * scale
    bad = np.abs(g - e) > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond the bound, e.g. got {g[bad][:3]} exact {e[bad][:3]}"
    d = ulps(got, exact.to(torch.bfloat16))
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
    exact = (a.double() @ w13.double().t()).cpu().numpy()
    scale = (a.double().abs() @ w13.double().abs().t()).cpu().numpy()
    g, u = exact[:, :ffn], exact[:, ffn:]
    dg = 0.5 * bf16_ulp(g) + 2.0 ** -20 * scale[:, :ffn]        # bf16 g: rounding + fp32 summation
    du = 0.5 * bf16_ulp(u) + 2.0 ** -20 * scale[:, ffn:]
    silu = g / (1.0 + np.exp(-g))
    want = silu * u
    tol = (np.abs(silu) * du + np.abs(u) * 1.1 * dg + np.abs(u) * 0.5 * bf16_ulp(silu)
           + bf16_ulp(want)) * 1.5
    got = out.double().cpu().numpy()
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{int(bad.sum())} outputs beyond the bound, e.g. got {got[bad][:3]} exact {want[bad][:3]}"
    d = ulps(out, ref)
    assert (d == 0).mean() >= 0.995, f"only {(d == 0).mean():.5f} equal to b2_swiglu of the rounded products"


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
