"""tcgen05 GEMM of libb2o against a plain PyTorch fp32 reference and against
the library's CUDA-core kernel (an independent implementation)."""
import pytest
import torch

from sol_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(fn, A, lda, sA, ak, B, ldb, sB, bk, D, ldd, sD, C, ldc, sC, M, N, K, batch, epi, sym, alpha, beta,
          gamma, scale=None, rowsq=None, simt=False):
    lib = _lib.load()
    st = _lib.stream_ptr()
    cp = C.data_ptr() if C is not None else None
    sp = scale.data_ptr() if scale is not None else None
    rp = rowsq.data_ptr() if rowsq is not None else None
    if simt:
        rc = lib.b2o_gemm_bf16_simt(A.data_ptr(), lda, sA, ak, B.data_ptr(), ldb, sB, bk, D.data_ptr(), ldd, sD, cp,
                                    ldc, sC, M, N, K, batch, epi, alpha, beta, gamma, sp, rp, st)
    else:
        rc = lib.b2o_gemm_bf16(A.data_ptr(), lda, sA, ak, B.data_ptr(), ldb, sB, bk, D.data_ptr(), ldd, sD, cp,
                               ldc, sC, M, N, K, batch, epi, sym, alpha, beta, gamma, sp, rp, st)
    _lib.check(rc, "gemm")


def _operands(batch, M, N, K, ak, bk, gen, dev, scale=1.0):
    A = (torch.randn(batch, M, K, generator=gen, device=dev) * scale).to(torch.bfloat16)
    B = (torch.randn(batch, N, K, generator=gen, device=dev) * scale).to(torch.bfloat16)
    As = A if ak else A.transpose(1, 2).contiguous()   # stored layout
    Bs = B if bk else B.transpose(1, 2).contiguous()
    return A, B, As, Bs


def _run(As, Bs, A, B, M, N, K, batch, ak, bk, epi=0, sym=0, alpha=1.0, beta=0.0, gamma=0.0, C=None,
         scale=None, rowsq=None, simt=False):
    D = torch.full((batch, M, N), float("nan"), device=A.device).to(torch.bfloat16)
    lda = K if ak else M
    ldb = K if bk else N
    _call(None, As, lda, As[0].numel(), ak, Bs, ldb, Bs[0].numel(), bk, D, N, M * N,
          C, N, M * N, M, N, K, batch, epi, sym, alpha, beta, gamma, scale, rowsq, simt)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return D


@pytest.mark.parametrize("ak,bk", [(1, 1), (1, 0), (0, 1), (0, 0)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (384, 640, 320), (200, 296, 136), (128, 128, 64)])
def test_gemm_layouts_vs_torch(cuda, ak, bk, M, N, K):
    gen = torch.Generator(device=cuda).manual_seed(M * 7 + N + K + 10 * ak + bk)
    batch = 2
    A, B, As, Bs = _operands(batch, M, N, K, ak, bk, gen, cuda)
    D = _run(As, Bs, A, B, M, N, K, batch, ak, bk)
    ref = A.float() @ B.float().transpose(1, 2)
    assert not torch.isnan(D.float()).any()
    torch.testing.assert_close(D.float(), ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2 * ref.abs().max().item())
    Ds = _run(As, Bs, A, B, M, N, K, batch, ak, bk, simt=True)
    diff = (D.float() - Ds.float()).abs()
    assert (diff <= 1e-2 * ref.abs().max()).all()
    assert (D == Ds).float().mean() > 0.97


@pytest.mark.parametrize("kmajor", [1, 0])
@pytest.mark.parametrize("m,n", [(1024, 1024), (256, 1536), (384, 200 + 56)])
def test_symmetric_syrk(cuda, kmajor, m, n):
    """X X^T with only upper-triangle tiles computed and mirrored."""
    gen = torch.Generator(device=cuda).manual_seed(m + n + kmajor)
    batch = 3
    X = torch.randn(batch, m, n, generator=gen, device=cuda).to(torch.bfloat16)
    Xs = X if kmajor else X.transpose(1, 2).contiguous()
    D = _run(Xs, Xs, X, X, m, m, n, batch, kmajor, kmajor, sym=1)
    ref = X.float() @ X.float().transpose(1, 2)
    assert torch.equal(D, D.transpose(1, 2))
    torch.testing.assert_close(D.float(), ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2 * ref.abs().max().item())


def test_epilogues(cuda):
    gen = torch.Generator(device=cuda).manual_seed(5)
    m, batch = 512, 2
    X = (torch.randn(batch, m, 700 - 4, generator=gen, device=cuda) / 30).to(torch.bfloat16)
    R = (X.float() @ X.float().transpose(1, 2)).to(torch.bfloat16)
    a, b, c = 3.4445, -4.7750, 2.0315
    eye = torch.eye(m, device=cuda)
    # P = a I + b R + c R^2 (single rounding)
    P = _run(R, R, R, R, m, m, m, batch, 1, 1, epi=1, sym=1, alpha=a, beta=b, gamma=c, C=R)
    ref = a * eye + b * R.float() + c * (R.float() @ R.float())
    torch.testing.assert_close(P.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    # quintic B = bf16(b*A) + bf16(c*bf16(A A))
    Bq = _run(R, R, R, R, m, m, m, batch, 1, 1, epi=2, sym=1, beta=b, gamma=c, C=R)
    AA = (R.float() @ R.float()).to(torch.bfloat16)
    refB = ((b * R.float()).to(torch.bfloat16).float() + (c * AA.float()).to(torch.bfloat16).float())
    torch.testing.assert_close(Bq.float(), refB.to(torch.bfloat16).float(), rtol=2e-2,
                               atol=2e-2 * refB.abs().max().item())
    # per-batch scale and row sums of squares of the stored output
    scale = torch.tensor([0.5, 2.0], device=cuda)
    n = X.shape[2]
    ntn = (n + 255) // 256
    rowsq = torch.zeros(batch * ntn * m, device=cuda)
    # B MN-major (stored K x N = X itself): D = R X
    D = _run(R, X, R, None, m, n, m, batch, 1, 0, scale=scale, rowsq=rowsq)
    ref = scale.view(-1, 1, 1) * (R.float() @ X.float())
    torch.testing.assert_close(D.float(), ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2 * ref.abs().max().item())
    rs = rowsq.view(batch, ntn, m).sum(1)
    torch.testing.assert_close(rs, D.float().pow(2).sum(-1), rtol=1e-4, atol=1e-6)


def test_large_k_tall_syrk(cuda):
    """The NorMuon tall case: R = X^T X for X 5632 x 1024 (MN-major operands), K = 5632."""
    gen = torch.Generator(device=cuda).manual_seed(11)
    X = (torch.randn(2, 5632, 1024, generator=gen, device=cuda) / 80).to(torch.bfloat16)
    D = torch.empty(2, 1024, 1024, device=cuda, dtype=torch.bfloat16)
    _call(None, X, 1024, X[0].numel(), 0, X, 1024, X[0].numel(), 0, D, 1024, 1024 * 1024, None, 0, 0,
          1024, 1024, 5632, 2, 0, 1, 1.0, 0.0, 0.0)
    torch.cuda.synchronize()
    ref = X.float().transpose(1, 2) @ X.float()
    torch.testing.assert_close(D.float(), ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2 * ref.abs().max().item())


@pytest.mark.parametrize("out_dtype", [2, 1])
def test_binary16_operands(cuda, out_dtype):
    """kind::f16 with binary16 operands (the Gram iteration's storage type)."""
    gen = torch.Generator(device=cuda).manual_seed(21)
    M, N, K, batch = 384, 512, 320, 2
    A = torch.randn(batch, M, K, generator=gen, device=cuda).half()
    X = torch.randn(batch, K, N, generator=gen, device=cuda).half()   # B MN-major
    odt = torch.float16 if out_dtype == 2 else torch.bfloat16
    D = torch.empty(batch, M, N, device=cuda, dtype=odt)
    lib = _lib.load()
    rc = lib.b2o_gemm(A.data_ptr(), K, M * K, 1, X.data_ptr(), N, K * N, 0, D.data_ptr(), N, M * N, None, 0, 0,
                      M, N, K, batch, 2, out_dtype, 0, 0, 1.0, 0.0, 0.0, None, None, _lib.stream_ptr())
    _lib.check(rc, "gemm f16")
    torch.cuda.synchronize()
    ref = A.float() @ X.float()
    torch.testing.assert_close(D.float(), ref.to(odt).float(), rtol=1e-2, atol=1e-2 * ref.abs().max().item())
