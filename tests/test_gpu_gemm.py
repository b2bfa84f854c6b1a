"""sae_b200_gemm on the tcgen05 tile GEMM, against a plain PyTorch fp32 product.

The module API's dense products under bf16 autocast -- decode (x_hat = acts
W_dec^T, sae_trainer_rolling.py:922-925), its input and weight gradients, and
the encoder's weight gradient (592-607) -- take bf16 operands. The library
runs them on the tensor cores when both operands are stored K-major, and the
Python wrapper transposes the ones that are not. The reference here is
torch's fp32 matmul of the same bf16 values (exact products, fp32 sums): the
only difference is the summation order, so fp32 outputs agree to 1e-5
relative (3e-5 allowed for the tensor cores' fp32 accumulation over up to
8192 terms); bf16 outputs to one bf16 rounding (2^-8 relative).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

FP32_TOL = 3e-5
BF16_TOL = 2 ** -8


def _lib():
    from sae_b200 import _lib as L
    L.load()
    return L


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


def _call(L, M, N, K, A, sam, sak, B, sbn, sbk, C, scm, scn, alpha=1.0, beta=0.0, bias=None):
    dt = {torch.float32: L.DTYPE_F32, torch.bfloat16: L.DTYPE_BF16}
    L.call("sae_b200_gemm", M, N, K, alpha, A.data_ptr(), dt[A.dtype], sam, sak, B.data_ptr(),
           dt[B.dtype], sbn, sbk, beta, C.data_ptr(), dt[C.dtype], scm, scn,
           0 if bias is None else bias.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _operands(M, N, K, seed, pad_a=0, pad_b=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K + pad_a, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K + pad_b, device="cuda", generator=g).to(torch.bfloat16)
    return A, B


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 200), (1000, 136, 1000),
                                   (4096, 1536, 8192)])
def test_k_major_fp32_output(M, N, K):
    """Ragged M, N and K (TMA zero fill past the edges, row-guarded stores)."""
    L = _lib()
    A, B = _operands(M, N, K, 1)
    C = torch.full((M, N), float("nan"), device="cuda")
    launches = L.launch_count()
    _call(L, M, N, K, A, K, 1, B, K, 1, C, N, 1)
    torch.cuda.synchronize()
    assert L.launch_count() == launches + 1
    assert L.device_status() == 0
    ref = A.float() @ B.float().t()
    assert torch.isfinite(C).all()
    assert _rel(C, ref) < FP32_TOL


def test_pitched_operands_alpha_beta_bias():
    """Row pitches beyond K, alpha, an accumulating beta and a column bias."""
    L = _lib()
    M, N, K = 384, 640, 320
    A, B = _operands(M, N, K, 2, pad_a=24, pad_b=8)
    C0 = torch.randn(M, N + 4, device="cuda")
    C = C0.clone()
    bias = torch.randn(N, device="cuda")
    _call(L, M, N, K, A, K + 24, 1, B, K + 8, 1, C, N + 4, 1, alpha=0.5, beta=1.0, bias=bias)
    torch.cuda.synchronize()
    ref = 0.5 * (A[:, :K].float() @ B[:, :K].float().t()) + C0[:, :N] + bias
    assert _rel(C[:, :N], ref) < FP32_TOL
    assert torch.equal(C[:, N:], C0[:, N:])       # the pitch padding is never written


def test_column_major_output_with_bias():
    """C with scm == 1: the library computes C^T = B A^T (bias per row of C^T)."""
    L = _lib()
    M, N, K = 512, 384, 256
    A, B = _operands(M, N, K, 3)
    Ct = torch.empty(N, M, device="cuda")        # C[m, n] at n * M + m
    bias = torch.randn(N, device="cuda")
    _call(L, M, N, K, A, K, 1, B, K, 1, Ct, 1, M, bias=bias)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t() + bias
    assert _rel(Ct.t(), ref) < FP32_TOL


def test_bf16_output():
    L = _lib()
    M, N, K = 640, 1024, 512
    A, B = _operands(M, N, K, 4)
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _call(L, M, N, K, A, K, 1, B, K, 1, C, N, 1)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    err = (C.float() - ref).abs() / ref.abs().clamp(min=1.0)
    assert float(err.max()) <= BF16_TOL
    assert _rel(C.float(), ref) < BF16_TOL


def test_transpose():
    L = _lib()
    for rows, cols, lds, ldd in ((1000, 136, 136, 1008), (64, 64, 72, 64), (33, 7, 7, 33)):
        src = torch.randn(rows, lds, device="cuda").to(torch.bfloat16)
        dst = torch.zeros(cols, ldd, device="cuda", dtype=torch.bfloat16)
        L.call("sae_b200_transpose", src.data_ptr(), L.DTYPE_BF16, rows, cols, lds,
               dst.data_ptr(), ldd, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert torch.equal(dst[:, :rows], src[:, :cols].t())
        assert not dst[:, rows:].any()


def test_wrapper_transposes_mn_major_operands():
    """The module API's weight-gradient shape: dW[F, d] = dpre^T xc with both
    operands stored [B, .] (the contraction dimension outermost): the wrapper
    transposes them and the product runs on the tensor cores."""
    from sae_b200.sae import gemm
    L = _lib()
    Btok, F, d = 2048, 1024, 256
    g = torch.Generator(device="cuda").manual_seed(5)
    dpre = torch.randn(Btok, F, device="cuda", generator=g).to(torch.bfloat16)
    xc = torch.randn(Btok, d, device="cuda", generator=g).to(torch.bfloat16)
    dW = torch.empty(F, d, device="cuda")
    gemm(F, d, Btok, dpre, 1, F, xc, 1, d, dW, d, 1)
    torch.cuda.synchronize()
    assert _rel(dW, dpre.float().t() @ xc.float()) < FP32_TOL
    # decode: x_hat = acts [B, F] . W_fm [F, d] -- the weight is the MN-major operand
    W = torch.randn(F, d, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(Btok, d, device="cuda", dtype=torch.bfloat16)
    gemm(Btok, d, F, dpre, F, 1, W, 1, d, out, d, 1)
    torch.cuda.synchronize()
    ref = dpre.float() @ W.float()
    assert _rel(out.float(), ref) < BF16_TOL
    assert L.device_status() == 0


def test_small_and_fp32_products_stay_exact_on_cuda_cores():
    """Shapes below the tile size and fp32 operands take the CUDA-core kernel."""
    L = _lib()
    A = torch.randn(7, 33, device="cuda")
    B = torch.randn(5, 33, device="cuda")
    C = torch.empty(7, 5, device="cuda")
    _call(L, 7, 5, 33, A, 33, 1, B, 33, 1, C, 5, 1)
    torch.cuda.synchronize()
    torch.testing.assert_close(C, A @ B.t(), rtol=1e-5, atol=1e-5)
