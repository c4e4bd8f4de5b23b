"""GPU: the tcgen05 NT GEMM (3xTF32 and BF16) against float64, with the error
bar of an FP32 (non-TF32) cuBLAS product of the same operands.  3xTF32 shapes
with M a multiple of 256 and K >= 512 run on CTA pairs (cta_group::2), the
others on single CTAs with 128 x 128 tiles, or 128 x 64 tiles when fewer than
148 tiles of 128 x 128 cover the output; every path appears below, with and
without lower_only."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def split(torch, tb, x):
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    tb.check(tb.lib().tb_split_tf32(x.data_ptr(), hi.data_ptr(), lo.data_ptr(), x.numel(), None))
    return hi, lo


@pytest.mark.parametrize("M,N,K,alpha,beta,lower,kind", [
    (128, 128, 32, 1.0, 0.0, 0, "x3"), (256, 384, 96, 1.0, 0.0, 0, "x3"), (1024, 1024, 1024, 1.0, 0.0, 0, "x3"),
    (512, 256, 4096, 1.0, 0.0, 0, "x3"), (384, 384, 256, -1.0, 1.0, 1, "x3"), (2048, 1024, 512, 0.5, 2.0, 0, "x3"),
    (768, 768, 512, -1.0, 1.0, 1, "x3"), (640, 384, 1024, 1.0, 0.0, 0, "x3"), (256, 128, 8192, 1.0, 0.0, 0, "x3"),
    (512, 384, 512, -1.0, 1.0, 1, "x3"), (1152, 2432, 256, 0.5, 1.0, 0, "x3"), (1152, 1152, 384, -1.0, 1.0, 1, "x3"),
    (128, 128, 64, 1.0, 0.0, 0, "bf16"), (1024, 512, 2048, 0.5, 1.0, 0, "bf16"), (768, 768, 128, 1.0, 0.0, 1, "bf16"),
    (768, 768, 1024, 1.0, 0.0, 1, "bf16"), (512, 384, 2048, 1.0, 0.5, 0, "bf16")])
def test_gemm_nt_matches_float64(cuda, tblib, M, N, K, alpha, beta, lower, kind):
    torch = cuda
    L = tblib.lib()
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g)
    Cin = torch.randn(M, N, device="cuda", generator=g)
    Cout = torch.full((M, N), float("nan"), device="cuda")
    if kind == "x3":
        ah, al = split(torch, tblib, A)
        bh, bl = split(torch, tblib, B)
        rc = L.tb_gemm_nt_tf32x3(ah.data_ptr(), al.data_ptr(), K, bh.data_ptr(), bl.data_ptr(), K, M, N, K, alpha,
                                 beta, Cin.data_ptr(), N, Cout.data_ptr(), N, lower, None)
        Ar, Br = A.double(), B.double()
    else:
        Ab, Bb = A.bfloat16(), B.bfloat16()
        rc = L.tb_gemm_nt_bf16(Ab.data_ptr(), K, Bb.data_ptr(), K, M, N, K, alpha, beta, Cin.data_ptr(), N,
                               Cout.data_ptr(), N, lower, None)
        Ar, Br = Ab.double(), Bb.double()
    tblib.check(rc)
    torch.cuda.synchronize()
    tblib.check(L.tb_gemm_status(None))
    ref = alpha * (Ar @ Br.T) + beta * Cin.double()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    fp32 = (alpha * (Ar.float() @ Br.float().T) + beta * Cin).double()
    torch.backends.cuda.matmul.allow_tf32 = prev
    if lower:
        keep = torch.ones(M // 128, N // 128, dtype=torch.bool, device="cuda").tril()
        keep = keep.repeat_interleave(128, 0).repeat_interleave(128, 1)
        assert bool(torch.isnan(Cout[~keep]).all()), "tiles above the diagonal must not be written"
    else:
        keep = torch.ones(M, N, dtype=torch.bool, device="cuda")
    err = (Cout.double() - ref)[keep].abs().max().item()
    err_fp32 = (fp32 - ref)[keep].abs().max().item()
    assert err <= 4 * err_fp32 + 1e-6 * ref.abs().max().item(), (err, err_fp32)
