"""GPU: the tensor-core GEMM engine alone (hffn_gemm_tc_f32), every operand major, against float64 torch.

out [n, m] = (A B^T)^T, A and B each K-major ([rows, k]) or MN-major (stored [k, rows]); operands split into tf32
hi / lo parts on the host side of the test (torch rounding of the low 13 mantissa bits)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def tf32_split(t: torch.Tensor):
    bits = t.contiguous().view(torch.int32)
    hi = ((bits + 0x1000) & ~0x1FFF).view(torch.float32)      # round to nearest (ties away) at 10 mantissa bits
    rest = t - hi
    lo = ((rest.view(torch.int32) + 0x1000) & ~0x1FFF).view(torch.float32)
    return hi.contiguous(), lo.contiguous()


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 300, 512), (96, 64, 100)])
def test_gemm_majors(a_mn, b_mn, m, n, k):
    from hffn_b200 import _native as native
    if (a_mn and m % 32) or (b_mn and n % 32):
        pytest.skip("MN-major extents are multiples of 32")
    g = torch.Generator().manual_seed(m * 7 + n * 3 + k + 11 * a_mn + 13 * b_mn)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    a_store = a.T.contiguous() if a_mn else a          # [k, m] or [m, k]
    b_store = b.T.contiguous() if b_mn else b
    a_hi, a_lo = (t.cuda() for t in tf32_split(a_store))
    b_hi, b_lo = (t.cuda() for t in tf32_split(b_store))
    out = torch.full((n, m), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = native.lib.hffn_gemm_tc_f32(a_mn, b_mn, a_hi.data_ptr(), a_lo.data_ptr(), b_hi.data_ptr(),
                                         b_lo.data_ptr(), out.data_ptr(), m, n, k, m if a_mn else k,
                                         n if b_mn else k, err.data_ptr(), native.stream_handle(torch.device("cuda")))
    native.check(status, "hffn_gemm_tc_f32")
    torch.cuda.synchronize()
    expected = (b.double() @ a.double().T)
    assert int(err) == 0
    error = float((out.double().cpu() - expected).abs().max())
    assert error <= 1e-5 * float(expected.abs().max()) + 1e-5, (a_mn, b_mn, m, n, k, error)
