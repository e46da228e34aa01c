"""tcgen05 GEMM against a plain PyTorch fp32 reference of the same op
(bf16 inputs, fp32 accumulate, one bf16 rounding of the result)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from dispatcher_b200 import ops  # noqa: E402


def ref_mm(a, w):
    return a.float() @ w.float().T


def rel_err(got, ref):
    return ((got.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 320, 128), (1000, 1024, 1024),
                                   (4096, 3072, 1024), (513, 2816, 2816), (257, 5003, 128),
                                   (64, 100, 192)])
def test_gemm_store(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    out = ops.gemm(a, w)
    # bf16 output rounding bound (2^-8 relative) plus accumulation-order noise
    assert rel_err(out, ref_mm(a, w)) < 8e-3


def test_gemm_strided_views_and_residual():
    M, K, N = 700, 1024, 1024
    big = torch.randn(M, 3 * K, device="cuda").bfloat16()
    a = big[:, K:2 * K]                      # row stride 3K, like the proj3 output views
    w = torch.randn(N, K, device="cuda").bfloat16() * 0.05
    r = torch.randn(M, N, device="cuda").bfloat16()
    ref = r.float() + (ref_mm(a, w).bfloat16().float())
    out = r.clone()
    ops.gemm(a, w, out=out, epilogue=ops.EPI_RESIDUAL, residual=out)   # in place
    assert rel_err(out, ref) < 8e-3


def test_gemm_swiglu():
    M, K, ff = 520, 1024, 2816
    a = torch.randn(M, K, device="cuda").bfloat16()
    wg = (torch.randn(ff, K, device="cuda") * 0.03).bfloat16()
    wu = (torch.randn(ff, K, device="cuda") * 0.03).bfloat16()
    w = ops.interleave_swiglu(wg, wu)
    out = ops.gemm(a, w, epilogue=ops.EPI_SWIGLU)
    ref = torch.nn.functional.silu(ref_mm(a, wg)) * ref_mm(a, wu)
    assert out.shape == (M, ff)
    assert rel_err(out, ref) < 1e-2


def test_gemm_status_stays_clear():
    a = torch.randn(256, 128, device="cuda").bfloat16()
    w = torch.randn(384, 128, device="cuda").bfloat16()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.gemm(a, w, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
