"""The decode GEMV and FFN entry points on their own, against torch fp32 on
the same bf16 operands: shapes the decoder at the default config does not
reach (several 1024-column passes, output widths that leave a partial
16-row tile, FFN widths that leave a partial 8-element tile) at 1, 2, 7 and
16 lockstep rows.  Tolerance: the result is fp32 accumulated from bf16
products, so it must match the fp32 reference within a few bf16 ulps of
the output scale (plus the bf16 rounding of the FFN's u, as the reference
rounds it)."""

import ctypes

import pytest
import torch

from dispatcher_b200._lib import call

pytestmark = pytest.mark.gpu

EPS = torch.finfo(torch.float32).eps


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B", [1, 2, 7, 16])
@pytest.mark.parametrize("k,n", [(2816, 1024), (1024, 200), (96, 40)])
def test_linear_residual(B, k, n):
    """x += y . W^T (and x_copy = the new x): K over 1, 2 or 3 passes of 1024
    columns, N = 200 / 40 leave a partial tile of row pairs."""
    g = torch.Generator(device="cuda").manual_seed(B * 7 + k)
    y = (torch.randn(B, k, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * k ** -0.5).bfloat16()
    x = torch.randn(B, n, device="cuda", generator=g)
    x_copy = torch.zeros_like(x)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = x + y.float() @ w.float().T
    call("dh_decode_linear_residual", _p(y), _p(w), _p(x), _p(x_copy), B, k, n, _p(st), _stream())
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    err = (x - want).abs().max().item()
    assert err < 2e-3 * (1 + want.abs().max().item()), err
    assert torch.equal(x, x_copy)


@pytest.mark.parametrize("B", [1, 2, 7, 16])
@pytest.mark.parametrize("d,ff", [(1024, 2816), (128, 203), (256, 40)])
def test_fused_ffn(B, d, ff):
    """x += (silu(h Wg^T) * (h Wu^T)) Wd^T with h = RMSNorm(x_in) (bf16) and
    the product rounded to bf16 as the reference rounds it; ff = 203 leaves
    a partial tile of 8 u elements."""
    g = torch.Generator(device="cuda").manual_seed(B * 11 + ff)
    x_in = torch.randn(B, d, device="cuda", generator=g)
    norm_w = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    wg = (torch.randn(ff, d, device="cuda", generator=g) * d ** -0.5).bfloat16()
    wu = (torch.randn(ff, d, device="cuda", generator=g) * d ** -0.5).bfloat16()
    wd = (torch.randn(d, ff, device="cuda", generator=g) * ff ** -0.5).bfloat16()
    wdT = wd.T.contiguous()
    x = x_in.clone()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    h = (x_in * torch.rsqrt(x_in.pow(2).mean(-1, keepdim=True) + EPS) * norm_w.float()).bfloat16()
    gt = h.float() @ wg.float().T
    up = h.float() @ wu.float().T
    u = (gt * torch.sigmoid(gt) * up).bfloat16()
    want = x_in + u.float() @ wd.float().T
    call("dh_decode_ffn", _p(x_in), _p(norm_w), _p(wg), _p(wu), _p(wdT), _p(x), B, d, ff, _p(st),
         _stream())
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    # u is rounded to bf16 on both sides, but from slightly different fp32
    # sums: a few elements can land one bf16 ulp apart
    err = (x - want).abs().max().item()
    assert err < 1e-2 * (1 + want.abs().max().item()), err
