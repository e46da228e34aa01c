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


def _tree_state(B, d, H, L, T, docs, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hd = d // H
    bf16 = torch.bfloat16
    st = dict(
        x=torch.randn(B, d, device="cuda", generator=g),
        norm_w=(1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(bf16),
        w3=(torch.randn(3 * d, d, device="cuda", generator=g) * d ** -0.5).to(bf16),
        wi=(torch.randn(L, H, d, device="cuda", generator=g) * d ** -0.5).to(bf16),
        wf=(torch.randn(L, H, d, device="cuda", generator=g) * d ** -0.5).to(bf16),
        wr=(torch.randn(L, H, d, device="cuda", generator=g) * d ** -0.5).to(bf16),
        bi=0.5 * torch.randn(L, H, device="cuda", generator=g),
        bf=0.5 * torch.randn(L, H, device="cuda", generator=g),
        br=0.5 * torch.randn(L, H, device="cuda", generator=g),
        B_hist=torch.randn(B, T + 1, d, device="cuda", generator=g).to(bf16),
        rg_hist=torch.rand(B, T + 1, L, H, device="cuda", generator=g).to(bf16),
        V_ring=torch.randn(B, 2 ** (L + 1) - 2, d, device="cuda", generator=g).to(bf16),
        t_buf=torch.full((1,), T, dtype=torch.long, device="cuda"),
        doc=None,
    )
    if docs:
        # a document boundary every ~T/5 positions, different per row
        sep = (torch.rand(B, T + 1, device="cuda", generator=g) < 5.0 / T).int()
        st["doc"] = torch.cumsum(sep, 1, dtype=torch.int32) - sep
    return st, hd


@pytest.mark.parametrize("B", [1, 4])
@pytest.mark.parametrize("H,L,T", [(2, 3, 3), (2, 16, 40000), (16, 16, 33000), (4, 12, 1500)])
@pytest.mark.parametrize("docs", [False, True])
def test_mixer_in_gates_matches_separate_launches(B, H, L, T, docs):
    """dh_decode_mixer_in_gates + dh_decode_tree_recur (W3 GEMV with the
    gate readouts folded in) against dh_decode_mixer_in + dh_decode_tree_step
    on the same state: every level live (t >= 2^(L-1)) or some masked (t <
    2^(L-1)), 2..16 heads (np 16 and 48), up to 16 levels, with and without
    document masks.  v0 / A / B_hist[:, t] come from the same kind of
    tensor-core GEMV; the gate pre-activations are fp32 sums in another
    order, so the sigmoid gates and what follows may differ by one bf16 ulp."""
    d = 128
    st, hd = _tree_state(B, d, H, L, T, docs, seed=B * 31 + H * 7 + L)
    from dispatcher_b200.ops import pack_gate_weights
    wg_np, _, np_ = pack_gate_weights(st["wi"], st["wf"], st["wr"], st["bi"], st["bf"], st["br"])
    wg_t = wg_np.t().contiguous()
    max_len = T + 1
    outs = []
    for fused in (False, True):
        v0 = torch.zeros(B, d, device="cuda", dtype=torch.bfloat16)
        a = torch.zeros_like(v0)
        y = torch.zeros_like(v0)
        bh, rg, vr = st["B_hist"].clone(), st["rg_hist"].clone(), st["V_ring"].clone()
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        s = _stream()
        if fused:
            pre = torch.zeros(B, L * np_, device="cuda")
            call("dh_decode_mixer_in_gates", _p(st["x"]), _p(st["norm_w"]), _p(st["w3"]), _p(v0),
                 _p(a), _p(bh), _p(st["t_buf"]), max_len, B, d, _p(wg_t), np_, L, H, _p(pre),
                 _p(st["doc"]), _p(status), s)
            call("dh_decode_tree_recur", _p(st["bi"]), _p(st["bf"]), _p(st["br"]),
                 _p(st["t_buf"]), _p(pre), np_, _p(rg), _p(v0), _p(vr), _p(y), _p(st["doc"]),
                 B, max_len, L, H, hd, s)
        else:
            ig = torch.zeros(B, L, H, device="cuda")
            fg = torch.zeros_like(ig)
            ctr = torch.zeros(H, dtype=torch.int32, device="cuda")
            call("dh_decode_mixer_in", _p(st["x"]), _p(st["norm_w"]), _p(st["w3"]), _p(v0),
                 _p(a), _p(bh), _p(st["t_buf"]), max_len, B, d, _p(status), s)
            call("dh_decode_tree_step", _p(a), _p(bh), _p(st["wi"]), _p(st["wf"]), _p(st["wr"]),
                 _p(st["bi"]), _p(st["bf"]), _p(st["br"]), _p(st["t_buf"]), _p(ig), _p(fg),
                 _p(rg), _p(v0), _p(vr), _p(y), _p(ctr), _p(st["doc"]), B, max_len, L, H, hd, d,
                 s)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        if fused:
            assert int(torch.count_nonzero(pre)) == 0      # left zero for the next step
        outs.append((v0, a, bh, rg, vr, y))
    (v0s, as_, bhs, rgs, vrs, ys), (v0f, af, bhf, rgf, vrf, yf) = outs
    for u, v in ((v0s, v0f), (as_, af), (bhs, bhf)):
        assert torch.allclose(u.float(), v.float(), rtol=2 ** -7, atol=1e-3)
    assert torch.equal(bhs[:, :T], bhf[:, :T])
    # one bf16 ulp of values in (0, 1) for the gates, of the output scale after
    assert (rgs.float() - rgf.float()).abs().max().item() <= 2 ** -8
    scale = 1 + ys.float().abs().max().item()
    assert (ys.float() - yf.float()).abs().max().item() <= 2e-2 * scale
    assert (vrs.float() - vrf.float()).abs().max().item() <= 2e-2 * (1 + vrs.float().abs().max().item())
    # untouched history rows stay bit-identical
    assert torch.equal(rgs[:, :T], rgf[:, :T])
