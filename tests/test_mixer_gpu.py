"""Mixer kernels of the parallel forward against the oracle (the reference's
eager mixer restated): tree mask (exact), gate readout, the reference's
gate_preacts op, the level sweep, window attention, and the whole mixer at
the configuration-1 shape (one tree layer, B=2, T=1024, default width)."""

import pytest
import torch
import torch.nn.functional as F

import oracle
from dispatcher_b200 import ops, make_state_dict, small_config, DispatcherConfig
from tests.helpers import cast_sd, max_err

pytestmark = pytest.mark.gpu


def mixer_setup(cfg, seed, nondeg, B, T, eot_at=()):
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    g = torch.Generator().manual_seed(seed + 40)
    x = torch.randn(B, T, cfg.d_model, generator=g)
    ids = torch.randint(0, cfg.vocab_size - 1, (B, T), generator=g)
    for b, t in eot_at:
        ids[b, t] = cfg.eot_token
    mask = oracle.tree_mask(ids, cfg.levels, cfg.eot_token, cfg.doc_reset)
    return sd, x, ids, mask


@pytest.mark.parametrize("T", [1, 2, 5, 64, 160, 1000])
def test_tree_mask_exact(T):
    cfg = small_config(max_len=1024)
    g = torch.Generator().manual_seed(T)
    ids = torch.randint(0, cfg.vocab_size, (3, T), generator=g)
    ids[1, T // 2] = cfg.eot_token
    ids[2, ::7] = cfg.eot_token
    ref = oracle.tree_mask(ids, cfg.levels, cfg.eot_token, True)
    ref = ref.expand(3, T, cfg.levels) if ref.dim() == 3 else ref
    got = ops.tree_mask(ids.cuda(), cfg.levels, cfg.eot_token, True).cpu()
    assert torch.equal(got, (ref != 0).to(torch.uint8))
    wrap = ops.tree_mask(ids.cuda(), cfg.levels, cfg.eot_token, False).cpu()
    assert torch.equal(wrap[0], (oracle.level_mask(T, cfg.levels) != 0).to(torch.uint8))


def _gpu_internals(sd, p, cfg, x, mask, B, T):
    """proj3 GEMM + gates + scan on the GPU; returns gates and V."""
    d, H, L = cfg.d_model, cfg.num_heads, cfg.levels
    w3 = torch.cat([sd[p + n + ".weight"] for n in ("linear_in", "gate_hidden",
                                                    "gate_hidden_src")]).cuda().bfloat16()
    P = ops.gemm(x.reshape(B * T, d).cuda().bfloat16(), w3)
    wg, bias, NP = ops.pack_gate_weights(*(sd[p + n].cuda() for n in (
        "gate_out", "forget_out", "reset_out", "gate_out_bias", "forget_out_bias",
        "reset_out_bias")))
    n_lv = oracle.n_levels(L, T)
    m8 = None
    if mask.dim() == 3:
        m8 = (mask != 0).to(torch.uint8).cuda().contiguous()
    gates = ops.mixer_gates(P[:, d:2 * d], P[:, 2 * d:], wg, bias, NP, H, L, n_lv, B, mask=m8)
    V = ops.level_scan(P[:, :d], gates, H, L, n_lv, B)
    return gates, V.view(B, T, d), n_lv


@pytest.mark.parametrize("T,eot", [(160, ((1, 57), (1, 130))), (37, ()), (256, ((0, 3),)), (1, ())])
def test_gates_and_scan_small(T, eot):
    cfg = small_config()
    B = 2
    sd, x, ids, mask = mixer_setup(cfg, 1, True, B, T, eot)
    p = "blocks.0.mixer."
    ref = oracle.mixer_internals(sd, p, cfg.num_heads, cfg.levels, x, mask)
    gates, V, n_lv = _gpu_internals(sd, p, cfg, x, mask, B, T)
    H = cfg.num_heads
    g = gates.float().cpu()[:, :, :n_lv]                        # (B, H, n_lv, T, 4)
    for gi, name in enumerate(("admit", "forget", "transmit")):
        want = ref[name].view(B, H, T, n_lv).permute(0, 1, 3, 2)
        assert max_err(g[..., gi], want) < 2e-2, name
    assert torch.equal(g[..., 3], torch.zeros_like(g[..., 3]))
    ref16 = oracle.mixer_internals(cast_sd(sd, torch.bfloat16), p, H, cfg.levels,
                                   x.bfloat16(), mask.bfloat16())["V"].float()
    bound = 2 * max_err(ref16, ref["V"]) + 2e-2
    assert max_err(V.float().cpu(), ref["V"]) < bound


def test_gates_default_width():
    """The gate kernel at the default width (16 heads: the epilogue writes each
    position's (admit, forget, transmit, 0) straight from registers) against
    the oracle's masked sigmoid gates, with a document separator live."""
    cfg = DispatcherConfig()
    B, T = 2, 300
    sd, x, ids, mask = mixer_setup(cfg, 3, True, B, T, ((0, 77), (1, 201)))
    p = "blocks.0.mixer."
    ref = oracle.mixer_internals(sd, p, cfg.num_heads, cfg.levels, x, mask)
    gates, V, n_lv = _gpu_internals(sd, p, cfg, x, mask, B, T)
    H = cfg.num_heads
    g = gates.float().cpu()[:, :, :n_lv]                        # (B, H, n_lv, T, 4)
    for gi, name in enumerate(("admit", "forget", "transmit")):
        want = ref[name].view(B, H, T, n_lv).permute(0, 1, 3, 2)
        assert max_err(g[..., gi], want) < 2e-2, name
    assert torch.equal(g[..., 3], torch.zeros_like(g[..., 3]))


@pytest.mark.parametrize("T", [1000, 1024, 1500, 2048, 2049, 3000, 4096])
def test_level_scan_bit_exact_long(T):
    """The sweep alone at lengths where shifts of 1024 and 2048 occur (levels
    that stay inside a thread), against the oracle's level loop in bf16:
    same rounding points, so bit-exact.  The gates carry the level mask (admit
    0, forget 1 before the shift), as the gate kernel writes them."""
    B, H, hd, L = 2, 2, 64, 12
    d = H * hd
    n_lv = oracle.n_levels(L, T)
    g = torch.Generator().manual_seed(T)
    v0 = torch.randn(B * T, d, generator=g).bfloat16()
    gates = torch.rand(B, H, L, T, 4, generator=g).bfloat16()
    gates[..., 3] = 0
    lm = oracle.level_mask(T, L)                                # (T, L), 1 where t >= 2^l
    gates[..., 0] *= lm.t().bfloat16()
    gates[..., 1] = torch.where(lm.t().bool(), gates[..., 1], torch.ones_like(gates[..., 1]))
    got = ops.level_scan(v0.cuda(), gates.cuda().contiguous(), H, L, n_lv, B).cpu()
    V = v0.view(B, T, H, hd).transpose(1, 2).reshape(B * H, T, hd)
    gl = gates[:, :, :n_lv].permute(0, 1, 3, 2, 4).reshape(B * H, T, n_lv, 4)
    want = oracle.level_sweep(V, gl[..., 0], gl[..., 1], gl[..., 2], n_lv)
    want = want.view(B, H, T, hd).transpose(1, 2).reshape(B * T, d)
    assert torch.equal(got, want)


@pytest.mark.parametrize("nondeg", [False, True])
def test_mixer_configuration_1(golden, nondeg):
    """Configuration 1 (one tree layer at the default width, B=2, T=1024,
    x ~ N(0,1) from seed 0): V after all levels, against the fp32 oracle,
    and the oracle itself against the reference's golden rows."""
    from tests.golden.make_golden import FULL_ROWS
    cfg = DispatcherConfig()
    seed, tag = (1, "s1nd") if nondeg else (0, "s0")
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    torch.manual_seed(0)
    x = torch.randn(2, 1024, cfg.d_model)
    mask = oracle.level_mask(1024, cfg.levels)
    p = "blocks.0.mixer."
    ref = oracle.mixer_internals(sd, p, cfg.num_heads, cfg.levels, x, mask)["V"]
    assert max_err(ref[:, FULL_ROWS], torch.from_numpy(golden[f"full_{tag}_c1_V_rows"])) < 1e-4
    ref16 = oracle.mixer_internals(cast_sd(sd, torch.bfloat16), p, cfg.num_heads, cfg.levels,
                                   x.bfloat16(), mask.bfloat16())["V"].float()
    _, V, _ = _gpu_internals(sd, p, cfg, x, mask, 2, 1024)
    err = max_err(V.float().cpu(), ref)
    bound = 2 * max_err(ref16, ref) + 2e-2
    assert err < bound, f"V max|d| {err:.4f} > bound {bound:.4f}"


def test_gate_preacts_op_matches_reference_semantics():
    """dispatcher::gate_preacts_fwd contract (fused_gates.py:307-314)."""
    cfg = small_config()
    B, T = 2, 100
    sd, x, ids, mask = mixer_setup(cfg, 2, True, B, T, ((0, 40),))
    p = "blocks.0.mixer."
    ref = oracle.mixer_internals(sd, p, cfg.num_heads, cfg.levels, x, mask)
    A, Bm = ref["A"].cuda(), ref["B"].cuda()
    n_lv = ref["n_lv"]
    outs = ops.gate_preacts_fwd(A, Bm, *(sd[p + n].cuda() for n in (
        "gate_out", "forget_out", "reset_out", "gate_out_bias", "forget_out_bias",
        "reset_out_bias")), n_lv, mask.cuda())
    for got, name in zip(outs, ("pre_i", "pre_f", "pre_r")):
        assert got.shape == (B, T, n_lv, cfg.num_heads) and got.dtype == torch.bfloat16
        want = ref[name]
        assert max_err(got.float().cpu(), want) < 0.02 * want.abs().max().item() + 1e-2, name


@pytest.mark.parametrize("T,window", [(100, 64), (300, 64), (256, 1024), (1100, 1024), (64, 0),
                                      (1, 64), (129, 128)])
def test_window_attention(T, window):
    B, H, hd = 2, 4, 64
    d = H * hd
    g = torch.Generator().manual_seed(T)
    qkv = torch.randn(B * T, 3 * d, generator=g).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = ops.window_attention(qkv.cuda().clone(), B, H, window, status=status).float().cpu()
    assert int(status.item()) == 0
    q, k, v = qkv.float().view(B, T, 3, H, hd).permute(2, 0, 3, 1, 4)
    cos, sin = oracle.rope_tables(T, hd)
    q, k = oracle.apply_rope(q, cos, sin), oracle.apply_rope(k, cos, sin)
    t = torch.arange(T)
    if 0 < window < T:
        band = (t[:, None] >= t[None, :]) & (t[:, None] - t[None, :] < window)
        y = F.scaled_dot_product_attention(q, k, v, attn_mask=band)
    else:
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    want = y.transpose(1, 2).reshape(B * T, d)
    assert max_err(got, want) < 3e-2
