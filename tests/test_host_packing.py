"""CPU checks of the host-side weight layouts the kernels read: the SwiGLU
row interleave of the gate/up GEMM, the gate-weight packs of the forward and
backward gate kernels, the decode step's packs, the level count of the
parallel forward, and the single-document rule of the incremental decoders.  No GPU is needed: these
are the torch reshapes that run once before any launch."""

import pytest
import torch

import oracle
from dispatcher_b200 import ops
from dispatcher_b200.config import DispatcherConfig, small_config
from dispatcher_b200.decoding import check_single_document
from dispatcher_b200.engine import n_levels


def _gate_weights(L=12, H=16, gh=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    W = [torch.randn(L, H, gh, generator=g).bfloat16() for _ in range(3)]
    b = [torch.randn(L, H, generator=g) for _ in range(3)]
    return W, b


@pytest.mark.parametrize("ff,block", [(2816, 128), (384, 128), (256, 64)])
def test_interleave_swiglu_rows(ff, block):
    """Output rows 2*block*j .. +block are gate rows block*j .., the next block
    the matching up rows: one GEMM N-tile holds both halves of SwiGLU."""
    d = 32
    wg = torch.arange(ff * d, dtype=torch.float32).reshape(ff, d)
    wu = -wg - 1
    w = ops.interleave_swiglu(wg, wu, block)
    assert w.shape == (2 * ff, d) and w.is_contiguous()
    for j in range(ff // block):
        assert torch.equal(w[2 * block * j:2 * block * j + block], wg[block * j:block * (j + 1)])
        assert torch.equal(w[2 * block * j + block:2 * block * (j + 1)], wu[block * j:block * (j + 1)])


def test_interleave_swiglu_rejects_ragged_width():
    with pytest.raises(ValueError, match="multiple of 128"):
        ops.interleave_swiglu(torch.zeros(200, 8), torch.zeros(200, 8))


@pytest.mark.parametrize("H", [16, 2, 5])
def test_pack_gate_weights_layout(H):
    """Row l*NP + g*H + h = W_g[l, h] (g = admit, forget, transmit), NP = 3H
    rounded up to 16 with zero rows; biases fp32 in the same columns."""
    L, gh = 12, 64
    W, b = _gate_weights(L, H, gh, seed=H)
    w, bias, NP = ops.pack_gate_weights(*W, *b)
    assert NP == -(-3 * H // 16) * 16 and NP % 16 == 0 and NP >= 3 * H
    assert w.shape == (L * NP, gh) and w.dtype == torch.bfloat16
    assert bias.shape == (L, NP) and bias.dtype == torch.float32
    w3 = w.reshape(L, NP, gh)
    for g in range(3):
        assert torch.equal(w3[:, g * H:(g + 1) * H], W[g])
        assert torch.equal(bias[:, g * H:(g + 1) * H], b[g])
    assert not w3[:, 3 * H:].any() and not bias[:, 3 * H:].any()


@pytest.mark.parametrize("n_lv", [12, 7, 1])
def test_pack_gate_weights_t_layout(n_lv):
    """Per level, W^T (gh rows) with the 3H gate rows as columns, padded to 64:
    element [l*gh + k, g*H + h] = W_g[l, h, k]; levels >= n_lv are dropped."""
    L, H, gh = 12, 16, 128
    W, _ = _gate_weights(L, H, gh, seed=n_lv)
    wt = ops.pack_gate_weights_t(*W, n_lv)
    assert wt.shape == (n_lv * gh, 64) and wt.is_contiguous()
    wt3 = wt.reshape(n_lv, gh, 64)
    for g in range(3):
        assert torch.equal(wt3[:, :, g * H:(g + 1) * H], W[g][:n_lv].transpose(1, 2))
    assert not wt3[:, :, 3 * H:].any()


def test_level_count_matches_oracle():
    for L in (1, 4, 8, 12):
        for T in (1, 2, 3, 4, 5, 63, 64, 65, 255, 256, 257, 4095, 4096, 4097, 100000):
            assert n_levels(L, T) == oracle.n_levels(L, T), (L, T)


def test_single_document_rule():
    """Incremental decoders take one document per row when doc_reset is on;
    without doc reset the separator is an ordinary token."""
    cfg = small_config()
    ids = torch.tensor([[1, 2, 3], [4, cfg.eot_token, 6]])
    with pytest.raises(ValueError, match="document separator"):
        check_single_document(cfg, ids)
    check_single_document(cfg, ids[:1])
    check_single_document(small_config(doc_reset=False), ids)


def test_config_validation_and_levels():
    with pytest.raises(ValueError, match="power of two"):
        DispatcherConfig(max_len=3000)
    with pytest.raises(ValueError, match="divisible"):
        DispatcherConfig(d_model=1000, num_heads=16)
    cfg = DispatcherConfig()
    assert cfg.levels == 12 and cfg.head_dim == 64 and cfg.attn_slots() == {7, 16}
    assert DispatcherConfig(attn_window=0).attn_slots() == set()


def _unswizzle(w, period=None):
    R, K = w.shape
    r = torch.arange(R)
    if period is not None:
        r = r % period
    pos = torch.arange(K // 8)[None, :] ^ (r[:, None] & 7)
    return torch.gather(w.view(R, K // 8, 8), 1, pos[:, :, None].expand(R, K // 8, 8)).view(R, K)


def test_swizzle_rows_permutes_chunks():
    """Chunk c of row r lands at c ^ (r & 7), counted per tile with `period`."""
    from dispatcher_b200.step_params import swizzle_rows
    w = torch.arange(40 * 128, dtype=torch.float32).reshape(40, 128).bfloat16()
    sw = swizzle_rows(w)
    assert torch.equal(sw[0], w[0])
    assert torch.equal(sw[3].view(16, 8)[5 ^ 3], w[3].view(16, 8)[5])
    assert torch.equal(_unswizzle(sw), w)
    swp = swizzle_rows(w, period=16)
    assert torch.equal(_unswizzle(swp, 16), w)
    assert torch.equal(swp[16], w[16]) and torch.equal(swp[19].view(16, 8)[2 ^ 3], w[19].view(16, 8)[2])


def test_decode_step_weight_packs():
    """Decode-step packs (all rows chunk-permuted): W3 / Wqkv, W_out, gate/up
    as (2 ff, d) row pairs, W_down^T; for a tree layer the gate readouts as
    three 16-row tiles per head (row l = level l, zero rows past L), their
    biases (H, L, 3) fp32 and each head's columns of W_out (H, d, hd); and a
    permuted copy of the tied output head."""
    from types import SimpleNamespace
    from dispatcher_b200.step_params import pack_step_weights
    g = torch.Generator().manual_seed(3)
    ff, d, L, H, gh = 384, 128, 8, 2, 128
    W, b = _gate_weights(L, H, gh, seed=3)
    w_out = torch.randn(d, d, generator=g).bfloat16()
    mk = lambda *s: torch.randn(*s, generator=g).bfloat16()  # noqa: E731
    tree = dict(kind="tree", w3=mk(3 * d, d), w_gate=mk(ff, d), w_up=mk(ff, d),
                w_down=mk(d, ff), w_out=w_out, wi=W[0], wf=W[1], wr=W[2],
                bi=b[0], bf=b[1], br=b[2])
    attn = dict(kind="attn", wqkv=mk(3 * d, d), w_gate=mk(ff, d), w_up=mk(ff, d),
                w_down=mk(d, ff), w_out=mk(d, d))
    emb = mk(515, d)
    packed = SimpleNamespace(layers=[tree, attn], lm_head=emb)
    pack_step_weights(packed)
    assert torch.equal(_unswizzle(packed.lm_head_sw[:512]), emb[:512])
    for lay in (tree, attn):
        gu = _unswizzle(lay["sw_gu"]).view(ff, 2, d)
        assert torch.equal(gu[:, 0], lay["w_gate"]) and torch.equal(gu[:, 1], lay["w_up"])
        assert torch.equal(_unswizzle(lay["sw_downT"]), lay["w_down"].t())
        src = lay["w3"] if lay["kind"] == "tree" else lay["wqkv"]
        assert torch.equal(_unswizzle(lay["sw_in3"]), src)
    assert torch.equal(_unswizzle(attn["sw_out"]), attn["w_out"])
    assert "sw_gates" not in attn
    tiles = _unswizzle(tree["sw_gates"], 16).view(H, 3, 16, gh)
    for gi in range(3):
        assert torch.equal(tiles[:, gi, :L].transpose(0, 1), W[gi])
    assert not tiles[:, :, L:].any()
    bh = tree["b_gates_heads"]
    assert bh.shape == (H, L, 3) and bh.dtype == torch.float32
    for gi in range(3):
        assert torch.equal(bh[:, :, gi].transpose(0, 1), b[gi])
    hd = d // H
    heads = _unswizzle(tree["sw_out"], d).view(H, d, hd)
    for h in range(H):
        assert torch.equal(heads[h], w_out[:, h * hd:(h + 1) * hd])
    before = tree["sw_gates"].data_ptr()
    pack_step_weights(packed)            # built once: a second call keeps the packs
    assert tree["sw_gates"].data_ptr() == before
