"""ctypes mirrors of `dh_layer_params` / `dh_step_params`
(include/dispatcher_b200.h) and the packing of one decoder's weights,
caches and scratch into them for the persistent decode-step kernel."""

import ctypes

import torch

_c = ctypes.c_int
_p = ctypes.c_void_p


class LayerParams(ctypes.Structure):
    _fields_ = [("kind", _c), ("norm1", _p), ("norm2", _p), ("w_in3", _p), ("w_gates", _p),
                ("b_gates", _p), ("w_out", _p), ("w_gu", _p), ("w_down", _p), ("b_hist", _p),
                ("rg_hist", _p), ("v_ring", _p), ("k_cache", _p), ("v_cache", _p)]


class StepParams(ctypes.Structure):
    _fields_ = [("n_layers", _c), ("batch", _c), ("d", _c), ("H", _c), ("hd", _c), ("L", _c),
                ("ff", _c), ("vocab", _c), ("max_len", _c), ("window", _c), ("nsplit", _c),
                ("tokens", _p), ("t_buf", _p), ("emb", _p), ("lm_head", _p), ("norm_out", _p),
                ("rope_cos", _p),
                ("rope_sin", _p), ("layers", _p), ("logits", _p), ("x", _p), ("x_in", _p),
                ("a", _p), ("v0", _p), ("y", _p), ("q", _p), ("part", _p), ("counters", _p),
                ("barrier", _p), ("status", _p), ("trace", _p)]


SYNC_WORDS = 4096   # DH_STEP_SYNC_WORDS


def _ptr(t):
    return t.data_ptr() if t is not None else None


def swizzle_rows(w, period=None):
    """Rows of a bf16 matrix with their 16-byte chunks XOR-permuted: chunk c of
    row r moves to position c ^ (r & 7), r counted from the start of the
    matrix (or of each `period`-row tile).  This is the layout the decode-step
    kernel's ldmatrix reads expect after a linear copy into shared memory."""
    R, K = w.shape
    if K % 64:
        raise ValueError(f"row width {K} is not a multiple of 64 elements")
    r = torch.arange(R, device=w.device)
    if period is not None:
        r = r % period
    ch = torch.arange(K // 8, device=w.device)
    pos = ch[None, :] ^ (r[:, None] & 7)
    out = torch.empty_like(w).view(R, K // 8, 8)
    out.scatter_(1, pos[:, :, None].expand(R, K // 8, 8), w.view(R, K // 8, 8))
    return out.view(R, K)


def pack_step_weights(packed):
    """Per-layer packed forms used by the decode-step kernel (built once), all
    with chunk-permuted rows (swizzle_rows): W3 / Wqkv, W_out, the gate/up
    row pairs (2 ff, d), W_down^T (ff, d); for a tree layer the gate readouts
    as three 16-row tiles per head (H, 3, 16, gh) (row l = level l, zero rows
    past L), their biases (H, L, 3) fp32 and each head's columns of W_out
    (H, d, hd); and the tied output head."""
    if getattr(packed, "lm_head_sw", None) is None:
        packed.lm_head_sw = swizzle_rows(packed.lm_head)
    for lay in packed.layers:
        if "sw_in3" in lay:
            continue
        lay["sw_in3"] = swizzle_rows(lay["w3"] if lay["kind"] == "tree" else lay["wqkv"])
        ff, d = lay["w_gate"].shape
        lay["sw_gu"] = swizzle_rows(torch.stack([lay["w_gate"], lay["w_up"]], 1).reshape(2 * ff, d))
        lay["sw_downT"] = swizzle_rows(lay["w_down"].t().contiguous())
        if lay["kind"] == "tree":
            L, H, gh = lay["wi"].shape
            tiles = torch.zeros(H, 3, 16, gh, device=lay["wi"].device, dtype=torch.bfloat16)
            for g, name in enumerate(("wi", "wf", "wr")):
                tiles[:, g, :L] = lay[name].transpose(0, 1)
            lay["sw_gates"] = swizzle_rows(tiles.reshape(H * 3 * 16, gh), period=16)
            lay["b_gates_heads"] = torch.stack([lay["bi"], lay["bf"], lay["br"]], -1).permute(
                1, 0, 2).float().contiguous()
            hd = d // H
            heads = lay["w_out"].view(d, H, hd).permute(1, 0, 2).reshape(H * d, hd)
            lay["sw_out"] = swizzle_rows(heads.contiguous(), period=d)
        else:
            lay["sw_out"] = swizzle_rows(lay["w_out"])


def build_step_params(dec):
    """StepParams for decoder `dec` (its packed weights, caches and scratch);
    the layer table is uploaded to the device and kept alive on `dec`."""
    cfg, W = dec.cfg, dec.w
    pack_step_weights(W)
    n = cfg.num_layers
    arr = (LayerParams * n)()
    for i, (lay, cache) in enumerate(zip(W.layers, dec.caches)):
        e = arr[i]
        e.kind = 0 if lay["kind"] == "tree" else 1
        e.norm1, e.norm2 = _ptr(lay["norm1"]), _ptr(lay["norm2"])
        e.w_in3, e.w_out = _ptr(lay["sw_in3"]), _ptr(lay["sw_out"])
        e.w_gu, e.w_down = _ptr(lay["sw_gu"]), _ptr(lay["sw_downT"])
        if lay["kind"] == "tree":
            e.w_gates, e.b_gates = _ptr(lay["sw_gates"]), _ptr(lay["b_gates_heads"])
            e.b_hist, e.rg_hist, e.v_ring = _ptr(cache.B_hist), _ptr(cache.rg_hist), _ptr(cache.V_ring)
        else:
            e.k_cache, e.v_cache = _ptr(cache.k), _ptr(cache.v)
    raw = bytes(arr)
    dec._layer_table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dec.device)
    rope = next((c for c in dec.caches if hasattr(c, "rope_cos")), None)
    p = StepParams()
    p.n_layers, p.batch, p.d, p.H = n, dec.batch, cfg.d_model, cfg.num_heads
    p.hd, p.L, p.ff, p.vocab = cfg.d_model // cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
    p.max_len, p.window, p.nsplit = dec.max_len, cfg.attn_window, dec.nsplit
    p.tokens, p.t_buf = _ptr(dec.token_buf), _ptr(dec.t_buf)
    p.emb, p.lm_head, p.norm_out = _ptr(W.emb), _ptr(W.lm_head_sw), _ptr(W.norm_out)
    if rope is None:
        dec._rope_dummy = torch.zeros(2, device=dec.device)
        p.rope_cos = p.rope_sin = _ptr(dec._rope_dummy)
    else:
        p.rope_cos, p.rope_sin = _ptr(rope.rope_cos), _ptr(rope.rope_sin)
    p.layers = _ptr(dec._layer_table)
    p.logits = _ptr(dec.logits_out)
    p.x, p.x_in = _ptr(dec.x), _ptr(dec.x_copy)
    p.a, p.v0, p.y, p.q = (_ptr(getattr(dec, n_)) for n_ in ("a", "v0", "y", "q"))
    p.part = _ptr(dec.part)
    p.counters, p.barrier, p.status = _ptr(dec.counters), _ptr(dec.barrier), _ptr(dec.status)
    return p
