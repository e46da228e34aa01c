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
                ("tokens", _p), ("t_buf", _p), ("emb", _p), ("norm_out", _p), ("rope_cos", _p),
                ("rope_sin", _p), ("layers", _p), ("logits", _p), ("x", _p), ("x_in", _p),
                ("a", _p), ("v0", _p), ("y", _p), ("q", _p), ("part", _p), ("counters", _p),
                ("barrier", _p), ("status", _p), ("trace", _p)]


SYNC_WORDS = 4096   # DH_STEP_SYNC_WORDS


def _ptr(t):
    return t.data_ptr() if t is not None else None


def pack_step_weights(packed):
    """Per-layer packed forms used by the step kernel (built once):
    w_gu (ff, 2, d) gate/up row pairs, w_downT (ff, d); tree blocks: the gate
    readouts per head (H, L, 3, gh), their biases (H, L, 3) fp32 and each
    head's columns of W_out (H, d, hd)."""
    for lay in packed.layers:
        if "w_gu_pairs" not in lay:
            lay["w_gu_pairs"] = torch.stack([lay["w_gate"], lay["w_up"]], 1).contiguous()
        if "w_downT" not in lay:
            lay["w_downT"] = lay["w_down"].t().contiguous()
        if lay["kind"] == "tree" and "w_gates_heads" not in lay:
            L, H, gh = lay["wi"].shape
            lay["w_gates_heads"] = torch.stack([lay["wi"], lay["wf"], lay["wr"]], 2).permute(
                1, 0, 2, 3).contiguous()
            lay["b_gates_heads"] = torch.stack([lay["bi"], lay["bf"], lay["br"]], -1).permute(
                1, 0, 2).float().contiguous()
            d = lay["w_out"].shape[0]
            lay["w_out_heads"] = lay["w_out"].view(d, H, d // H).permute(1, 0, 2).contiguous()


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
        e.w_gu, e.w_down = _ptr(lay["w_gu_pairs"]), _ptr(lay["w_downT"])
        if lay["kind"] == "tree":
            e.w_in3, e.w_out = _ptr(lay["w3"]), _ptr(lay["w_out_heads"])
            e.w_gates, e.b_gates = _ptr(lay["w_gates_heads"]), _ptr(lay["b_gates_heads"])
            e.b_hist, e.rg_hist, e.v_ring = _ptr(cache.B_hist), _ptr(cache.rg_hist), _ptr(cache.V_ring)
        else:
            e.w_in3, e.w_out = _ptr(lay["wqkv"]), _ptr(lay["w_out"])
            e.k_cache, e.v_cache = _ptr(cache.k), _ptr(cache.v)
    raw = bytes(arr)
    dec._layer_table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dec.device)
    rope = next((c for c in dec.caches if hasattr(c, "rope_cos")), None)
    p = StepParams()
    p.n_layers, p.batch, p.d, p.H = n, dec.batch, cfg.d_model, cfg.num_heads
    p.hd, p.L, p.ff, p.vocab = cfg.d_model // cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
    p.max_len, p.window, p.nsplit = dec.max_len, cfg.attn_window, dec.nsplit
    p.tokens, p.t_buf = _ptr(dec.token_buf), _ptr(dec.t_buf)
    p.emb, p.norm_out = _ptr(W.emb), _ptr(W.norm_out)
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
