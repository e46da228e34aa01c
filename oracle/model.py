"""Eager restatement of the reference parallel forward (test oracle).

All citations are to dispatcher_hybrid/modeling_dispatcher.py unless noted.
Weights come as a flat state dict with the reference's key names, so the
same dict loads into the reference model for the golden fixtures.
Arithmetic runs in the dtype of the weights, op by op, like the reference's
eager path, so the oracle run in bf16 is also the same-dtype eager baseline.
"""

import math

import torch
import torch.nn.functional as F


def n_levels(L, T):
    """Levels run by the parallel forward: min(L, floor(log2 T) + 1) (:76)."""
    return min(L, int(math.log2(T)) + 1)


def level_mask(T, L, dtype=torch.float32, device="cpu"):
    """mask[t, i] = 1 iff 2**i < T and t >= 2**i (:282-297)."""
    mask = torch.zeros(T, L, dtype=dtype, device=device)
    for i in range(L):
        if 2 ** i < T:
            mask[2 ** i:, i] = 1.0
    return mask


def tree_mask(ids, L, eot_token, doc_reset, dtype=torch.float32):
    """(T, L) wrap mask, or (B, T, L) with doc reset (:311-323): doc_id is the
    exclusive prefix count of EOT tokens and a level-i edge survives only when
    doc_id(t) == doc_id(t - 2**i) (compared through a circular roll)."""
    T = ids.shape[1]
    mask = level_mask(T, L, dtype, ids.device)
    if not doc_reset:
        return mask
    is_eot = (ids == eot_token).to(dtype)
    doc_id = torch.cumsum(is_eot, dim=1) - is_eot
    allowed = torch.stack([(doc_id == torch.roll(doc_id, 2 ** i, dims=1))
                           for i in range(L)], dim=-1).to(dtype)
    return mask.unsqueeze(0) * allowed[..., :mask.shape[-1]]


def rmsnorm(x, w):
    """torch.nn.RMSNorm with eps=None (:207-208): computed in fp32 with the
    fp32 machine epsilon, scaled by the weight in fp32, rounded once."""
    xf = x.float()
    eps = torch.finfo(torch.float32).eps
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype)


def _lin(x, w):
    return F.linear(x, w)


def mixer_internals(sd, p, H, L, x, mask):
    """The mixer up to (and including) the level scan (:63-121).

    Returns dict with V0 (B*H, T, hd), A, B, the sigmoid gates
    admit/forget/transmit (B*H, T, n_lv) after masking, and V after all
    levels, (B, T, d) — the quantity the tree layer feeds to linear_out."""
    batch, length, d = x.shape
    hd = d // H
    V = _lin(x, sd[p + "linear_in.weight"]).view(batch, length, H, hd).transpose(1, 2)
    V = V.reshape(batch * H, length, hd)                       # :70-71
    V0 = V
    A = _lin(x, sd[p + "gate_hidden.weight"])                  # :73
    B = _lin(x, sd[p + "gate_hidden_src.weight"])              # :74
    n_lv = n_levels(L, length)
    if mask.dim() == 3:                                        # :77-84
        m4 = mask[..., :n_lv].unsqueeze(-1)
        mbh = (mask[..., :n_lv].unsqueeze(1).expand(batch, H, length, n_lv)
               .reshape(batch * H, length, n_lv))
    else:
        m4 = mask[:, :n_lv].view(1, length, n_lv, 1)
        mbh = mask[:, :n_lv]
    shifts = [2 ** i for i in range(L)]
    rolled = torch.stack([torch.roll(B, shifts=s, dims=1)
                          for s in shifts[:n_lv]], dim=2) * m4     # :102-103
    hidden = F.relu(A.unsqueeze(2) + rolled) ** 2                  # :104
    pre = [torch.einsum("btld,lhd->btlh", hidden, sd[p + w][:n_lv]) + sd[p + b][:n_lv]
           for w, b in (("gate_out", "gate_out_bias"),
                        ("forget_out", "forget_out_bias"),
                        ("reset_out", "reset_out_bias"))]          # :105-109

    def heads_first(pr):                                           # :86-88
        return torch.sigmoid(pr).permute(0, 3, 1, 2).reshape(
            batch * H, length, n_lv).to(V.dtype)

    admit = heads_first(pre[0]) * mbh                              # :111
    forget = heads_first(pre[1]) * mbh + (1.0 - mbh)               # :113
    transmit = heads_first(pre[2])                                 # :114
    V = level_sweep(V, admit, forget, transmit, n_lv)
    Vout = V.view(batch, H, length, hd).transpose(1, 2).reshape(batch, length, d)
    return dict(V0=V0, A=A, B=B, pre_i=pre[0], pre_f=pre[1], pre_r=pre[2],
                admit=admit, forget=forget, transmit=transmit, V=Vout, n_lv=n_lv)


def gate_preacts(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask=None):
    """The reference op's math (fused_gates.py:307-314, the einsums of
    modeling_dispatcher.py:100-109): A, B (b, T, gh) -> pre_i, pre_f, pre_r
    (b, T, n_lv, H) = W_x[l] . relu(A + m * roll(B, 2^l))^2 + b_x, m the wrap
    mask times the optional (b, T, n_lv) doc mask.  Differentiable (plain
    torch ops), the autograd oracle of the backward op."""
    b, T, gh = A.shape
    wrap = level_mask(T, n_lv, dtype=A.dtype)                 # (T, n_lv)
    m = wrap.unsqueeze(0).expand(b, T, n_lv)
    if mask is not None:
        m = m * mask[..., :n_lv].to(A.dtype)
    rolled = torch.stack([torch.roll(B, shifts=2 ** l, dims=1) for l in range(n_lv)], dim=2)
    hidden = F.relu(A.unsqueeze(2) + rolled * m.unsqueeze(-1)) ** 2     # (b, T, n_lv, gh)
    return tuple(torch.einsum("btld,lhd->btlh", hidden, w[:n_lv]) + bb[:n_lv]
                 for w, bb in ((Wi, bi), (Wf, bf), (Wr, br)))


def level_sweep(V, admit, forget, transmit, n_lv):
    """The level loop (:116-120): V (B*H, T, hd), gates (B*H, T, n_lv) after
    masking; in V's dtype, so bf16 inputs round after every product and sum."""
    length = V.shape[1]
    for li in range(n_lv):
        shift = 2 ** li
        if shift > length:
            break
        msg = torch.roll(transmit[..., li:li + 1] * V, shifts=shift, dims=1)
        V = forget[..., li:li + 1] * V + admit[..., li:li + 1] * msg
    return V


def mixer_forward(sd, p, H, L, x, mask):
    """DispatcherMixer.forward, eager branch (:63-123)."""
    V = mixer_internals(sd, p, H, L, x, mask)["V"]
    return _lin(V, sd[p + "linear_out.weight"])                   # :122-123


def rope_tables(length, hd, dtype=torch.float32, device="cpu"):
    """cos/sin of angle t * 10000^(-2j/hd), made in fp32 then cast (:144-161)."""
    theta = 10000.0 ** (-torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd)
    angles = torch.arange(length, device=device, dtype=torch.float32)[:, None] * theta[None, :]
    return angles.cos().to(dtype), angles.sin().to(dtype)


def apply_rope(x, cos, sin):
    """Pairs (0::2, 1::2) rotated and re-interleaved (:163-166)."""
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2)


def window_attention(sd, p, H, window, x):
    """WindowAttention.forward (:168-185): banded causal SDPA."""
    batch, length, d = x.shape
    hd = d // H
    shape = (batch, length, H, hd)
    q = _lin(x, sd[p + "linear_q.weight"]).view(shape).transpose(1, 2)
    k = _lin(x, sd[p + "linear_k.weight"]).view(shape).transpose(1, 2)
    v = _lin(x, sd[p + "linear_v.weight"]).view(shape).transpose(1, 2)
    cos, sin = rope_tables(length, hd, x.dtype, x.device)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    if 0 < window < length:
        t = torch.arange(length, device=x.device)
        band = (t[:, None] >= t[None, :]) & (t[:, None] - t[None, :] < window)
        y = F.scaled_dot_product_attention(q, k, v, attn_mask=band)
    else:
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    y = y.transpose(1, 2).reshape(batch, length, d)
    return _lin(y, sd[p + "linear_out.weight"])


def swiglu(sd, p, h):
    """SwiGLU.forward (:196-197)."""
    return _lin(F.silu(_lin(h, sd[p + "linear_gate.weight"])) * _lin(h, sd[p + "linear_up.weight"]),
                sd[p + "linear_down.weight"])


def forward(sd, cfg, ids, return_hidden=False):
    """DispatcherHybridForCausalLM.forward (:325-351) -> logits (B, T, V)."""
    length = ids.shape[1]
    if length > cfg.max_len:
        raise ValueError(f"sequence length {length} exceeds max_len {cfg.max_len}")
    dtype = sd["embedding.weight"].dtype
    mask = tree_mask(ids, cfg.levels, cfg.eot_token, cfg.doc_reset, dtype)
    x = F.embedding(ids, sd["embedding.weight"])
    slots = cfg.attn_slots()
    hidden = []
    for i in range(cfg.num_layers):
        p = f"blocks.{i}."
        hidden.append(x)
        h = rmsnorm(x, sd[p + "norm1.weight"])
        if i in slots:                                              # :225-227
            x = x + window_attention(sd, p + "attn.", cfg.num_heads, cfg.attn_window, h)
        else:                                                       # :210-212
            x = x + mixer_forward(sd, p + "mixer.", cfg.num_heads, cfg.levels, h, mask)
        x = x + swiglu(sd, p + "ffn.", rmsnorm(x, sd[p + "norm2.weight"]))
    x = rmsnorm(x, sd["norm_out.weight"])
    logits = _lin(x, sd["lm_head.weight"])
    return (logits, hidden) if return_hidden else logits
