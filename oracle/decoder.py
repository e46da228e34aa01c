"""Eager restatement of the reference's exact incremental decoder (test oracle).

Follows dispatcher_hybrid/decoding.py: `_TreeLayerCache` (:50-76),
`_AttnCache` (:79-86), `_check_single_document` (:89-98) and
`IncrementalDecoder` (:101-304).  Its caches are exposed with the same
names and layouts so the B200 decoder's ring buffers, slot positions and
histories can be compared element for element:

    B_hist  (B, max_len, gh)     gate source vectors
    rg_hist (B, max_len, L, H)   transmit gates at their source position
    V_ring  (B, S, d)            level j in slots [2^(j+1)-2, 2^(j+2)-2),
                                 slot of position t = offset_j + (t & (2^(j+1)-1))
    k, v    (B, max_len, H, hd)  attention caches, k stored after RoPE
"""

import math

import torch
import torch.nn.functional as F

from .model import rmsnorm, rope_tables, swiglu, _lin


def RING_OFFSETS(L):
    """Ring j starts at slot 2^(j+1) - 2 (decoding.py:59-64)."""
    return [2 ** (j + 1) - 2 for j in range(L)]


def ring_slot(j, t):
    """Slot of position t in ring j: offset + (t & mask) (decoding.py:63-66)."""
    return (2 ** (j + 1) - 2) + (t & (2 ** (j + 1) - 1))


class _TreeCache:
    def __init__(self, batch, max_len, gh, L, H, hd, dtype):
        self.L, self.H, self.hd = L, H, hd
        d = H * hd
        self.B_hist = torch.zeros(batch, max_len, gh, dtype=dtype)
        self.rg_hist = torch.zeros(batch, max_len, L, H, dtype=dtype)
        self.S = 2 ** (L + 1) - 2
        self.V_ring = torch.zeros(batch, self.S, d, dtype=dtype)
        self.offsets = torch.tensor(RING_OFFSETS(L))
        self.masks = torch.tensor([2 ** (j + 1) - 1 for j in range(L)])

    def write_slab(self, j, slab):
        """decoding.py:68-76: the last 2^(j+1) positions of a (B, T, d) slab."""
        T = slab.shape[1]
        size = 2 ** (j + 1)
        p0 = max(0, T - size)
        pos = torch.arange(p0, T)
        self.V_ring[:, self.offsets[j] + (pos & self.masks[j])] = slab[:, p0:]


class _AttnCache:
    def __init__(self, batch, max_len, H, hd, dtype):
        self.k = torch.zeros(batch, max_len, H, hd, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.rope_cos, self.rope_sin = rope_tables(max_len, hd, dtype)


class OracleDecoder:
    """IncrementalDecoder (decoding.py:101-304) over a state dict."""

    def __init__(self, sd, cfg, max_len=None):
        self.sd, self.cfg = sd, cfg
        self.max_len = max_len or cfg.max_len
        self.dtype = sd["embedding.weight"].dtype
        self.caches = None
        self.batch = None
        self.t = 0

    def _alloc(self, batch):                                       # :129-140
        if self.caches is not None and self.batch == batch:
            return
        cfg = self.cfg
        self.batch = batch
        H, hd, L = cfg.num_heads, cfg.d_model // cfg.num_heads, cfg.levels
        slots = cfg.attn_slots()
        self.caches = [
            _AttnCache(batch, self.max_len, H, hd, self.dtype) if i in slots else
            _TreeCache(batch, self.max_len, cfg.d_model, L, H, hd, self.dtype)
            for i in range(cfg.num_layers)]

    # ---------- tree layer ----------
    def _tree_prefill(self, p, cache, x):                          # :143-185
        sd = self.sd
        m = p + "mixer."
        Bb, T = x.shape[0], x.shape[1]
        h1 = rmsnorm(x, sd[p + "norm1.weight"])
        A = _lin(h1, sd[m + "gate_hidden.weight"])
        Bs = _lin(h1, sd[m + "gate_hidden_src.weight"])
        cache.B_hist[:, :T] = Bs
        L, H, hd = cache.L, cache.H, cache.hd
        n_lv = min(L, int(math.log2(T)) + 1) if T > 1 else 1
        V = _lin(h1, sd[m + "linear_in.weight"]).view(Bb, T, H, hd)
        cache.write_slab(0, V.reshape(Bb, T, H * hd))
        rolled = torch.stack([torch.roll(Bs, shifts=2 ** l, dims=1)
                              for l in range(n_lv)], dim=2)
        wrap = torch.zeros(T, n_lv, 1, dtype=x.dtype)
        for l in range(n_lv):
            wrap[2 ** l:, l] = 1.0
        hidden = torch.relu(A.unsqueeze(2) + rolled * wrap) ** 2
        ein = lambda w, b: torch.einsum("btlg,lhg->btlh", hidden, sd[m + w][:n_lv]) + sd[m + b][:n_lv]
        pre_i = ein("gate_out", "gate_out_bias")
        pre_f = ein("forget_out", "forget_out_bias")
        pre_r = ein("reset_out", "reset_out_bias")
        ig = torch.sigmoid(pre_i) * wrap
        fg = torch.sigmoid(pre_f) * wrap + (1.0 - wrap)
        rg = torch.sigmoid(pre_r)
        cache.rg_hist[:, :T, :n_lv] = rg
        if n_lv < L:                                               # :168-174
            hid0 = torch.relu(A) ** 2
            for l in range(n_lv, L):
                cache.rg_hist[:, :T, l] = torch.sigmoid(
                    hid0 @ sd[m + "reset_out"][l].T + sd[m + "reset_out_bias"][l])
        for l in range(n_lv):                                      # :175-180
            src = rg[:, :, l].unsqueeze(-1) * V
            msg = torch.roll(src, shifts=2 ** l, dims=1)
            V = fg[:, :, l].unsqueeze(-1) * V + ig[:, :, l].unsqueeze(-1) * msg
            if l + 1 < L:
                cache.write_slab(l + 1, V.reshape(Bb, T, H * hd))
        for j in range(n_lv + 1, L):                               # :182-183
            cache.write_slab(j, V.reshape(Bb, T, H * hd))
        x = x + _lin(V.reshape(Bb, T, H * hd), sd[m + "linear_out.weight"])
        return x + swiglu(sd, p + "ffn.", rmsnorm(x, sd[p + "norm2.weight"]))

    def _tree_step(self, p, cache, x, t):                          # :187-222
        sd = self.sd
        m = p + "mixer."
        Bb = x.shape[0]
        L, H, hd = cache.L, cache.H, cache.hd
        h1 = rmsnorm(x, sd[p + "norm1.weight"])
        A = _lin(h1, sd[m + "gate_hidden.weight"])
        cache.B_hist[:, t] = _lin(h1, sd[m + "gate_hidden_src.weight"])
        V = _lin(h1, sd[m + "linear_in.weight"]).view(Bb, H, hd)
        cache.V_ring[:, cache.offsets[0] + (t & int(cache.masks[0]))] = V.reshape(Bb, -1)
        arangeL = torch.arange(L)
        src_t = t - torch.pow(2, arangeL)
        ok = src_t >= 0
        src_c = src_t.clamp(min=0)
        Bg = cache.B_hist[:, src_c] * ok.view(1, L, 1)
        hid = torch.relu(A.unsqueeze(1) + Bg) ** 2
        okf = ok.view(1, L, 1)
        i_ = torch.sigmoid(torch.einsum("blg,lhg->blh", hid, sd[m + "gate_out"])
                           + sd[m + "gate_out_bias"]) * okf
        f_ = torch.sigmoid(torch.einsum("blg,lhg->blh", hid, sd[m + "forget_out"])
                           + sd[m + "forget_out_bias"])
        f_ = f_ * okf + (~okf).to(f_.dtype)
        r_ = torch.sigmoid(torch.einsum("blg,lhg->blh", hid, sd[m + "reset_out"])
                           + sd[m + "reset_out_bias"])
        cache.rg_hist[:, t] = r_
        rg_src = cache.rg_hist[:, src_c, arangeL]
        slots = cache.offsets + (src_c & cache.masks)
        V_src = cache.V_ring[:, slots].view(Bb, L, H, hd)
        msg = rg_src.unsqueeze(-1) * V_src
        for l in range(L):
            V = f_[:, l].unsqueeze(-1) * V + i_[:, l].unsqueeze(-1) * msg[:, l]
            if l + 1 < L:
                cache.V_ring[:, cache.offsets[l + 1] + (t & int(cache.masks[l + 1]))] = V.reshape(Bb, -1)
        x = x + _lin(V.reshape(Bb, -1), sd[m + "linear_out.weight"])
        return x + swiglu(sd, p + "ffn.", rmsnorm(x, sd[p + "norm2.weight"]))

    # ---------- attention layer ----------
    def _attn_prefill(self, p, cache, x):                          # :225-245
        sd, cfg = self.sd, self.cfg
        a = p + "attn."
        Bb, T = x.shape[0], x.shape[1]
        H = cfg.num_heads
        hd = cfg.d_model // H
        h1 = rmsnorm(x, sd[p + "norm1.weight"])
        shape = (Bb, T, H, hd)
        q = _lin(h1, sd[a + "linear_q.weight"]).view(shape).transpose(1, 2)
        k = _lin(h1, sd[a + "linear_k.weight"]).view(shape).transpose(1, 2)
        v = _lin(h1, sd[a + "linear_v.weight"]).view(shape)
        cos, sin = rope_tables(T, hd, x.dtype)

        def rope(z):
            z1, z2 = z[..., 0::2], z[..., 1::2]
            return torch.stack([z1 * cos - z2 * sin, z1 * sin + z2 * cos], dim=-1).flatten(-2)
        qb, kb = rope(q), rope(k)
        cache.k[:, :T] = kb.transpose(1, 2)
        cache.v[:, :T] = v
        vb = v.transpose(1, 2)
        if 0 < cfg.attn_window < T:
            tt = torch.arange(T)
            band = (tt[:, None] >= tt[None, :]) & (tt[:, None] - tt[None, :] < cfg.attn_window)
            y = F.scaled_dot_product_attention(qb, kb, vb, attn_mask=band)
        else:
            y = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True)
        x = x + _lin(y.transpose(1, 2).reshape(Bb, T, H * hd), sd[a + "linear_out.weight"])
        return x + swiglu(sd, p + "ffn.", rmsnorm(x, sd[p + "norm2.weight"]))

    def _attn_step(self, p, cache, x, t):                          # :247-266
        sd, cfg = self.sd, self.cfg
        a = p + "attn."
        Bb = x.shape[0]
        H = cfg.num_heads
        hd = cfg.d_model // H
        h1 = rmsnorm(x, sd[p + "norm1.weight"])
        cos, sin = cache.rope_cos[t], cache.rope_sin[t]

        def rope(z):
            z1, z2 = z[..., 0::2], z[..., 1::2]
            return torch.stack([z1 * cos - z2 * sin, z1 * sin + z2 * cos], dim=-1).flatten(-2)
        q = rope(_lin(h1, sd[a + "linear_q.weight"]).view(Bb, H, hd))
        cache.k[:, t] = rope(_lin(h1, sd[a + "linear_k.weight"]).view(Bb, H, hd))
        cache.v[:, t] = _lin(h1, sd[a + "linear_v.weight"]).view(Bb, H, hd)
        lo = max(0, t + 1 - cfg.attn_window) if cfg.attn_window > 0 else 0
        k = cache.k[:, lo:t + 1]
        v = cache.v[:, lo:t + 1]
        att = torch.softmax(torch.einsum("bhd,bthd->bht", q, k) / math.sqrt(hd), dim=-1)
        y = torch.einsum("bht,bthd->bhd", att, v).reshape(Bb, -1)
        x = x + _lin(y, sd[a + "linear_out.weight"])
        return x + swiglu(sd, p + "ffn.", rmsnorm(x, sd[p + "norm2.weight"]))

    # ---------- public ----------
    def check_single_document(self, ids):                          # :89-98
        cfg = self.cfg
        if getattr(cfg, "doc_reset", False) and bool((ids == cfg.eot_token).any()):
            raise ValueError(
                f"prompt contains the document separator (token {cfg.eot_token}) "
                f"and this model was trained with doc_reset=True; the incremental "
                f"decoders assume a single document.")

    @torch.no_grad()
    def prefill(self, idx):                                        # :269-284
        self._squeeze = idx.dim() == 1
        ids = idx.view(1, -1) if self._squeeze else idx
        self.check_single_document(ids)
        if ids.shape[1] > self.max_len:
            raise ValueError(f"prompt of {ids.shape[1]} exceeds max_len {self.max_len}")
        self._alloc(ids.shape[0])
        x = F.embedding(ids, self.sd["embedding.weight"]).to(self.dtype)
        slots = self.cfg.attn_slots()
        for i, cache in enumerate(self.caches):
            p = f"blocks.{i}."
            x = (self._attn_prefill(p, cache, x) if i in slots
                 else self._tree_prefill(p, cache, x))
        self.t = ids.shape[1]
        out = _lin(rmsnorm(x, self.sd["norm_out.weight"]), self.sd["lm_head.weight"])
        return out[0] if self._squeeze else out

    @torch.no_grad()
    def step(self, tokens):                                        # :286-304
        if self.t >= self.max_len:
            raise ValueError(f"context exhausted at max_len {self.max_len}")
        t = self.t
        toks = tokens.view(-1)
        if toks.shape[0] != self.batch and not (self.batch == 1 and toks.shape[0] == 1):
            raise ValueError(f"got {toks.shape[0]} tokens for batch {self.batch}")
        x = F.embedding(toks, self.sd["embedding.weight"]).to(self.dtype)
        slots = self.cfg.attn_slots()
        for i, cache in enumerate(self.caches):
            p = f"blocks.{i}."
            x = (self._attn_step(p, cache, x, t) if i in slots
                 else self._tree_step(p, cache, x, t))
        self.t = t + 1
        out = _lin(rmsnorm(x, self.sd["norm_out.weight"]), self.sd["lm_head.weight"])
        return out[0] if self._squeeze else out
