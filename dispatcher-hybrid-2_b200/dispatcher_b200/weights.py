"""Seeded random-init weights with the reference's parameter names, shapes and
init distributions, so that a reference model (or this package's mirror)
can load them with `load_state_dict`.

Distributions follow `DispatcherPreTrainedModel._init_weights`
(dispatcher_hybrid/modeling_dispatcher.py:236-247): every Linear and the
embedding ~ N(0, 0.02); gate_out / forget_out / reset_out ~ N(0, 0.02);
gate_hidden_src (W1s) zero; gate biases constant (-2 admit, +2 forget, +2
transmit; modeling_dispatcher.py:53-60); RMSNorm weights one.  The draw order
is this module's own (a torch CPU generator walked over the keys in a fixed
order), so values differ from the reference's global-seed init but are
reproducible on any machine running the same torch build.

`nondegenerate=True` also draws W1s, the gate biases and the norm weights
at random: at the reference init W1s is exactly zero, which would leave the
shifted-source term of the gate hidden state untested.
"""

import torch

from .config import DispatcherConfig


def state_dict_keys(cfg):
    """(name, shape, kind) for every parameter, in reference state_dict order."""
    d, H, L, ff, V = (cfg.d_model, cfg.num_heads, cfg.levels,
                      cfg.dim_feedforward, cfg.vocab_size)
    slots = cfg.attn_slots()
    out = [("embedding.weight", (V, d), "normal")]
    for i in range(cfg.num_layers):
        p = f"blocks.{i}."
        if i in slots:
            for n in ("linear_q", "linear_k", "linear_v", "linear_out"):
                out.append((p + f"attn.{n}.weight", (d, d), "normal"))
        else:
            m = p + "mixer."
            out += [(m + "gate_out", (L, H, d), "normal"),
                    (m + "gate_out_bias", (L, H), "bias_i"),
                    (m + "forget_out", (L, H, d), "normal"),
                    (m + "forget_out_bias", (L, H), "bias_f"),
                    (m + "reset_out", (L, H, d), "normal"),
                    (m + "reset_out_bias", (L, H), "bias_r"),
                    (m + "linear_in.weight", (d, d), "normal"),
                    (m + "gate_hidden.weight", (d, d), "normal"),
                    (m + "gate_hidden_src.weight", (d, d), "w1s"),
                    (m + "linear_out.weight", (d, d), "normal")]
        out += [(p + "ffn.linear_gate.weight", (ff, d), "normal"),
                (p + "ffn.linear_up.weight", (ff, d), "normal"),
                (p + "ffn.linear_down.weight", (d, ff), "normal"),
                (p + "norm1.weight", (d,), "norm"),
                (p + "norm2.weight", (d,), "norm")]
    out.append(("norm_out.weight", (d,), "norm"))
    return out


def make_state_dict(cfg=None, seed=0, nondegenerate=False, dtype=torch.float32):
    """Return an fp32 (or `dtype`) CPU state dict; `lm_head.weight` is the
    embedding tensor itself (tied, modeling_dispatcher.py:265)."""
    cfg = cfg or DispatcherConfig()
    g = torch.Generator().manual_seed(int(seed))
    sd = {}
    for name, shape, kind in state_dict_keys(cfg):
        if kind == "normal":
            t = torch.empty(shape).normal_(0.0, 0.02, generator=g)
        elif kind == "w1s":
            t = (torch.empty(shape).normal_(0.0, 0.02, generator=g)
                 if nondegenerate else torch.zeros(shape))
        elif kind.startswith("bias_"):
            base = {"bias_i": cfg.gate_bias_flat, "bias_f": cfg.gate_fbias_flat,
                    "bias_r": 2.0}[kind]
            t = torch.full(shape, float(base))
            if nondegenerate:
                t = t + torch.empty(shape).normal_(0.0, 1.0, generator=g)
        elif kind == "norm":
            t = torch.ones(shape)
            if nondegenerate:
                t = t + torch.empty(shape).normal_(0.0, 0.1, generator=g)
        else:
            raise AssertionError(kind)
        sd[name] = t.to(dtype)
    sd["lm_head.weight"] = sd["embedding.weight"]
    return sd
