"""Device-side weight views for the kernels.

The kernels read weights as bf16 row-major matrices.  Most reference
parameters are used in place (no copy); the projections that share an input
are concatenated once so that one kernel streams them together:

    tree block:      W3   = [linear_in; gate_hidden; gate_hidden_src]  (3d, d)
    attention block: Wqkv = [linear_q; linear_k; linear_v]             (3d, d)

Gate biases are kept in fp32 (the kernels add them in fp32).  A packed set
remembers the parameters' version counters; `stale()` reports an in-place
update of any weight, after which the owner re-packs.
"""

import torch

from .config import DispatcherConfig


def _cfg_of(model):
    cfg = getattr(model, "config", None)
    if cfg is None:
        raise ValueError("model has no .config")
    return cfg


class PackedModel:
    def __init__(self, model, device=None):
        cfg = config_of(model)
        self.cfg = cfg
        params = dict(model.named_parameters())
        sd = {k: v.detach() for k, v in model.state_dict(keep_vars=True).items()}
        emb = sd["embedding.weight"]
        if emb.dtype != torch.bfloat16:
            raise ValueError(
                f"the B200 kernels compute in bfloat16 but the model is {emb.dtype}; "
                f"cast the model first, e.g. model.to(torch.bfloat16)")
        if device is None:
            device = emb.device
        if torch.device(device).type != "cuda":
            raise RuntimeError("the B200 backend needs the model on a CUDA device")
        self.device = torch.device(device)
        self._params = list(params.values())
        self._versions = [p._version for p in self._params]

        def dev(t, dtype=torch.bfloat16):
            return t.to(self.device, dtype).contiguous()

        self.emb = dev(emb)
        self.norm_out = dev(sd["norm_out.weight"])
        self.lm_head = dev(sd["lm_head.weight"]) if "lm_head.weight" in sd else self.emb
        slots = cfg.attn_slots()
        self.layers = []
        for i in range(cfg.num_layers):
            p = f"blocks.{i}."
            lay = dict(kind="attn" if i in slots else "tree",
                       norm1=dev(sd[p + "norm1.weight"]), norm2=dev(sd[p + "norm2.weight"]),
                       w_gate=dev(sd[p + "ffn.linear_gate.weight"]),
                       w_up=dev(sd[p + "ffn.linear_up.weight"]),
                       w_down=dev(sd[p + "ffn.linear_down.weight"]))
            if i in slots:
                a = p + "attn."
                lay["wqkv"] = torch.cat([dev(sd[a + n + ".weight"]) for n in
                                         ("linear_q", "linear_k", "linear_v")], 0).contiguous()
                lay["w_out"] = dev(sd[a + "linear_out.weight"])
            else:
                m = p + "mixer."
                lay["w3"] = torch.cat([dev(sd[m + n + ".weight"]) for n in
                                       ("linear_in", "gate_hidden", "gate_hidden_src")], 0).contiguous()
                lay["w_out"] = dev(sd[m + "linear_out.weight"])
                for g, name in (("i", "gate_out"), ("f", "forget_out"), ("r", "reset_out")):
                    lay["w" + g] = dev(sd[m + name])
                    lay["b" + g] = dev(sd[m + name + "_bias"], torch.float32)
            self.layers.append(lay)

    def stale(self):
        return any(p._version != v for p, v in zip(self._params, self._versions))


def config_of(model):
    cfg = _cfg_of(model)
    # accept any object with the reference config's attributes
    if not hasattr(cfg, "attn_slots"):
        cfg = DispatcherConfig(**{k: getattr(cfg, k) for k in (
            "vocab_size", "d_model", "num_heads", "dim_feedforward", "num_layers", "max_len",
            "attn_layers", "attn_window", "gate_bias_flat", "gate_fbias_flat", "doc_reset",
            "eot_token")})
    return cfg
