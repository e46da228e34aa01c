"""Weights in the reference's formats.

Two sources, both handled without the reference package:

* a released model directory (HuggingFace `save_pretrained` layout, as the
  reference's scripts/convert_checkpoint.py writes it): `config.json` with the
  DispatcherConfig fields and `model.safetensors` (or a sharded
  `model.safetensors.index.json`, or `pytorch_model.bin`), the tied embedding
  stored once;
* a research training checkpoint (`torch.save` dict with `args` and
  `model_state_dict`), remapped with the converter's rules
  (scripts/convert_checkpoint.py:25-57): the `mask` buffer is dropped and the
  FFN weights move under the `ffn.` prefix.
"""

import json
import os

import torch

from .config import DispatcherConfig

CONFIG_KEYS = ("vocab_size", "d_model", "num_heads", "dim_feedforward", "num_layers", "max_len",
               "attn_layers", "attn_window", "gate_bias_flat", "gate_fbias_flat", "doc_reset",
               "eot_token")
FFN_KEYS = ("linear_gate", "linear_up", "linear_down")


def config_from_dict(d):
    """DispatcherConfig from a config.json dict (extra HF keys are ignored)."""
    kw = {k: d[k] for k in CONFIG_KEYS if k in d}
    if "attn_layers" in kw:
        kw["attn_layers"] = tuple(kw["attn_layers"])
    return DispatcherConfig(**kw)


def _load_tensors(path):
    st = os.path.join(path, "model.safetensors")
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(st) or os.path.exists(index):
        from safetensors.torch import load_file
        if os.path.exists(st):
            return load_file(st)
        with open(index) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        sd = {}
        for shard in shards:
            sd.update(load_file(os.path.join(path, shard)))
        return sd
    binf = os.path.join(path, "pytorch_model.bin")
    if os.path.exists(binf):
        return torch.load(binf, map_location="cpu", weights_only=True)
    raise FileNotFoundError(f"no model.safetensors, model.safetensors.index.json or "
                            f"pytorch_model.bin in {path}")


def load_pretrained(path):
    """(config, state dict) of a released model directory."""
    with open(os.path.join(path, "config.json")) as f:
        cfg = config_from_dict(json.load(f))
    return cfg, _load_tensors(path)


def remap_research_keys(state_dict):
    """Research checkpoint key -> release key; returns (mapped, dropped)."""
    mapped, dropped = {}, []
    for k, v in state_dict.items():
        if k == "mask":                  # regenerated from max_len
            dropped.append(k)
            continue
        parts = k.split(".")
        if len(parts) >= 3 and parts[0] == "blocks" and parts[2] in FFN_KEYS:
            parts = parts[:2] + ["ffn"] + parts[2:]
        mapped[".".join(parts)] = v
    return mapped, dropped


def config_from_research_args(args, vocab_size):
    attn_layers = args.get("attn_layers") or ""
    if isinstance(attn_layers, str):
        attn_layers = tuple(int(z) for z in attn_layers.split(",") if z)
    return DispatcherConfig(
        vocab_size=vocab_size, d_model=args["d_model"], num_heads=args["num_heads"],
        dim_feedforward=args["dim_feedforward"], num_layers=args["num_layers"],
        max_len=args["bptt"], attn_layers=tuple(attn_layers),
        attn_window=args.get("attn_window") or 0,
        gate_bias_flat=args.get("gate_bias_flat", 0.0),
        gate_fbias_flat=args.get("gate_fbias_flat", 0.0),
        doc_reset=bool(args.get("doc_reset")), eot_token=args.get("eot_token") or 50256)


def load_research_checkpoint(path):
    """(config, state dict) of a research training checkpoint."""
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    sd = ckpt["model_state_dict"]
    cfg = config_from_research_args(ckpt["args"], sd["embedding.weight"].shape[0])
    mapped, _ = remap_research_keys(sd)
    return cfg, mapped


def check_keys(model, state_dict):
    """Load `state_dict` into `model` strictly, except the tied lm_head."""
    missing, unexpected = model.load_state_dict(state_dict, strict=False)
    missing = [k for k in missing if k != "lm_head.weight"]
    if missing or unexpected:
        raise ValueError(f"state dict mismatch\n  missing: {missing}\n  unexpected: {unexpected}")
    return model
