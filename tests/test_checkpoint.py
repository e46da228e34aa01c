"""Loading weights in the reference's formats: a released model directory
(written here by the reference's own save_pretrained, tests/golden/tiny_ckpt,
made by tests/golden/make_checkpoint.py) and a research training checkpoint
(remapped as scripts/convert_checkpoint.py:25-57 does).  The loaded weights
must reproduce the reference's logits for the fixture's multi-document input
(through the oracle on the CPU, through the B200 engine on the GPU)."""

import os

import numpy as np
import pytest
import torch

import oracle
from dispatcher_b200 import DispatcherHybridForCausalLM
from dispatcher_b200.checkpoint import (load_pretrained, load_research_checkpoint,
                                        remap_research_keys)
from tests.helpers import bf16_bound, cast_sd, decisive_argmax_ok, max_err

CKPT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_ckpt")


@pytest.fixture(scope="module")
def golden_logits():
    z = np.load(os.path.join(CKPT, "reference_logits.npz"))
    return torch.from_numpy(z["ids"]), torch.from_numpy(z["logits"])


def _sd32(model):
    return {k: v.float() for k, v in model.state_dict().items()}


def test_pretrained_directory_loads_every_tensor():
    from safetensors.torch import load_file
    cfg, sd = load_pretrained(CKPT)
    assert (cfg.num_layers, cfg.d_model, cfg.num_heads, cfg.attn_slots()) == (2, 128, 2, {0})
    model = DispatcherHybridForCausalLM.from_pretrained(CKPT)
    raw = load_file(os.path.join(CKPT, "model.safetensors"))
    got = model.state_dict()
    for k, v in raw.items():
        assert torch.equal(got[k], v.float()), k
    assert torch.equal(got["lm_head.weight"], got["embedding.weight"])   # tied


def test_loaded_weights_reproduce_reference_logits(golden_logits):
    ids, want = golden_logits
    model = DispatcherHybridForCausalLM.from_pretrained(CKPT)
    got = oracle.forward(_sd32(model), model.config, ids)
    assert max_err(got, want) < 1e-4


def test_research_checkpoint_is_remapped(tmp_path):
    model = DispatcherHybridForCausalLM.from_pretrained(CKPT)
    cfg = model.config
    research = {}
    for k, v in model.state_dict().items():
        if k == "lm_head.weight":
            continue
        parts = k.split(".")
        if len(parts) >= 4 and parts[2] == "ffn":        # release -> research layout
            parts = parts[:2] + parts[3:]
        research[".".join(parts)] = v.clone()
    research["mask"] = torch.zeros(1)
    mapped, dropped = remap_research_keys(research)
    assert dropped == ["mask"]
    args = dict(d_model=cfg.d_model, num_heads=cfg.num_heads,
                dim_feedforward=cfg.dim_feedforward, num_layers=cfg.num_layers,
                bptt=cfg.max_len, attn_layers="1", attn_window=cfg.attn_window,
                gate_bias_flat=cfg.gate_bias_flat, gate_fbias_flat=cfg.gate_fbias_flat,
                doc_reset=True, eot_token=cfg.eot_token)
    path = tmp_path / "final.pt"
    torch.save({"args": args, "model_state_dict": research}, path)
    cfg2, sd2 = load_research_checkpoint(str(path))
    assert cfg2.to_dict() == cfg.to_dict()
    m2 = DispatcherHybridForCausalLM.from_research_checkpoint(str(path))
    for k, v in model.state_dict().items():
        assert torch.equal(m2.state_dict()[k], v), k


def test_state_dict_mismatch_is_reported(tmp_path):
    from safetensors.torch import load_file, save_file
    import shutil
    bad = tmp_path / "bad"
    shutil.copytree(CKPT, bad)
    sd = load_file(str(bad / "model.safetensors"))
    sd.pop("norm_out.weight")
    save_file(sd, str(bad / "model.safetensors"))
    with pytest.raises(ValueError, match="norm_out.weight"):
        DispatcherHybridForCausalLM.from_pretrained(str(bad))


@pytest.mark.gpu
def test_pretrained_on_b200_matches_reference(golden_logits):
    ids, want = golden_logits
    model = DispatcherHybridForCausalLM.from_pretrained(CKPT, dtype=torch.bfloat16, device="cuda")
    got = model(ids.cuda()).logits.float().cpu()
    sd32 = _sd32(DispatcherHybridForCausalLM.from_pretrained(CKPT))
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), model.config, ids).float()
    err = max_err(got, want)
    assert err < bf16_bound(want, ref16), err
    ok, agree = decisive_argmax_ok(got, want, err)
    assert ok, agree
