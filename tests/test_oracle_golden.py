"""Pin the CPU oracle to the reference: every golden vector in
tests/golden/golden.npz (produced by the reference package itself, see
tests/golden/make_golden.py) must be reproduced by the oracle restatement.
fp32 on both sides; the bound allows only summation-order noise."""

import numpy as np
import pytest
import torch

import oracle
from dispatcher_b200.config import DispatcherConfig, small_config
from dispatcher_b200.weights import make_state_dict

TAGS = (("s0", 0, False), ("s1nd", 1, True))


def close(got, want, rtol=2e-5, atol=2e-5):
    got = torch.as_tensor(got).double()
    want = torch.as_tensor(np.asarray(want)).double()
    assert got.shape == want.shape, (got.shape, want.shape)
    scale = want.abs().max().item() + 1e-30
    err = (got - want).abs().max().item()
    assert err <= atol + rtol * scale, f"max|d| {err:.3e} (scale {scale:.3e})"


@pytest.mark.parametrize("tag,seed,nondeg", TAGS)
def test_small_forward_and_mixer(golden, tag, seed, nondeg):
    cfg = small_config()
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    ids = torch.from_numpy(golden[f"small_{tag}_ids"])
    close(oracle.forward(sd, cfg, ids), golden[f"small_{tag}_logits"])
    x = torch.from_numpy(golden[f"small_{tag}_mix_x"])
    mask = oracle.tree_mask(ids, cfg.levels, cfg.eot_token, cfg.doc_reset)
    inner = oracle.mixer_internals(sd, "blocks.0.mixer.", cfg.num_heads, cfg.levels, x, mask)
    close(inner["V"], golden[f"small_{tag}_mix_V"])
    close(oracle.mixer_forward(sd, "blocks.0.mixer.", cfg.num_heads, cfg.levels, x, mask),
          golden[f"small_{tag}_mix_out"])


@pytest.mark.parametrize("tag,seed,nondeg", TAGS)
def test_small_decoder_caches(golden, tag, seed, nondeg):
    cfg = small_config()
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    prompt = torch.from_numpy(golden[f"small_{tag}_dec_prompt"])
    nexts = torch.from_numpy(golden[f"small_{tag}_dec_nexts"])
    dec = oracle.OracleDecoder(sd, cfg)
    close(dec.prefill(prompt), golden[f"small_{tag}_dec_prefill_logits"])
    tree = dec.caches[0]
    close(tree.V_ring, golden[f"small_{tag}_dec_ring_after_prefill"])
    close(tree.rg_hist[:, :40], golden[f"small_{tag}_dec_rg_after_prefill"])
    steps = torch.stack([dec.step(nexts[:, j]) for j in range(10)], 1)
    close(steps, golden[f"small_{tag}_dec_step_logits"])
    close(tree.V_ring, golden[f"small_{tag}_dec_ring_after_steps"])
    close(tree.B_hist[:, :50], golden[f"small_{tag}_dec_Bhist_after_steps"])
    close(tree.rg_hist[:, :50], golden[f"small_{tag}_dec_rg_after_steps"])
    close(dec.caches[1].k[:, :50], golden[f"small_{tag}_dec_k_after_steps"])
    close(dec.caches[1].v[:, :50], golden[f"small_{tag}_dec_v_after_steps"])
    assert tree.V_ring.shape[1] == 2 ** (cfg.levels + 1) - 2


@pytest.mark.parametrize("tag,seed,nondeg", TAGS)
def test_small_eot_rejection_and_greedy(golden, tag, seed, nondeg):
    cfg = small_config()
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    prompt = torch.from_numpy(golden[f"small_{tag}_dec_prompt"])
    bad = prompt.clone()
    bad[0, 5] = cfg.eot_token
    with pytest.raises(ValueError, match="document separator"):
        oracle.OracleDecoder(sd, cfg).prefill(bad)
    assert "document separator" in str(golden[f"small_{tag}_dec_eot_error"])
    gen = oracle.fast_generate(oracle.OracleDecoder(sd, cfg), prompt[:1, :12], max_new_tokens=8)
    assert torch.equal(gen, torch.from_numpy(golden[f"small_{tag}_fastgen_greedy"]))


@pytest.mark.slow
@pytest.mark.parametrize("tag,seed,nondeg", TAGS)
def test_full_config_mixer_and_model(golden, tag, seed, nondeg):
    from tests.golden.make_golden import FULL_ROWS
    cfg = DispatcherConfig()
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    torch.manual_seed(0)
    x = torch.randn(2, 1024, cfg.d_model)
    mask = oracle.level_mask(1024, cfg.levels)
    inner = oracle.mixer_internals(sd, "blocks.0.mixer.", cfg.num_heads, cfg.levels, x, mask)
    close(inner["V"][:, FULL_ROWS], golden[f"full_{tag}_c1_V_rows"])
    out = torch.nn.functional.linear(inner["V"], sd["blocks.0.mixer.linear_out.weight"])
    close(out[:, FULL_ROWS], golden[f"full_{tag}_c1_out_rows"])
    ids = torch.from_numpy(golden[f"full_{tag}_ids"])
    logits = oracle.forward(sd, cfg, ids)
    close(logits[:, -1], golden[f"full_{tag}_last_logits"])
    assert torch.equal(logits.argmax(-1), torch.from_numpy(golden[f"full_{tag}_argmax"]))
    dec = oracle.OracleDecoder(sd, cfg)
    dec.prefill(torch.from_numpy(golden[f"full_{tag}_dec_prompt"]))
    nexts = torch.from_numpy(golden[f"full_{tag}_dec_nexts"])
    st = [dec.step(nexts[j:j + 1]) for j in range(4)]
    close(st[-1], golden[f"full_{tag}_dec_last_step_logits"])
    assert torch.equal(torch.stack(st, 1).argmax(-1), torch.from_numpy(golden[f"full_{tag}_dec_argmax"]))


@pytest.mark.parametrize("tag,seed,nondeg", TAGS)
def test_gate_preacts_oracle_matches_pinned_mixer(golden, tag, seed, nondeg):
    """oracle.gate_preacts (the op-level restatement whose fp32 autograd is the
    backward's oracle) equals the pre-activations of the golden-pinned mixer
    restatement on the reference's own inputs."""
    cfg = small_config()
    sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    ids = torch.from_numpy(golden[f"small_{tag}_ids"])
    x = torch.from_numpy(golden[f"small_{tag}_mix_x"])
    mask = oracle.tree_mask(ids, cfg.levels, cfg.eot_token, cfg.doc_reset)
    p = "blocks.0.mixer."
    inner = oracle.mixer_internals(sd, p, cfg.num_heads, cfg.levels, x, mask)
    outs = oracle.gate_preacts(inner["A"], inner["B"], sd[p + "gate_out"], sd[p + "forget_out"],
                               sd[p + "reset_out"], sd[p + "gate_out_bias"],
                               sd[p + "forget_out_bias"], sd[p + "reset_out_bias"],
                               inner["n_lv"], mask)
    for got, name in zip(outs, ("pre_i", "pre_f", "pre_r")):
        close(got, inner[name])
