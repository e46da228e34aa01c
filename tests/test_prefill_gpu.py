"""Whole-model parallel forward (prefill) on the B200 engine against the
oracle; the reference's own invariants (tests/test_parity.py of the
reference): exact causality, bounded cross-document influence."""

import pytest
import torch

import oracle
from dispatcher_b200 import (DispatcherHybridForCausalLM, DispatcherConfig, small_config,
                             make_state_dict)
from tests.helpers import bf16_bound, cast_sd, decisive_argmax_ok, max_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    cfg = small_config()
    sd = make_state_dict(cfg, seed=1, nondegenerate=True)
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    return cfg, model, sd


@pytest.mark.parametrize("B,T,eots", [(2, 160, ((1, 57), (1, 130))), (1, 1, ()), (3, 37, ()),
                                      (2, 256, ((0, 0), (1, 255))), (1, 129, ((0, 64),))])
def test_forward_matches_oracle(small, B, T, eots):
    cfg, model, sd = small
    g = torch.Generator().manual_seed(B * 1000 + T)
    ids = torch.randint(0, cfg.vocab_size - 1, (B, T), generator=g)
    for b, t in eots:
        ids[b, t] = cfg.eot_token
    ref32 = oracle.forward(sd, cfg, ids)
    ref16 = oracle.forward(cast_sd(sd, torch.bfloat16), cfg, ids).float()
    got = model(ids.cuda()).logits.float().cpu()
    err = max_err(got, ref32)
    assert err < bf16_bound(ref32, ref16), err
    ok, agree = decisive_argmax_ok(got, ref32, err)
    assert ok, agree


def test_causality_exact(small):
    """Poking token t leaves every logit before t bit-identical
    (tests/test_parity.py:30-41 of the reference)."""
    cfg, model, _ = small
    torch.manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size - 1, (1, 256)).cuda()
    base = model(ids).logits.clone()
    for cut in (17, 128, 255):
        poked = ids.clone()
        poked[0, cut] = (poked[0, cut] + 79) % (cfg.vocab_size - 1)
        after = model(poked).logits
        assert torch.equal(after[0, :cut], base[0, :cut]), f"future leak at t={cut}"


def test_doc_reset_bounds_cross_document_flow(small):
    cfg, model, _ = small
    torch.manual_seed(1)
    eot = cfg.eot_token
    tail = torch.randint(0, eot, (1, 64))
    a = torch.cat([torch.randint(0, eot, (1, 64)), torch.tensor([[eot]]), tail], 1).cuda()
    b = torch.cat([torch.randint(0, eot, (1, 64)), torch.tensor([[eot]]), tail], 1).cuda()
    la = model(a).logits[0, 65:].float()
    lb = model(b).logits[0, 65:].float()
    assert (la - lb).abs().max().item() < 20.0


def test_enable_fused_gates_contract(small):
    cfg, model, _ = small
    assert model.enable_fused_gates() is model
    assert all(b.mixer.use_fused_gates for b in model.blocks if hasattr(b, "mixer"))


@pytest.mark.slow
def test_full_config_forward():
    cfg = DispatcherConfig()
    sd = make_state_dict(cfg, seed=1, nondegenerate=True)
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (1, 300), generator=g)
    ids[0, 100] = cfg.eot_token
    ref32 = oracle.forward(sd, cfg, ids)
    ref16 = oracle.forward(cast_sd(sd, torch.bfloat16), cfg, ids).float()
    got = model(ids.cuda()).logits.float().cpu()
    err = max_err(got, ref32)
    assert err < bf16_bound(ref32, ref16), err
    ok, agree = decisive_argmax_ok(got, ref32, err)
    assert ok and agree > 0.9, agree
