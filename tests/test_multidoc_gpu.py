"""Multi-document decoding (FusedGraphedHybridDecoder(multi_document=True)):
prompts and fed tokens may contain the document separator of a doc_reset
model.  The reference decoder refuses such prompts (decoding.py:89-98); its
parallel forward masks every tree level across a separator
(modeling_dispatcher.py:311-323), so the decoder must reproduce the forward's
logits on the same multi-document sequence."""

import pytest
import torch

import oracle
from dispatcher_b200 import (DispatcherConfig, DispatcherHybridForCausalLM,
                             FusedGraphedHybridDecoder, small_config, make_state_dict)
from tests.helpers import bf16_bound, cast_sd, decisive_argmax_ok, max_err

pytestmark = pytest.mark.gpu


def _ids_with_separators(cfg, batch, length, seps, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size - 1, (batch, length), generator=g)
    for b, t in seps:
        ids[b, t] = cfg.eot_token
    return ids


def _decode(dec, ids, prompt, stepwise=False):
    first = (dec.prefill_stepwise if stepwise else dec.prefill)(ids[:, :prompt])[:, -1]
    got = [first.float()]
    for i in range(ids.shape[1] - prompt - 1):
        got.append(dec.step(ids[:, prompt + i]).float())
    return torch.stack(got, dim=1).cpu()


@pytest.fixture(scope="module")
def small():
    cfg = small_config()
    assert cfg.doc_reset
    sd32 = make_state_dict(cfg, seed=1, nondegenerate=True)
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    return cfg, model.eval(), sd32


@pytest.mark.parametrize("stepwise,batch", [(False, 2), (True, 2), (False, 4)])
def test_multi_document_decode_matches_oracle_forward(small, stepwise, batch):
    """batch 4 takes the tensor-core tree step (document mask in the gate
    operand and in the recurrence)."""
    cfg, model, sd32 = small
    prompt, total = 60, 72
    # separators in the prompt (one pair back to back) and among the fed tokens
    seps = ((0, 10), (1, 33), (1, 34), (0, 63), (1, 70)) + ((3, 5), (3, 66))[:2 * (batch > 2)]
    ids = _ids_with_separators(cfg, batch, total, seps, 5)
    ref32 = oracle.forward(sd32, cfg, ids)[:, prompt - 1:total - 1]
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), cfg, ids)[:, prompt - 1:total - 1].float()
    dec = FusedGraphedHybridDecoder(model, multi_document=True)
    got = _decode(dec, ids, prompt, stepwise)
    assert int(dec.status.item()) == 0
    err = max_err(got, ref32)
    assert err < bf16_bound(ref32, ref16), err
    ok, agree = decisive_argmax_ok(got, ref32, err)
    assert ok, agree


def test_separator_changes_the_continuation(small):
    """The same tokens with and without a separator before them decode
    differently: the mask really cuts the history."""
    cfg, model, _ = small
    a = _ids_with_separators(cfg, 1, 40, (), 9)
    b = a.clone()
    b[0, 20] = cfg.eot_token
    la = _decode(FusedGraphedHybridDecoder(model, multi_document=True), a, 30)
    lb = _decode(FusedGraphedHybridDecoder(model, multi_document=True), b, 30)
    assert max_err(la, lb) > 1e-2


def test_default_decoder_still_refuses_separators(small):
    cfg, model, _ = small
    ids = _ids_with_separators(cfg, 1, 20, ((0, 5),), 3)
    with pytest.raises(ValueError):
        FusedGraphedHybridDecoder(model).prefill(ids.cuda())
    with pytest.raises(ValueError):
        FusedGraphedHybridDecoder(model, step_kernel="persistent", multi_document=True)


def test_multi_document_full_config_matches_forward():
    cfg = DispatcherConfig()
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    prompt, total = 600, 610
    ids = _ids_with_separators(cfg, 2, total, ((0, 200), (1, 450), (0, 603)), 11).cuda()
    want = model(ids).logits[:, prompt - 1:total - 1].float().cpu()
    got = _decode(FusedGraphedHybridDecoder(model, multi_document=True), ids, prompt)
    err = max_err(got, want)
    assert err < 1.0, err     # the reference's bf16 decoder-vs-forward bound
    ok, agree = decisive_argmax_ok(got, want, err)
    assert ok, agree
