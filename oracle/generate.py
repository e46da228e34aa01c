"""Restatement of `fast_generate`'s sampling loop (test oracle).

dispatcher_hybrid/modeling_dispatcher.py:379-442, with the decoder passed in
instead of chosen by name.
"""

import torch
import torch.nn.functional as F


def masked_logits(logits, temperature=1.0, top_k=None):
    """fp32 logits over max(T, 1e-6), every logit below the k-th largest set
    to -inf (modeling_dispatcher.py:427-430)."""
    logits = logits.float() / max(temperature, 1e-6)
    if top_k is not None:
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    return logits


def sampling_probs(logits, temperature=1.0, top_k=None):
    """The distribution a sampled token is drawn from (:427-432)."""
    return F.softmax(masked_logits(logits, temperature, top_k), dim=-1)


@torch.no_grad()
def fast_generate(dec, input_ids, max_new_tokens=50, do_sample=False,
                  temperature=1.0, top_k=None, eos_token_id=None,
                  num_return_sequences=1):
    ids = input_ids.view(1, -1) if input_ids.dim() == 1 else input_ids   # :397
    if num_return_sequences > 1:                                        # :398-404
        if ids.shape[0] != 1:
            raise ValueError("num_return_sequences needs a single prompt")
        if not do_sample:
            raise ValueError("num_return_sequences without sampling would "
                             "return identical rows")
        ids = ids.expand(num_return_sequences, -1)
    Bb = ids.shape[0]
    logits = dec.prefill(ids)[:, -1]                                    # :423
    finished = torch.zeros(Bb, dtype=torch.bool, device=ids.device)
    out = [ids]
    for _ in range(max_new_tokens):                                     # :426-441
        logits = masked_logits(logits, temperature, top_k)
        nxt = (torch.multinomial(F.softmax(logits, dim=-1), 1)[:, 0] if do_sample
               else logits.argmax(-1))
        if eos_token_id is not None:
            nxt = torch.where(finished, torch.full_like(nxt, eos_token_id), nxt)
            finished = finished | (nxt == eos_token_id)
        out.append(nxt.unsqueeze(1))
        if eos_token_id is not None and bool(finished.all()):
            break
        if dec.t >= dec.max_len:
            break
        logits = dec.step(nxt)
    return torch.cat(out, dim=1)
