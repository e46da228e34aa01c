"""`fast_generate` on the B200 decoder (modeling_dispatcher.py:379-442).

Identical sampling semantics: temperature floor 1e-6, top-k by k-th value,
multinomial or argmax, eos freezing, stop at max_len.  The decoder names
of the reference ("auto", "eager", "graphed", "fused") are accepted; all of
them run the B200 decoder, since that is the only compute path here.
"""

import torch
import torch.nn.functional as F

from .decoding import FusedGraphedHybridDecoder, select_greedy  # noqa: F401 (re-exported)

def masked_logits(logits, temperature=1.0, top_k=None):
    """fp32 logits over max(T, 1e-6) with every logit below the k-th largest
    set to -inf (modeling_dispatcher.py:427-430)."""
    logits = logits.float() / max(temperature, 1e-6)
    if top_k is not None:
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    return logits


def sampling_distribution(logits, temperature=1.0, top_k=None):
    """(B, vocab) probabilities a sampled next token is drawn from
    (modeling_dispatcher.py:427-432)."""
    return F.softmax(masked_logits(logits, temperature, top_k), dim=-1)


def select_top_k(top_k, temperature=1.0, seed=None):
    """Token choice for lockstep_loop: a draw from softmax(logits / T) over
    the logits >= the top_k-th largest (ties kept, the reference's mask,
    modeling_dispatcher.py:427-432), as a Gumbel-max.  Inside the loop's
    graph it runs as one device kernel (dh_decode_sample_top_k, uniforms
    from a hash of seed, position, row and index); called directly (the
    loop's first token) it uses torch's generator.  Same distribution as
    the reference's multinomial; the draws themselves differ."""
    inv_t = 1.0 / max(temperature, 1e-6)

    def select(logits):
        lf = logits.float()
        kth = torch.topk(lf, top_k, dim=-1).values[:, -1:]
        u = torch.rand(lf.shape, device=lf.device).clamp_(min=1e-20)
        z = torch.where(lf >= kth, lf * inv_t - torch.log(-torch.log(u)),
                        torch.full_like(lf, float("-inf")))
        return z.argmax(-1)
    select.top_k, select.temperature = top_k, temperature
    select.seed = int(seed if seed is not None else torch.initial_seed()) & (2 ** 64 - 1)
    return select


DECODERS = {"fused": FusedGraphedHybridDecoder, "graphed": FusedGraphedHybridDecoder,
            "eager": FusedGraphedHybridDecoder, "b200": FusedGraphedHybridDecoder}


@torch.no_grad()
def fast_generate(model, input_ids, max_new_tokens=50, do_sample=False, temperature=1.0,
                  top_k=None, eos_token_id=None, num_return_sequences=1, decoder="auto"):
    ids = input_ids.view(1, -1) if input_ids.dim() == 1 else input_ids
    if num_return_sequences > 1:
        if ids.shape[0] != 1:
            raise ValueError("num_return_sequences needs a single prompt")
        if not do_sample:
            raise ValueError("num_return_sequences without sampling would "
                             "return identical rows")
        ids = ids.expand(num_return_sequences, -1)
    if decoder == "auto":
        dec = FusedGraphedHybridDecoder(model)
    elif isinstance(decoder, str):
        if decoder not in DECODERS:
            raise KeyError(decoder)
        dec = DECODERS[decoder](model)
    else:
        dec = decoder
    Bb = ids.shape[0]
    logits = dec.prefill(ids)[:, -1]
    finished = torch.zeros(Bb, dtype=torch.bool, device=ids.device)
    out = [ids]
    for _ in range(max_new_tokens):
        logits = masked_logits(logits, temperature, top_k)
        nxt = (torch.multinomial(F.softmax(logits, dim=-1), 1)[:, 0] if do_sample
               else logits.argmax(-1))
        nxt = nxt.to(ids.device)
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
