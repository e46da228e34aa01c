"""Shared helpers for the parity tests.

Tolerance rule for bf16 kernels (stated once, used everywhere): the B200
result is compared with the fp32 oracle, and its max |error| must stay
within  2 x (max |error| of the oracle's own bf16 eager run) + 0.02,
i.e. within the rounding noise of the reference's bf16 path.  Argmax must
agree wherever the fp32 top-2 margin exceeds 0.75 (the reference's own
"decisive margin" rule, tests/test_decoding.py:61-68 of the reference) or
exceeds 4x the measured error, whichever is smaller.
"""

import torch

DECISIVE = 0.75


def max_err(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def bf16_bound(ref32, ref16):
    return 2.0 * max_err(ref16, ref32) + 0.02


def decisive_argmax_ok(got, ref32, err):
    ref = ref32.float().cpu()
    got = got.float().cpu()
    top2 = torch.topk(ref, 2, dim=-1).values
    margin = top2[..., 0] - top2[..., 1]
    decisive = margin > min(DECISIVE, max(4 * err, 1e-3))
    agree = got.argmax(-1) == ref.argmax(-1)
    return bool((agree | ~decisive).all()), float(agree.float().mean())


def cast_sd(sd, dtype):
    out = {k: v.to(dtype) for k, v in sd.items()}
    out["lm_head.weight"] = out["embedding.weight"]
    return out
