"""Differentiable gate readout, the drop-in for the reference's
`fused_gate_preacts` (fused_gates.py:176-314): two `torch.library` custom
ops, forward and backward, wired together with `register_autograd`, so the
op stays opaque to torch.compile as the reference's does.

    pre_i, pre_f, pre_r = fused_gate_preacts(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask)

Forward: the tcgen05 gate kernel (`dh_gate_preacts_fwd`); backward: the
tcgen05 backward kernel (`dh_gate_preacts_bwd`).  Gradient dtypes follow the
reference's autograd rule (fused_gates.py:283-300): dA, dB in bf16, dW and db
in fp32, padded with zeros to the weights' full level count.
"""

from typing import List, Optional

import torch

from . import ops


@torch.library.custom_op("dispatcher_b200::gate_preacts_fwd", mutates_args=())
def _gate_preacts_fwd_op(A: torch.Tensor, B: torch.Tensor, Wi: torch.Tensor, Wf: torch.Tensor,
                         Wr: torch.Tensor, bi: torch.Tensor, bf: torch.Tensor, br: torch.Tensor,
                         n_lv: int, mask: Optional[torch.Tensor]) -> List[torch.Tensor]:
    outs = ops.gate_preacts_fwd(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask)
    return [outs[0], outs[1], outs[2]]


@_gate_preacts_fwd_op.register_fake
def _(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask):
    b, T, _ = A.shape
    H = Wi.shape[1]
    return [torch.empty(b, T, n_lv, H, device=A.device, dtype=torch.bfloat16) for _ in range(3)]


@torch.library.custom_op("dispatcher_b200::gate_preacts_bwd", mutates_args=())
def _gate_preacts_bwd_op(A: torch.Tensor, B: torch.Tensor, Wi: torch.Tensor, Wf: torch.Tensor,
                         Wr: torch.Tensor, dPi: torch.Tensor, dPf: torch.Tensor,
                         dPr: torch.Tensor, n_lv: int,
                         mask: Optional[torch.Tensor]) -> List[torch.Tensor]:
    return ops.gate_preacts_bwd(A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, mask)


@_gate_preacts_bwd_op.register_fake
def _(A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, mask):
    b, T, gh = A.shape
    H = Wi.shape[1]
    f32 = lambda *sh: torch.empty(*sh, device=A.device, dtype=torch.float32)  # noqa: E731
    return [f32(b, T, gh), f32(b, T, gh), f32(n_lv, H, gh), f32(n_lv, H, gh), f32(n_lv, H, gh),
            f32(n_lv, H), f32(n_lv, H), f32(n_lv, H)]


def _setup_context(ctx, inputs, output):
    A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask = inputs
    ctx.save_for_backward(A.to(torch.bfloat16), B.to(torch.bfloat16), Wi, Wf, Wr)
    ctx.n_lv = n_lv
    ctx.mask = mask
    ctx.w_levels = Wi.shape[0]
    ctx.dtypes = (A.dtype, B.dtype, Wi.dtype, bi.dtype)


def _backward(ctx, grads):
    A, B, Wi, Wf, Wr = ctx.saved_tensors
    n_lv, L = ctx.n_lv, ctx.w_levels
    dPi, dPf, dPr = (g if g is not None else torch.zeros(A.shape[0], A.shape[1], n_lv, Wi.shape[1],
                                                         device=A.device, dtype=torch.bfloat16)
                     for g in grads)
    dA, dB, dWi, dWf, dWr, dbi, dbf, dbr = torch.ops.dispatcher_b200.gate_preacts_bwd(
        A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, ctx.mask)

    def pad(g):
        if L == n_lv:
            return g
        out = torch.zeros((L,) + tuple(g.shape[1:]), device=g.device, dtype=g.dtype)
        out[:n_lv] = g
        return out

    return (dA.to(torch.bfloat16), dB.to(torch.bfloat16), pad(dWi), pad(dWf), pad(dWr),
            pad(dbi), pad(dbf), pad(dbr), None, None)


torch.library.register_autograd("dispatcher_b200::gate_preacts_fwd", _backward,
                                setup_context=_setup_context)


def fused_gate_preacts(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask=None):
    """(pre_i, pre_f, pre_r), each (b, T, n_lv, H) bf16, differentiable:
    W_x[l] . relu(A + m * roll(B, 2^l))^2 + b_x with the wrap mask in the
    kernel and the optional (b, T, n_lv) doc mask m (fused_gates.py:307-314)."""
    out = torch.ops.dispatcher_b200.gate_preacts_fwd(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask)
    return out[0], out[1], out[2]
