"""Backward of the gate readout (dh_gate_preacts_bwd, the reference op
dispatcher::gate_preacts_bwd, fused_gates.py:96-173, 225-304) against fp32
autograd through the oracle's restatement of the op's math."""

import pytest
import torch

import oracle
from dispatcher_b200 import ops
from dispatcher_b200.fused_gates import fused_gate_preacts

pytestmark = pytest.mark.gpu

NAMES = ("dA", "dB", "dWi", "dWf", "dWr", "dbi", "dbf", "dbr")


def _case(T, with_mask, b=2, H=16, gh=128, L=12, seed=0):
    g = torch.Generator().manual_seed(seed + 7 * T + with_mask)
    n_lv = oracle.n_levels(L, T)
    A = (torch.randn(b, T, gh, generator=g) * 0.5).bfloat16()
    B = (torch.randn(b, T, gh, generator=g) * 0.5).bfloat16()
    W = [(torch.randn(L, H, gh, generator=g) * 0.05).bfloat16() for _ in range(3)]
    bias = [torch.randn(L, H, generator=g) for _ in range(3)]
    dP = [torch.randn(b, T, n_lv, H, generator=g).bfloat16() for _ in range(3)]
    mask = None
    if with_mask:
        ids = torch.randint(0, 100, (b, T), generator=g)
        ids[0, T // 3] = 100
        ids[1, T // 2] = 100
        ids[1, T // 2 + 1] = 100
        mask = oracle.tree_mask(ids, L, 100, True)            # (b, T, L)
    return A, B, W, bias, dP, mask, n_lv


def _autograd(A, B, W, bias, dP, mask, n_lv):
    leaves = [A.float().requires_grad_(), B.float().requires_grad_(),
              *(w.float().requires_grad_() for w in W), *(x.clone().requires_grad_() for x in bias)]
    outs = oracle.gate_preacts(*leaves, n_lv, mask)
    loss = sum((o * d.float()).sum() for o, d in zip(outs, dP))
    return torch.autograd.grad(loss, leaves)


@pytest.mark.parametrize("T,with_mask,H,gh", [
    (200, False, 16, 128), (200, True, 16, 128), (64, False, 16, 128), (1, False, 16, 128),
    (300, True, 16, 128), (1024, False, 16, 128), (200, True, 8, 128), (130, False, 5, 128),
    # the default gate-hidden width (16 slices of 64 columns): dA kept in
    # registers across all levels of a slice, dW / db summed over 16 slices
    (512, False, 16, 1024), (512, True, 16, 1024), (77, True, 8, 1024)])
def test_gate_preacts_bwd_matches_autograd(T, with_mask, H, gh):
    """16 heads: dP rows arrive by TMA; other head counts: per-thread loads."""
    A, B, W, bias, dP, mask, n_lv = _case(T, with_mask, H=H, gh=gh)
    want = _autograd(A, B, W, bias, dP, mask, n_lv)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = ops.gate_preacts_bwd(A.cuda(), B.cuda(), *(w.cuda() for w in W),
                               *(d.cuda() for d in dP), n_lv,
                               mask.cuda() if mask is not None else None, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for name, gv, wv in zip(NAMES, got, want):
        if name.startswith("dW") or name.startswith("db"):
            wv = wv[:n_lv]
        gv = gv.cpu()
        assert gv.shape == wv.shape, name
        # bf16 operands (x and h rounded as the forward rounds them): ~0.5 % of scale
        tol = 0.02 * wv.abs().max().item() + 1e-3
        err = (gv - wv).abs().max().item()
        assert err < tol, (name, err, tol)


def test_fused_gate_preacts_autograd_rules():
    """The differentiable op: forward = the forward kernel; backward gives the
    reference's dtypes (dA, dB bf16) and pads dW, db to all levels."""
    T = 200
    A, B, W, bias, dP, mask, n_lv = _case(T, True)
    L = W[0].shape[0]
    leaves = [A.cuda().requires_grad_(), B.cuda().requires_grad_(),
              *(w.cuda().requires_grad_() for w in W), *(x.cuda().requires_grad_() for x in bias)]
    outs = fused_gate_preacts(*leaves, n_lv, mask.cuda())
    loss = sum((o.float() * d.cuda().float()).sum() for o, d in zip(outs, dP))
    grads = torch.autograd.grad(loss, leaves)
    assert grads[0].dtype == torch.bfloat16 and grads[1].dtype == torch.bfloat16
    assert grads[2].shape == (L, *W[0].shape[1:]) and grads[5].shape == (L, bias[0].shape[1])
    assert not grads[2][n_lv:].any() and not grads[5][n_lv:].any()
    want = _autograd(A, B, W, bias, dP, mask, n_lv)
    for name, gv, wv in zip(NAMES, grads, want):
        gv, wv = gv.float().cpu(), wv
        assert (gv - wv).abs().max().item() < 0.03 * wv.abs().max().item() + 2e-3, name
