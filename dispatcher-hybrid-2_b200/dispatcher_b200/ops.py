"""Thin tensor-level wrappers over the C ABI (bf16 CUDA tensors only).

Each wrapper validates devices/dtypes/contiguity, allocates outputs with
PyTorch (plumbing), passes raw pointers and torch's current stream, and
raises `DispatcherB200Error` on a nonzero status.  No wrapper has a fallback.
"""

import ctypes

import torch

from . import _lib

EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(t, name, dtype=torch.bfloat16):
    if not t.is_cuda:
        raise RuntimeError(f"{name}: B200 kernels need CUDA tensors")
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: innermost dimension must be contiguous")


def gemm(a, w, out=None, epilogue=EPI_STORE, residual=None, status=None):
    """out = a @ w.T (bf16, fp32 accumulate) with an optional fused epilogue.
    a: (M, K) row-strided; w: (N, K).  SwiGLU: w interleaved (see
    `interleave_swiglu`), out (M, N // 2)."""
    _check(a, "a")
    _check(w, "w")
    M, K = a.shape
    N = w.shape[0]
    n_out = N // 2 if epilogue == EPI_SWIGLU else N
    if out is None:
        out = torch.empty(M, n_out, device=a.device, dtype=torch.bfloat16)
    _check(out, "out")
    if epilogue == EPI_RESIDUAL:
        _check(residual, "residual")
    _lib.call("dh_gemm_bf16", _p(a), a.stride(0), _p(w), w.stride(0), _p(out), out.stride(0),
              _p(residual), residual.stride(0) if residual is not None else 0, M, N, K,
              epilogue, _p(status), _stream())
    return out


def interleave_swiglu(w_gate, w_up, block=128):
    """Rows [2*block*j, 2*block*j + block) = gate rows [block*j, block*(j+1)),
    the next block = the matching up rows (layout of dh_gemm_bf16 epilogue 2)."""
    ff, d = w_gate.shape
    if ff % block:
        raise ValueError(f"dim_feedforward {ff} must be a multiple of {block}")
    g = w_gate.reshape(ff // block, block, d)
    u = w_up.reshape(ff // block, block, d)
    return torch.stack([g, u], 1).reshape(2 * ff, d).contiguous()


# ------------------------------------------------------------------ mixer ops
def tree_mask(ids, L, eot_token, doc_reset=True):
    """uint8 (B, T, L) wrap + doc-reset mask (modeling_dispatcher.py:282-323)."""
    if not ids.is_cuda:
        raise RuntimeError("tree_mask: B200 kernels need CUDA tensors")
    ids = ids.to(torch.long).contiguous()
    B, T = ids.shape
    mask = torch.empty(B, T, L, device=ids.device, dtype=torch.uint8)
    _lib.call("dh_tree_mask", _p(ids), B, T, L, int(eot_token), int(bool(doc_reset)), _p(mask),
              _stream())
    return mask


def pack_gate_weights(wi, wf, wr, bi, bf, br):
    """(L, H, gh) x 3 + (L, H) x 3 -> bf16 (L*NP, gh) and fp32 (L, NP), NP = 3H
    rounded up to 16 (rows [l*NP + g*H + h], zero padding)."""
    L, H, gh = wi.shape
    NP = ((3 * H + 15) // 16) * 16
    w = torch.zeros(L, NP, gh, device=wi.device, dtype=torch.bfloat16)
    b = torch.zeros(L, NP, device=wi.device, dtype=torch.float32)
    for g, (ww, bb) in enumerate(((wi, bi), (wf, bf), (wr, br))):
        w[:, g * H:(g + 1) * H] = ww[:L].to(torch.bfloat16)
        b[:, g * H:(g + 1) * H] = bb[:L].float()
    return w.reshape(L * NP, gh).contiguous(), b.contiguous(), NP


def mixer_gates(a, b, wg, bias, NP, H, L, n_lv, batch, mask=None, rg_hist=None, status=None):
    """Sigmoid gates (batch, H, L, T, 4) bf16 from A, B rows (batch*T, gh):
    (admit, forget, transmit, 0) per position, the level sweep's input."""
    _check(a, "a")
    _check(b, "b")
    M, gh = a.shape
    T = M // batch
    gates = torch.empty(batch, H, L, T, 4, device=a.device, dtype=torch.bfloat16)
    _lib.call("dh_mixer_gates", _p(a), a.stride(0), _p(b), b.stride(0), _p(wg), _p(bias),
              _p(mask), batch, T, H, L, NP, gh, n_lv, _p(gates), _p(rg_hist),
              rg_hist.shape[1] if rg_hist is not None else 0, _p(status), _stream())
    return gates


def gate_preacts_fwd(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask=None):
    """Drop-in for the reference's `fused_gate_preacts` (fused_gates.py:307-314):
    A, B (b, T, gh) -> (pre_i, pre_f, pre_r), each (b, T, n_lv, H) bf16,
    pre-sigmoid, wrap mask in-kernel, optional (b, T, n_lv) doc mask."""
    b_, T, gh = A.shape
    H = Wi.shape[1]
    A2 = A.to(torch.bfloat16).reshape(b_ * T, gh).contiguous()
    B2 = B.to(torch.bfloat16).reshape(b_ * T, gh).contiguous()
    wg, bias, NP = pack_gate_weights(Wi[:n_lv], Wf[:n_lv], Wr[:n_lv], bi[:n_lv], bf[:n_lv],
                                     br[:n_lv])
    m8 = None
    if mask is not None:
        m8 = (mask[..., :n_lv] != 0).to(torch.uint8).contiguous()
    outs = [torch.empty(b_, T, n_lv, H, device=A.device, dtype=torch.bfloat16) for _ in range(3)]
    _lib.call("dh_gate_preacts_fwd", _p(A2), gh, _p(B2), gh, _p(wg), _p(bias), _p(m8),
              n_lv, b_, T, H, n_lv, NP, gh, n_lv, _p(outs[0]), _p(outs[1]), _p(outs[2]), None,
              _stream())
    return outs[0], outs[1], outs[2]


def pack_gate_weights_t(wi, wf, wr, n_lv):
    """(L, H, gh) x 3 -> bf16 (n_lv*gh, 64): per level W^T with the 3H gate
    rows (i, f, r) as columns, zero padded to 64 (the backward's K-major
    operand)."""
    H, gh = wi.shape[1], wi.shape[2]
    w = torch.cat([wi[:n_lv], wf[:n_lv], wr[:n_lv]], dim=1).to(torch.bfloat16)  # (n_lv, 3H, gh)
    wt = torch.zeros(n_lv, gh, 64, device=wi.device, dtype=torch.bfloat16)
    wt[:, :, :3 * H] = w.transpose(1, 2)
    return wt.reshape(n_lv * gh, 64).contiguous()


def gate_preacts_bwd(A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, mask=None, status=None):
    """Drop-in for the reference's backward op (fused_gates.py:225-263): the
    gradients of gate_preacts_fwd given dPi, dPf, dPr (b, T, n_lv, H).
    Returns [dA, dB, dWi, dWf, dWr, dbi, dbf, dbr], fp32: dA, dB (b, T, gh),
    dW_x (n_lv, H, gh), db_x (n_lv, H)."""
    b_, T, gh = A.shape
    H = Wi.shape[1]
    dev = A.device
    A2 = A.to(torch.bfloat16).contiguous()
    B2 = B.to(torch.bfloat16).contiguous()
    wt = pack_gate_weights_t(Wi, Wf, Wr, n_lv)
    dps = [d.to(torch.bfloat16).contiguous() for d in (dPi, dPf, dPr)]
    dps = [d if d.data_ptr() % 16 == 0 else d.clone() for d in dps]  # 16-byte row loads
    m8 = None
    if mask is not None:
        m8 = (mask[..., :n_lv] != 0).to(torch.uint8).contiguous()
    f32 = torch.float32
    dA = torch.zeros(b_, T, gh, device=dev, dtype=f32)
    dB = torch.zeros(b_, T, gh, device=dev, dtype=f32)
    dW = [torch.zeros(n_lv, H, gh, device=dev, dtype=f32) for _ in range(3)]
    db = [torch.zeros(n_lv, H, device=dev, dtype=f32) for _ in range(3)]
    _lib.call("dh_gate_preacts_bwd", _p(A2), gh, _p(B2), gh, _p(wt), _p(m8), n_lv, b_, T, H,
              n_lv, gh, _p(dps[0]), _p(dps[1]), _p(dps[2]), _p(dA), _p(dB), _p(dW[0]),
              _p(dW[1]), _p(dW[2]), _p(db[0]), _p(db[1]), _p(db[2]), _p(status), _stream())
    return [dA, dB, *dW, *db]


def level_scan(v0, gates, H, L, n_lv, batch, out=None, ring=None):
    """Level sweep over v0 rows (batch*T, d) -> V (batch*T, d) bf16."""
    _check(v0, "v0")
    M, d = v0.shape
    T = M // batch
    if out is None:
        out = torch.empty(M, d, device=v0.device, dtype=torch.bfloat16)
    _lib.call("dh_level_scan", _p(v0), v0.stride(0), _p(gates), _p(out), out.stride(0), batch,
              T, H, d // H, L, n_lv, _p(ring), _stream())
    return out


def rope_tables(max_len, hd, device):
    theta = 10000.0 ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)
    ang = torch.arange(max_len, dtype=torch.float32)[:, None] * theta[None, :]
    return ang.cos().to(device).contiguous(), ang.sin().to(device).contiguous()


def window_attention(qkv, batch, H, window, rope=True, out=None, status=None):
    """qkv (batch*T, 3d) bf16 (q, k rotated in place when rope) -> (batch*T, d)
    on the tcgen05 attention kernel."""
    _check(qkv, "qkv")
    M, d3 = qkv.shape
    d = d3 // 3
    T = M // batch
    hd = d // H
    if rope:
        cos, sin = rope_tables(T, hd, qkv.device)
        _lib.call("dh_rope_qk", _p(qkv), qkv.stride(0), M, T, d, hd, _p(cos), _p(sin), _stream())
    if out is None:
        out = torch.empty(M, d, device=qkv.device, dtype=torch.bfloat16)
    _lib.call("dh_window_attn_prefill_tc", _p(qkv), qkv.stride(0), _p(out), out.stride(0),
              batch, T, H, hd, window, _p(status), _stream())
    return out
