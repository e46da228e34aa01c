"""Put the B200 backend behind the reference's own model object.

    from dispatcher_hybrid import DispatcherHybridForCausalLM     # the reference
    from dispatcher_b200 import integration
    model = DispatcherHybridForCausalLM(cfg).to("cuda", torch.bfloat16)
    integration.install(model)
    model.enable_fused_gates()          # mixer gate readout -> dh_gate_preacts_fwd/bwd
    model.fast_generate(ids, decoder="fused")   # -> the B200 decoder

`install(model)` rebinds, in the package the model's class comes from, the
three names the reference looks up at call time:

- `<pkg>.fused_gates.fused_gate_preacts`, which the mixer imports inside its
  forward when `use_fused_gates and x.is_cuda`
  (modeling_dispatcher.py:90-99), to this package's differentiable op (the
  tcgen05 forward and backward kernels);
- the CUDA kernels of the reference's custom ops `dispatcher::gate_preacts_fwd`
  and `dispatcher::gate_preacts_bwd` (fused_gates.py:186-263), when that
  module has registered them, so a caller of `torch.ops.dispatcher.*` reaches
  the same kernels (their fake impls and the autograd rule stay the
  reference's);
- `<pkg>.decoding.FusedGraphedHybridDecoder` (and `GraphedHybridDecoder`),
  which `fast_generate` imports inside its body and lists in `choices`
  (modeling_dispatcher.py:406-420), to this package's decoder.

Nothing here imports the reference: the package is found from the model
object.  If the reference's fused_gates module cannot be imported (it needs
triton), a stand-in module holding only `fused_gate_preacts` takes its place
in `sys.modules`.  `uninstall()` puts every rebound name back.
"""

import importlib
import sys
import types

import torch

from . import ops
from .decoding import FusedGraphedHybridDecoder
from .fused_gates import fused_gate_preacts

_saved = []          # (object, attribute, previous value or _MISSING)
_kernels = []        # the reference op kernels registered here
_MISSING = object()


def _set(obj, name, value):
    _saved.append((obj, name, getattr(obj, name, _MISSING)))
    setattr(obj, name, value)


def _package_of(model):
    mod = type(model).__module__
    if "." not in mod:
        raise ValueError(f"cannot find the reference package of {type(model).__name__} "
                         f"(module {mod!r})")
    return mod.rsplit(".", 1)[0]


def _fwd_kernel(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask):
    return list(ops.gate_preacts_fwd(A, B, Wi, Wf, Wr, bi, bf, br, n_lv, mask))


def _bwd_kernel(A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, mask):
    return list(ops.gate_preacts_bwd(A, B, Wi, Wf, Wr, dPi, dPf, dPr, n_lv, mask))


def _reference_op(name):
    ns = getattr(torch.ops, "dispatcher", None)
    if ns is None:
        return None
    try:
        return getattr(ns, name)
    except (AttributeError, RuntimeError):
        return None


def install(model):
    """Route the reference model's fused gate path and its "fused" decoder to
    this package's kernels; returns `model`."""
    pkg = _package_of(model)
    parent = importlib.import_module(pkg)
    # the mixer's gate readout
    fg_name = pkg + ".fused_gates"
    try:
        fg = importlib.import_module(fg_name)
    except Exception:
        fg = types.ModuleType(fg_name)
        fg.__doc__ = "stand-in for the reference's fused_gates: dispatcher_b200 kernels"
        _saved.append((sys.modules, fg_name, sys.modules.get(fg_name, _MISSING)))
        sys.modules[fg_name] = fg
        _set(parent, "fused_gates", fg)
    _set(fg, "fused_gate_preacts", fused_gate_preacts)
    # the reference's custom ops, when its module registered them
    for name, fn in (("gate_preacts_fwd", _fwd_kernel), ("gate_preacts_bwd", _bwd_kernel)):
        if _reference_op(name) is not None and name not in _kernels:
            torch.library.register_kernel(f"dispatcher::{name}", "cuda", fn)
            _kernels.append(name)
    # the decoders fast_generate chooses from
    dec = importlib.import_module(pkg + ".decoding")
    _set(dec, "FusedGraphedHybridDecoder", FusedGraphedHybridDecoder)
    _set(dec, "GraphedHybridDecoder", FusedGraphedHybridDecoder)
    return model


def uninstall():
    """Restore every name `install` rebound (the op kernels stay registered:
    torch.library offers no removal; they serve CUDA tensors only)."""
    while _saved:
        obj, name, old = _saved.pop()
        if obj is sys.modules:
            if old is _MISSING:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = old
        elif old is _MISSING:
            delattr(obj, name)
        else:
            setattr(obj, name, old)
