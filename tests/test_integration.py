"""The reference-side drop-in (`dispatcher_b200.integration`) installed on the
reference's own model object, on the CPU: which names it rebinds, the
reference op's shapes through its fake implementation, the decoder that
`fast_generate` picks, and that `uninstall` restores everything.  Skipped
where the reference package is not importable."""

import pytest
import torch

from tests.conftest import reference_package

ref = reference_package()
pytestmark = pytest.mark.skipif(ref is None, reason="reference package not importable here")


@pytest.fixture
def ref_model():
    from dispatcher_hybrid import DispatcherConfig, DispatcherHybridForCausalLM
    from dispatcher_b200 import integration
    cfg = DispatcherConfig(vocab_size=100, d_model=64, num_heads=4, dim_feedforward=128,
                           num_layers=3, max_len=64, attn_layers=(2,), attn_window=16,
                           eot_token=99)
    torch.manual_seed(0)
    model = DispatcherHybridForCausalLM(cfg).eval()
    yield integration.install(model)
    integration.uninstall()


def test_install_rebinds_the_reference_lookups(ref_model):
    import sys
    import dispatcher_b200
    from dispatcher_b200.decoding import FusedGraphedHybridDecoder
    fg = sys.modules["dispatcher_hybrid.fused_gates"]
    dec = sys.modules["dispatcher_hybrid.decoding"]
    assert fg.fused_gate_preacts is dispatcher_b200.fused_gate_preacts
    assert dec.FusedGraphedHybridDecoder is FusedGraphedHybridDecoder
    assert dec.GraphedHybridDecoder is FusedGraphedHybridDecoder
    assert ref_model.enable_fused_gates() is ref_model
    assert all(b.mixer.use_fused_gates for b in ref_model.blocks if hasattr(b, "mixer"))


def test_reference_ops_keep_their_fake_shapes(ref_model):
    from torch._subclasses.fake_tensor import FakeTensorMode
    if not hasattr(torch.ops, "dispatcher"):
        pytest.skip("the reference's fused_gates module did not register its ops")
    with FakeTensorMode():
        A = torch.empty(2, 16, 64, device="cuda")
        W = torch.empty(6, 4, 64, device="cuda")
        b = torch.empty(6, 4, device="cuda")
        outs = torch.ops.dispatcher.gate_preacts_fwd(A, A, W, W, W, b, b, b, 5, None)
        assert [tuple(o.shape) for o in outs] == [(2, 16, 5, 4)] * 3
        assert all(o.dtype == torch.bfloat16 for o in outs)
        dP = torch.empty(2, 16, 5, 4, device="cuda", dtype=torch.bfloat16)
        grads = torch.ops.dispatcher.gate_preacts_bwd(A, A, W, W, W, dP, dP, dP, 5, None)
        assert tuple(grads[0].shape) == (2, 16, 64) and tuple(grads[2].shape) == (5, 4, 64)


def test_fast_generate_picks_the_b200_decoder(ref_model):
    ids = torch.tensor([1, 2, 3])
    # "fused" is now this package's decoder, which refuses to run without CUDA
    with pytest.raises(RuntimeError, match="requires CUDA"):
        ref_model.fast_generate(ids, max_new_tokens=2, decoder="fused")
    # "auto" on the CPU falls through to the reference's own eager decoder,
    # as the reference documents (modeling_dispatcher.py:408-416)
    out = ref_model.fast_generate(ids, max_new_tokens=2, decoder="auto")
    assert out.shape == (1, 5) and torch.equal(out[0, :3], ids)


def test_uninstall_restores_the_reference():
    import sys
    from dispatcher_hybrid import DispatcherConfig, DispatcherHybridForCausalLM
    from dispatcher_b200 import integration
    import dispatcher_hybrid.decoding as dec
    before = dec.FusedGraphedHybridDecoder
    fg = sys.modules.get("dispatcher_hybrid.fused_gates")
    fg_before = getattr(fg, "fused_gate_preacts", None) if fg else None
    cfg = DispatcherConfig(vocab_size=100, d_model=64, num_heads=4, dim_feedforward=128,
                           num_layers=2, max_len=64, attn_layers=(), attn_window=16,
                           eot_token=99)
    integration.install(DispatcherHybridForCausalLM(cfg))
    assert dec.FusedGraphedHybridDecoder is not before
    integration.uninstall()
    assert dec.FusedGraphedHybridDecoder is before
    fg = sys.modules.get("dispatcher_hybrid.fused_gates")
    if fg_before is not None:
        assert fg.fused_gate_preacts is fg_before
