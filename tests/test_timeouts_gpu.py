"""The failure path of the bounded device-side waits, without a GPU fault.

`dh_set_wait_limit(0)` makes every wait that reports a timeout give up at its
first poll.  Each kernel must then return (never hang), issue no further
copies or MMAs, leave DH_ERR_TIMEOUT in its status word, and leave the
context usable: the next call with the default limit is correct.  With the
limit at 0 the GEMM and gate producers give up before their first copy and
the MMA warps are released only by a successful wait; the decode GEMVs'
producer issues its first ring of bulk copies before any wait and drains
them (with a fixed bound) before the kernel returns.  So these launches read
and write only their own buffers and leave nothing in flight.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from dispatcher_b200 import DispatcherHybridForCausalLM, ops, small_config  # noqa: E402
from dispatcher_b200._lib import DispatcherB200Error, call  # noqa: E402

DH_ERR_TIMEOUT = 4


class wait_limit:
    def __init__(self, polls):
        self.polls = polls

    def __enter__(self):
        call("dh_set_wait_limit", self.polls)

    def __exit__(self, *exc):
        torch.cuda.synchronize()
        call("dh_set_wait_limit", -1)


def test_gemm_gives_up_then_recovers():
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(512, 1024, device="cuda", generator=g).bfloat16()
    w = torch.randn(768, 1024, device="cuda", generator=g).bfloat16()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    with wait_limit(0):
        ops.gemm(a, w, status=st)
    assert int(st.item()) == DH_ERR_TIMEOUT
    st.zero_()
    out = ops.gemm(a, w, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = a.float() @ w.float().T
    assert ((out.float() - ref).abs().max() / ref.abs().max()).item() < 8e-3


def test_gate_kernel_gives_up_then_recovers():
    b, T, gh, H, L = 2, 300, 256, 4, 9
    g = torch.Generator(device="cuda").manual_seed(4)
    A = (torch.randn(b, T, gh, device="cuda", generator=g) * 0.5).bfloat16()
    B = (torch.randn(b, T, gh, device="cuda", generator=g) * 0.5).bfloat16()
    W = [(torch.randn(L, H, gh, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(3)]
    bias = [torch.randn(L, H, device="cuda", generator=g) for _ in range(3)]
    n_lv = 9
    wg, bias_np, NP = ops.pack_gate_weights(*W, *bias)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    with wait_limit(0):
        ops.mixer_gates(A.view(b * T, gh), B.view(b * T, gh), wg, bias_np, NP, H, L, n_lv, b,
                        status=st)
    assert int(st.item()) == DH_ERR_TIMEOUT
    st.zero_()
    got = ops.mixer_gates(A.view(b * T, gh), B.view(b * T, gh), wg, bias_np, NP, H, L, n_lv, b,
                          status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    want = ops.mixer_gates(A.view(b * T, gh), B.view(b * T, gh), wg, bias_np, NP, H, L, n_lv, b)
    assert torch.equal(got, want)


def test_prefill_raises_on_timeout_and_recovers():
    """The user-facing path: a forward whose waits gave up raises
    DispatcherB200Error (at the latest when its status is checked), and the
    next forward is correct."""
    cfg = small_config()
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (2, 64), generator=torch.Generator().manual_seed(0))
    ids = ids.cuda()
    good = model(ids).logits.clone()
    model._engine.check_status(sync=True)
    with wait_limit(0):
        model(ids)
    with pytest.raises(DispatcherB200Error, match="DH_ERR_TIMEOUT"):
        model._engine.check_status(sync=True)
    again = model(ids).logits
    model._engine.check_status(sync=True)
    assert torch.equal(again, good)


def test_decode_gemv_gives_up_then_recovers():
    """The lockstep decode's tensor-core GEMVs (bulk-copy weight ring): a
    step graph captured with the limit at 0 reports DH_ERR_TIMEOUT through
    the decoder's status word; a decoder captured with the default limit
    then gives the same logits as one that never saw a timeout."""
    from dispatcher_b200 import FusedGraphedHybridDecoder
    cfg = small_config()
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size - 1, (4, 40), generator=torch.Generator().manual_seed(2))
    ids = ids.cuda()
    ref = FusedGraphedHybridDecoder(model)
    ref.prefill(ids)
    want = ref.step(ids[:, -1])
    ref.check_status(sync=True)
    bad = FusedGraphedHybridDecoder(model)
    bad.prefill(ids)
    bad.check_status(sync=True)
    with wait_limit(0):
        bad._capture()          # the step graph bakes in the limit of its launches
    bad.step(ids[:, -1])
    with pytest.raises(DispatcherB200Error, match="DH_ERR_TIMEOUT"):
        bad.check_status(sync=True)
    good = FusedGraphedHybridDecoder(model)
    good.prefill(ids)
    got = good.step(ids[:, -1])
    good.check_status(sync=True)
    assert (got.float() - want.float()).abs().max().item() < 1e-2


def test_persistent_step_gives_up_then_recovers():
    """The persistent step kernel (step_kernel="persistent"): with the limit at
    0 every hand-off spin and every ring wait gives up at its first poll, the
    kernel returns with DH_ERR_TIMEOUT in the status word (raised by the
    decoder), and a fresh decoder is correct afterwards."""
    from dispatcher_b200 import FusedGraphedHybridDecoder
    cfg = small_config()
    model = DispatcherHybridForCausalLM(cfg, seed=1, nondegenerate=True).to("cuda", torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size - 1, (1, 40), generator=torch.Generator().manual_seed(4))
    ids = ids.cuda()
    ref = FusedGraphedHybridDecoder(model, step_kernel="persistent")
    ref.prefill(ids)
    assert ref.persistent
    want = ref.step(ids[:, -1])
    ref.check_status(sync=True)
    bad = FusedGraphedHybridDecoder(model, step_kernel="persistent")
    bad.prefill(ids)
    bad.check_status(sync=True)
    with wait_limit(0):       # launches read the limit (a captured graph keeps it)
        bad._capture()
        bad.step(ids[:, -1])
    with pytest.raises(DispatcherB200Error, match="DH_ERR_TIMEOUT"):
        bad.check_status(sync=True)
    good = FusedGraphedHybridDecoder(model, step_kernel="persistent")
    good.prefill(ids)
    got = good.step(ids[:, -1])
    good.check_status(sync=True)
    assert (got.float() - want.float()).abs().max().item() < 1e-2
