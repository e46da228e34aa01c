"""Parity of the B200 decoder with the oracle (the reference's eager decoder
restated), on seeded random-init weights.  Mirrors the reference's
tests/test_decoding.py contract: decoder vs parallel forward, caches and
ring slot positions, batched vs solo rows, error behaviour."""

import pytest
import torch

import oracle
from dispatcher_b200 import (DispatcherHybridForCausalLM, FusedGraphedHybridDecoder,
                             DispatcherConfig, small_config, make_state_dict)
from tests.helpers import bf16_bound, cast_sd, decisive_argmax_ok, max_err

pytestmark = pytest.mark.gpu


def build(cfg, seed, nondeg):
    sd32 = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
    model = DispatcherHybridForCausalLM(cfg, seed=seed, nondegenerate=nondeg)
    model = model.to("cuda", torch.bfloat16).eval()
    return model, sd32


@pytest.fixture(scope="module")
def small_nd():
    return (small_config(),) + build(small_config(), 1, True)


@pytest.fixture(scope="module")
def small_s0():
    return (small_config(),) + build(small_config(), 0, False)


def _compare(cfg, model, sd32, prompt=48, steps=12, seed=0, batch=1):
    """Reference `_compare` (tests/test_decoding.py:33-44): decoder logits at
    positions prompt.. vs the parallel forward's, here against the fp32
    oracle with the bf16 bound measured from the oracle's own bf16 run."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size - 1, (batch, prompt + steps), generator=g)
    ref32 = oracle.forward(sd32, cfg, ids)[:, prompt - 1:]
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), cfg, ids)[:, prompt - 1:].float()
    dec = FusedGraphedHybridDecoder(model)
    pre = dec.prefill(ids[:, :prompt].cuda())
    got = [pre[:, -1].float()]
    for t in range(prompt, prompt + steps):
        got.append(dec.step(ids[:, t].cuda()).float())
    got = torch.stack(got, 1)[:, :-1].cpu()
    ref32, ref16 = ref32[:, :-1], ref16[:, :-1]
    err = max_err(got, ref32)
    bound = bf16_bound(ref32, ref16)
    assert err < bound, f"max|dlogit| {err:.4f} vs fp32 exceeds bf16 bound {bound:.4f}"
    ok, agree = decisive_argmax_ok(got, ref32, err)
    assert ok, f"decisive argmax flip (agreement {agree:.3f})"
    return dec, ids, err, bound


def test_decoder_matches_forward_small_nondegenerate(small_nd):
    _compare(*small_nd)


def test_decoder_matches_forward_small_seed0(small_s0):
    _compare(*small_s0)


@pytest.mark.parametrize("batch,mode", [(3, "fused"), (8, "fused"), (9, "tree_tc")])
def test_decoder_batched(small_nd, batch, mode):
    """Up to 8 rows the tree gate readouts are folded into the W3 GEMV (one
    8-column mma tile of lockstep rows); from 9 rows they are their own
    tensor-core launch over all heads per level, and every GEMV takes two
    8-column tiles."""
    dec = _compare(*small_nd, batch=batch, seed=5)[0]
    assert dec.gates_fused if mode == "fused" else dec.tree_tc


def test_prefill_logits_match_forward(small_nd):
    cfg, model, sd32 = small_nd
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab_size - 1, (2, 70), generator=g)
    ref32 = oracle.forward(sd32, cfg, ids)
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), cfg, ids).float()
    got = FusedGraphedHybridDecoder(model).prefill(ids.cuda()).float().cpu()
    assert max_err(got, ref32) < bf16_bound(ref32, ref16)


def test_caches_and_ring_slots_match_oracle(small_nd):
    """Ring contents, B/rg histories and KV caches after prefill + steps; the
    set of written ring slots must be identical (slot indexing is exact)."""
    cfg, model, sd32 = small_nd
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab_size - 1, (2, 37), generator=g)
    nexts = torch.randint(0, cfg.vocab_size - 1, (2, 9), generator=g)
    ref = oracle.OracleDecoder(sd32, cfg)
    ref.prefill(prompt)
    dec = FusedGraphedHybridDecoder(model)
    dec.prefill(prompt.cuda())
    for j in range(9):
        ref.step(nexts[:, j])
        dec.step(nexts[:, j].cuda())
    T = 37 + 9
    for i, (rc, mc) in enumerate(zip(ref.caches, dec.caches)):
        if hasattr(rc, "V_ring"):
            r_ring, m_ring = rc.V_ring, mc.V_ring.float().cpu()
            # written slots (rows), not elements: a bf16 f*V + a*msg can cancel
            # to exactly zero in one channel where the fp32 oracle does not
            assert torch.equal(r_ring.abs().sum(-1) != 0, m_ring.abs().sum(-1) != 0), \
                f"layer {i}: ring slot pattern differs"
            assert max_err(m_ring, r_ring) < 0.05 * r_ring.abs().max().item() + 1e-2
            assert max_err(mc.B_hist[:, :T].float().cpu(), rc.B_hist[:, :T]) < 0.02 * rc.B_hist.abs().max().item() + 1e-3
            assert max_err(mc.rg_hist[:, :T].float().cpu(), rc.rg_hist[:, :T]) < 0.02
            assert not mc.B_hist[:, T:].any() and not mc.rg_hist[:, T:].any()
        else:
            assert max_err(mc.k[:, :T].float().cpu(), rc.k[:, :T]) < 0.02 * rc.k.abs().max().item() + 1e-3
            assert max_err(mc.v[:, :T].float().cpu(), rc.v[:, :T]) < 0.02 * rc.v.abs().max().item() + 1e-3
            assert not mc.k[:, T:].any()


def test_ring_slot_positions_are_bit_exact(small_nd):
    """After t positions, ring j holds exactly the slots of positions
    max(0, t-2^(j+1)) .. t-1 (decoding.py:63-76); every other slot is zero."""
    cfg, model, _ = small_nd
    L = cfg.levels
    for T in (1, 2, 3, 7, 64, 129):
        ids = torch.randint(0, cfg.vocab_size - 1, (1, T))
        dec = FusedGraphedHybridDecoder(model)
        dec.prefill(ids.cuda())
        ring = dec.caches[0].V_ring[0].float().cpu()
        written = ring.abs().sum(-1) != 0
        expect = torch.zeros_like(written)
        for j in range(L):
            for p in range(max(0, T - 2 ** (j + 1)), T):
                expect[oracle.ring_slot(j, p)] = True
        assert torch.equal(written, expect), f"T={T}: ring slots differ"


def test_batched_equals_solo(small_nd):
    cfg, model, _ = small_nd
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg.vocab_size - 1, (3, 40), generator=g).cuda()
    nexts = torch.randint(0, cfg.vocab_size - 1, (3, 8), generator=g).cuda()
    dec = FusedGraphedHybridDecoder(model)
    batched = [dec.prefill(prompts)[:, -1]]
    batched += [dec.step(nexts[:, j]) for j in range(8)]
    batched = torch.stack(batched, 1).float()
    for b in range(3):
        solo = FusedGraphedHybridDecoder(model)
        s = [solo.prefill(prompts[b])[-1]] + [solo.step(nexts[b, j]) for j in range(8)]
        gap = max_err(torch.stack(s).float(), batched[b])
        assert gap < 0.02, f"row {b}: batched vs solo {gap:.3e}"


def test_errors_match_reference_behaviour(small_nd):
    cfg, model, _ = small_nd
    dec = FusedGraphedHybridDecoder(model, max_len=64)
    bad = torch.tensor([3, 4, cfg.eot_token, 5]).cuda()
    with pytest.raises(ValueError, match="document separator"):
        dec.prefill(bad)
    with pytest.raises(ValueError, match="exceeds max_len"):
        dec.prefill(torch.ones(65, dtype=torch.long).cuda())
    dec.prefill(torch.ones(63, dtype=torch.long).cuda())
    dec.step(torch.tensor([1]).cuda())
    with pytest.raises(ValueError, match="context exhausted"):
        dec.step(torch.tensor([1]).cuda())
    with pytest.raises(ValueError, match="dtype"):
        FusedGraphedHybridDecoder(model, dtype=torch.float32)
    with pytest.raises(ValueError, match="tokens for batch"):
        d2 = FusedGraphedHybridDecoder(model)
        d2.prefill(torch.ones(2, 5, dtype=torch.long).cuda())
        d2.step(torch.ones(3, dtype=torch.long).cuda())


def test_fast_generate_greedy_tracks_oracle(small_nd):
    cfg, model, sd32 = small_nd
    ids = torch.tensor([[464, 118, 286, 262]])
    got = model.fast_generate(ids.cuda(), max_new_tokens=10).cpu()
    # teacher-forced check: each generated token is the fp32 argmax unless
    # the fp32 top-2 margin is inside the bf16 noise
    logits = oracle.forward(sd32, cfg, got[:, :-1])[0, 3:]
    top2 = torch.topk(logits, 2, -1).values
    decisive = (top2[:, 0] - top2[:, 1]) > 0.05
    agree = logits.argmax(-1) == got[0, 4:]
    assert bool((agree | ~decisive).all())
    assert got.shape == (1, 14) and torch.equal(got[:, :4], ids)


def test_fast_generate_sampling_and_eos(small_nd):
    cfg, model, _ = small_nd
    torch.manual_seed(0)
    ids = torch.tensor([[464, 118, 286, 262]]).cuda()
    out = model.fast_generate(ids, max_new_tokens=6, do_sample=True, temperature=0.8, top_k=50,
                              num_return_sequences=3)
    assert out.shape == (3, 10) and (out[:, :4] == ids).all()
    two = torch.randint(0, cfg.vocab_size - 1, (2, 8)).cuda()
    first = int(model.fast_generate(two[:1], max_new_tokens=1)[0, -1])
    out = model.fast_generate(two, max_new_tokens=6, eos_token_id=first)
    assert int(out[0, 8]) == first and (out[0, 8:] == first).all()


@pytest.mark.slow
def test_full_config_decode_vs_oracle():
    """Default 292M config: prefill 48 + 4 steps against the fp32 oracle."""
    cfg = DispatcherConfig()
    model, sd32 = build(cfg, 0, False)
    _compare(cfg, model, sd32, prompt=48, steps=4)
    del model
    model, sd32 = build(cfg, 1, True)
    _compare(cfg, model, sd32, prompt=48, steps=4, seed=1)


def test_engine_prefill_caches_match_stepwise(small_nd):
    """The parallel prefill's cache fill (B_hist, rg_hist of all levels, ring
    slabs, K/V) equals the state built by stepping the prompt one token at a
    time through the decode step: slot pattern exactly, values within bf16."""
    cfg, model, _ = small_nd
    g = torch.Generator().manual_seed(21)
    for T in (1, 5, 64, 100):
        ids = torch.randint(0, cfg.vocab_size - 1, (2, T), generator=g).cuda()
        a = FusedGraphedHybridDecoder(model)
        la = a.prefill(ids).float()
        b = FusedGraphedHybridDecoder(model)
        lb = b.prefill_stepwise(ids).float()
        assert max_err(la, lb) < 0.05, T
        for ca, cb in zip(a.caches, b.caches):
            names = ("B_hist", "rg_hist", "V_ring") if hasattr(ca, "V_ring") else ("k", "v")
            for n in names:
                xa, xb = getattr(ca, n).float(), getattr(cb, n).float()
                # written slots / positions: any nonzero channel (a single bf16
                # channel can legitimately round to 0.0 in one of the two routes)
                wa, wb = xa.abs().flatten(2).sum(-1) != 0, xb.abs().flatten(2).sum(-1) != 0
                if not torch.equal(wa, wb):
                    bad = (wa != wb).nonzero()[:6].tolist()
                    raise AssertionError(f"T={T} {n}: written slots differ at (row, slot) {bad}")
                scale = xb.abs().max().item() + 1e-6
                assert max_err(xa, xb) < 0.03 * scale + 1e-3, f"T={T} {n}"
        nxt = torch.randint(0, cfg.vocab_size - 1, (2,), generator=g).cuda()
        assert max_err(a.step(nxt).float(), b.step(nxt).float()) < 0.05


@pytest.mark.parametrize("kernel", ["graph", "persistent"])
def test_step_kernels_match_oracle(small_nd, kernel):
    """Both step implementations against the fp32 oracle (prompt 40 + 8 steps)."""
    cfg, model, sd32 = small_nd
    g = torch.Generator().manual_seed(17)
    ids = torch.randint(0, cfg.vocab_size - 1, (2, 48), generator=g)
    ref32 = oracle.forward(sd32, cfg, ids)[:, 39:47]
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), cfg, ids)[:, 39:47].float()
    dec = FusedGraphedHybridDecoder(model, step_kernel=kernel)
    got = [dec.prefill(ids[:, :40].cuda())[:, -1].float()]
    got += [dec.step(ids[:, t].cuda()).float() for t in range(40, 47)]
    got = torch.stack(got, 1).cpu()
    assert dec.persistent == (kernel == "persistent")
    assert max_err(got, ref32) < bf16_bound(ref32, ref16)
    assert int(dec.status.item()) == 0


def test_batch_above_16_uses_chunked_kernels(small_nd):
    """Lockstep batches above 16 rows run the per-op kernels in 16-row chunks."""
    cfg, model, sd32 = small_nd
    g = torch.Generator().manual_seed(8)
    ids = torch.randint(0, cfg.vocab_size - 1, (18, 30), generator=g)
    dec = FusedGraphedHybridDecoder(model)
    out = dec.prefill(ids.cuda())
    assert not dec.persistent
    nxt = torch.randint(0, cfg.vocab_size - 1, (18,), generator=g)
    got = dec.step(nxt.cuda()).float().cpu()
    ref = oracle.forward(sd32, cfg, torch.cat([ids, nxt[:, None]], 1))[:, -1]
    ref16 = oracle.forward(cast_sd(sd32, torch.bfloat16), cfg,
                           torch.cat([ids, nxt[:, None]], 1))[:, -1].float()
    assert max_err(got, ref) < bf16_bound(ref, ref16)
    assert out.shape == (18, 30, cfg.vocab_size)


def test_lockstep_loop_matches_stepwise_greedy(small_nd):
    """The captured loop (step kernels + device argmax fed back + token
    gather, one graph per step) picks the same tokens as step() + argmax."""
    from dispatcher_b200.generation import select_greedy, select_top_k
    cfg, model, _ = small_nd
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab_size - 1, (3, 40), generator=g).cuda()
    dec = FusedGraphedHybridDecoder(model)
    tok = dec.prefill(ids)[:, -1].argmax(-1)
    want = [tok]
    for _ in range(10):
        tok = dec.step(tok).argmax(-1)
        want.append(tok)
    dec2 = FusedGraphedHybridDecoder(model)
    dec2.prefill(ids)
    loop = dec2.lockstep_loop(select_greedy)
    got = [dec2.token_buf.clone()]
    for _ in range(10):
        got.append(loop.step().clone())
    assert dec2.t == dec.t
    assert torch.equal(torch.stack(got), torch.stack(want))
    # the FFN adds its CTAs' partial sums with atomics: the fp32 summation
    # order varies between runs, the bf16 logits by about an ulp
    assert (dec2.logits_out.float() - dec.logits_out.float()).abs().max().item() < 2e-2
    # sampled choices stay among each row's logits >= its 5th largest
    dec3 = FusedGraphedHybridDecoder(model)
    dec3.prefill(ids)
    loop = dec3.lockstep_loop(select_top_k(5, 0.8, seed=3))
    for _ in range(6):
        loop.step()
        lg = dec3.logits_out.float()
        kth = torch.topk(lg, 5, dim=-1).values[:, -1]
        assert bool((lg.gather(1, dec3.token_buf[:, None])[:, 0] >= kth).all())


def test_device_argmax_matches_torch_with_ties():
    """dh_decode_argmax: first index of the row maximum, as torch.argmax."""
    import ctypes
    from dispatcher_b200._lib import call
    g = torch.Generator(device="cuda").manual_seed(7)
    B, V = 5, 50257
    lg = (torch.randn(B, V, device="cuda", generator=g) * 3).bfloat16()
    lg[1, 100] = lg[1, 4000] = lg[1].max() + 1       # a tie: the first index wins
    lg[2, V - 1] = 100.0                             # the last column
    lg[3, 0] = 100.0                                 # the first column
    nxt = torch.full((B,), -1, dtype=torch.long, device="cuda")
    out = torch.full((B,), -1, dtype=torch.long, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    call("dh_decode_argmax", p(lg), p(nxt), p(out), B, V,
         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    want = lg.argmax(-1)
    assert torch.equal(nxt, want) and torch.equal(out, want)
    assert int(want[1]) == 100


def _sample(lg, k, temp, seed, t):
    import ctypes
    from dispatcher_b200._lib import call
    B, V = lg.shape
    nxt = torch.full((B,), -1, dtype=torch.long, device="cuda")
    tb = torch.tensor([t], dtype=torch.long, device="cuda")
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    call("dh_decode_sample_top_k", p(lg), p(nxt), None, B, V, k, temp, seed, p(tb),
         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return nxt


def test_device_top_k_sampling_candidates_and_distribution():
    """dh_decode_sample_top_k: every draw is a logit >= the k-th largest
    (ties at the k-th kept, the reference's mask), k = 1 without ties is the
    argmax, and the frequencies follow softmax(logit / T) over the
    candidates."""
    g = torch.Generator(device="cuda").manual_seed(9)
    # coarse values: many ties, also at the k-th largest
    lg = (torch.randint(-20, 20, (6, 50257), device="cuda", generator=g) * 0.25).bfloat16()
    for k in (1, 7, 50, 50257):
        for t in range(3):
            tok = _sample(lg, k, 0.8, 1234, 100 + t)
            kth = torch.topk(lg.float(), k, dim=-1).values[:, -1]
            assert bool((lg.float().gather(1, tok[:, None])[:, 0] >= kth).all()), k
    lg1 = torch.randn(4, 1000, device="cuda", generator=g).bfloat16()
    assert torch.equal(_sample(lg1, 1, 0.8, 5, 7), lg1.argmax(-1))
    # distribution: 64 identical rows x 64 positions = 4096 draws
    V, k, temp = 16, 8, 0.8
    base = torch.linspace(-1.0, 1.5, V, device="cuda").bfloat16()
    rows = base[None].expand(64, V).contiguous()
    counts = torch.zeros(V, device="cuda")
    for t in range(64):
        counts += torch.bincount(_sample(rows, k, temp, 77, t), minlength=V).float()
    freq = counts / counts.sum()
    lf = base.float()
    kth = torch.topk(lf, k).values[-1]
    want = torch.softmax(torch.where(lf >= kth, lf / temp, torch.full_like(lf, float("-inf"))), 0)
    assert (freq - want).abs().max().item() < 0.03, (freq, want)
    assert counts[lf < kth].sum().item() == 0
