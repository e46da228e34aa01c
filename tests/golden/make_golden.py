"""Generate the golden fixtures that pin the oracle to the reference itself.

Run from the repository root in a container where the reference package is
importable (it is not needed anywhere else):

    python tests/golden/make_golden.py --reference <path to dispatcher-hybrid-2>

Weights come from `dispatcher_b200.weights.make_state_dict` (seeded, the
reference's init distributions) and are loaded into the reference model with
`load_state_dict`, so the oracle and the kernels can regenerate the identical
weights from the seed alone.  Every output below is produced by the
reference's own code (`DispatcherHybridForCausalLM.forward`,
`DispatcherMixer.forward`, `IncrementalDecoder`) in fp32 on the CPU.
"""

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "dispatcher-hybrid-2_b200"))

from dispatcher_b200.config import small_config  # noqa: E402
from dispatcher_b200.weights import make_state_dict  # noqa: E402

# positions kept from large tensors (every 64th row plus the first few)
FULL_ROWS = np.unique(np.concatenate([np.arange(0, 4), np.arange(0, 1024, 64), [1023]]))


def ref_model(cfg_kwargs, sd):
    from dispatcher_hybrid import DispatcherConfig, DispatcherHybridForCausalLM
    cfg = DispatcherConfig(**cfg_kwargs)
    m = DispatcherHybridForCausalLM(cfg).eval()
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing), (missing, unexpected)
    assert m.lm_head.weight.data_ptr() == m.embedding.weight.data_ptr()
    return m


def small_fixtures(out):
    cfg = small_config()
    ck = cfg.to_dict()
    for tag, seed, nondeg in (("s0", 0, False), ("s1nd", 1, True)):
        sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
        m = ref_model(ck, sd)
        g = torch.Generator().manual_seed(100 + seed)
        ids = torch.randint(0, cfg.vocab_size - 1, (2, 160), generator=g)
        ids[1, 57] = cfg.eot_token            # exercises the doc-reset mask
        ids[1, 130] = cfg.eot_token
        with torch.no_grad():
            logits = m(ids).logits
            # single mixer, layer 0, with the (B, T, L) doc mask
            x = torch.randn(2, 160, cfg.d_model, generator=g)
            mask = m._tree_mask(ids, 160)
            cap = {}
            mx = m.blocks[0].mixer
            hk = mx.linear_out.register_forward_pre_hook(lambda mod, a: cap.setdefault("V", a[0].clone()))
            y = mx(x, mask)
            hk.remove()
        out[f"small_{tag}_ids"] = ids.numpy()
        out[f"small_{tag}_logits"] = logits.numpy()
        out[f"small_{tag}_mix_x"] = x.numpy()
        out[f"small_{tag}_mix_V"] = cap["V"].numpy()
        out[f"small_{tag}_mix_out"] = y.numpy()

        # exact incremental decoder: prefill 40, then 10 steps
        from dispatcher_hybrid.decoding import IncrementalDecoder
        g2 = torch.Generator().manual_seed(200 + seed)
        prompt = torch.randint(0, cfg.vocab_size - 1, (2, 40), generator=g2)
        nexts = torch.randint(0, cfg.vocab_size - 1, (2, 10), generator=g2)
        dec = IncrementalDecoder(m)
        pl = dec.prefill(prompt)
        tree = dec.caches[0]
        out[f"small_{tag}_dec_prompt"] = prompt.numpy()
        out[f"small_{tag}_dec_nexts"] = nexts.numpy()
        out[f"small_{tag}_dec_prefill_logits"] = pl.numpy()
        out[f"small_{tag}_dec_ring_after_prefill"] = tree.V_ring.numpy().copy()
        out[f"small_{tag}_dec_rg_after_prefill"] = tree.rg_hist[:, :40].numpy().copy()
        steps = [dec.step(nexts[:, j]) for j in range(10)]
        out[f"small_{tag}_dec_step_logits"] = torch.stack(steps, 1).numpy()
        out[f"small_{tag}_dec_ring_after_steps"] = tree.V_ring.numpy().copy()
        out[f"small_{tag}_dec_Bhist_after_steps"] = tree.B_hist[:, :50].numpy().copy()
        out[f"small_{tag}_dec_rg_after_steps"] = tree.rg_hist[:, :50].numpy().copy()
        att = dec.caches[1]
        out[f"small_{tag}_dec_k_after_steps"] = att.k[:, :50].numpy().copy()
        out[f"small_{tag}_dec_v_after_steps"] = att.v[:, :50].numpy().copy()

        # doc-separator rejection message
        bad = prompt.clone()
        bad[0, 5] = cfg.eot_token
        try:
            IncrementalDecoder(m).prefill(bad)
            msg = ""
        except ValueError as e:
            msg = str(e)
        out[f"small_{tag}_dec_eot_error"] = np.array(msg)

        # greedy fast_generate through the eager decoder
        gen = m.fast_generate(prompt[:1, :12], max_new_tokens=8, decoder="eager")
        out[f"small_{tag}_fastgen_greedy"] = gen.numpy()


def full_fixtures(out):
    from dispatcher_b200.config import DispatcherConfig
    cfg = DispatcherConfig()
    ck = cfg.to_dict()
    for tag, seed, nondeg in (("s0", 0, False), ("s1nd", 1, True)):
        sd = make_state_dict(cfg, seed=seed, nondegenerate=nondeg)
        m = ref_model(ck, sd)
        # configuration 1: one tree mixer, B=2, T=1024, x ~ N(0,1) from seed 0
        torch.manual_seed(0)
        x = torch.randn(2, 1024, cfg.d_model)
        mask = m.level_mask(1024)
        mx = m.blocks[0].mixer
        cap = {}
        hk = mx.linear_out.register_forward_pre_hook(lambda mod, a: cap.setdefault("V", a[0].clone()))
        with torch.no_grad():
            y = mx(x, mask)
        hk.remove()
        out[f"full_{tag}_c1_V_rows"] = cap["V"][:, FULL_ROWS].numpy()
        out[f"full_{tag}_c1_out_rows"] = y[:, FULL_ROWS].numpy()
        out[f"full_{tag}_c1_V_sums"] = np.array([cap["V"].double().sum().item(),
                                                 cap["V"].double().abs().sum().item()])
        # whole model, 64 tokens, one row with an EOT
        g = torch.Generator().manual_seed(300 + seed)
        ids = torch.randint(0, 50256, (2, 64), generator=g)
        ids[1, 20] = 50256
        with torch.no_grad():
            logits = m(ids).logits
        out[f"full_{tag}_ids"] = ids.numpy()
        out[f"full_{tag}_last_logits"] = logits[:, -1].numpy()
        out[f"full_{tag}_argmax"] = logits.argmax(-1).numpy()
        # decoder: prefill 48, 4 steps
        from dispatcher_hybrid.decoding import IncrementalDecoder
        dec = IncrementalDecoder(m)
        prompt = ids[:1, :48].clone()
        prompt[prompt == 50256] = 7
        dec.prefill(prompt)
        nexts = torch.tensor([11, 2222, 31337, 50000])
        st = [dec.step(nexts[j:j + 1]) for j in range(4)]
        out[f"full_{tag}_dec_prompt"] = prompt.numpy()
        out[f"full_{tag}_dec_nexts"] = nexts.numpy()
        out[f"full_{tag}_dec_last_step_logits"] = st[-1].numpy()
        out[f"full_{tag}_dec_argmax"] = torch.stack(st, 1).argmax(-1).numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}
    small_fixtures(out)
    full_fixtures(out)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, "
          f"{os.path.getsize(args.out) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
