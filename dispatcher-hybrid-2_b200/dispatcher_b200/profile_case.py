"""Run a fixed, small workload for profiling (e.g. under ncu):

    python -m dispatcher_b200.profile_case prefill --batch 1 --seq 1024 --iters 2
    python -m dispatcher_b200.profile_case decode --batch 1 --ctx 1024 --iters 4
    python -m dispatcher_b200.profile_case gate_bwd --batch 4 --seq 4096 --iters 2

Default 292M config, seeded random-init bf16 weights, uniform token ids."""

import argparse

import torch

from . import DispatcherConfig, DispatcherHybridForCausalLM, FusedGraphedHybridDecoder
from .engine import PrefillEngine


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["prefill", "decode", "gate_bwd"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--step-kernel", default="graph")
    a = ap.parse_args()
    cfg = DispatcherConfig()
    g = torch.Generator().manual_seed(0)
    if a.what == "gate_bwd":  # one tree layer's gate readout backward, all levels
        from . import ops
        b, T, gh, H, L = a.batch, a.seq, cfg.d_model, cfg.num_heads, cfg.levels
        n_lv = min(L, T.bit_length())
        A, B = ((torch.randn(b, T, gh, generator=g) * 0.5).bfloat16().cuda() for _ in range(2))
        W = [(torch.randn(L, H, gh, generator=g) * 0.05).bfloat16().cuda() for _ in range(3)]
        dP = [torch.randn(b, T, n_lv, H, generator=g).bfloat16().cuda() for _ in range(3)]
        for _ in range(a.iters):
            ops.gate_preacts_bwd(A, B, *W, *dP, n_lv)
        torch.cuda.synchronize()
        print("ok")
        return
    model = DispatcherHybridForCausalLM(cfg, seed=0).to("cuda", torch.bfloat16)
    if a.what == "prefill":
        ids = torch.randint(0, cfg.vocab_size, (a.batch, a.seq), generator=g).cuda()
        eng = PrefillEngine(model)
        for _ in range(a.iters):
            eng.forward(ids)
    else:
        ids = torch.randint(0, cfg.eot_token, (a.batch, a.ctx), generator=g).cuda()
        dec = FusedGraphedHybridDecoder(model, step_kernel=a.step_kernel)
        tok = dec.prefill(ids)[:, -1].argmax(-1)
        for _ in range(a.iters):
            tok = dec.step(tok).argmax(-1)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
