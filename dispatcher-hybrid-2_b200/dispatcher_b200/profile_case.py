"""Run a fixed, small workload for profiling (e.g. under ncu):

    python -m dispatcher_b200.profile_case prefill --batch 1 --seq 1024 --iters 2
    python -m dispatcher_b200.profile_case decode --batch 1 --ctx 1024 --iters 4

Default 292M config, seeded random-init bf16 weights, uniform token ids."""

import argparse

import torch

from . import DispatcherConfig, DispatcherHybridForCausalLM, FusedGraphedHybridDecoder
from .engine import PrefillEngine


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["prefill", "decode"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--step-kernel", default="graph")
    a = ap.parse_args()
    cfg = DispatcherConfig()
    model = DispatcherHybridForCausalLM(cfg, seed=0).to("cuda", torch.bfloat16)
    g = torch.Generator().manual_seed(0)
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
