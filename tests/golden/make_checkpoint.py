"""Writes tests/golden/tiny_ckpt/: a tiny Dispatcher-Hybrid checkpoint saved by
the reference package itself (save_pretrained, safetensors, bf16 — the format
its scripts/convert_checkpoint.py produces), plus the reference's own fp32
logits on a fixed multi-document input.  Run in a container that has the
reference source tree:

    python tests/golden/make_checkpoint.py /path/to/reference
"""

import json
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tiny_ckpt")


def main(ref_root):
    sys.path.insert(0, ref_root)
    from dispatcher_hybrid import DispatcherConfig, DispatcherHybridForCausalLM
    cfg = DispatcherConfig(vocab_size=515, d_model=128, num_heads=2, dim_feedforward=384,
                           num_layers=2, max_len=256, attn_layers=(1,), attn_window=64,
                           eot_token=514)
    torch.manual_seed(7)
    model = DispatcherHybridForCausalLM(cfg)
    with torch.no_grad():   # non-degenerate source projection (zero-initialised otherwise)
        for blk in model.blocks:
            if hasattr(blk, "mixer"):
                blk.mixer.gate_hidden_src.weight.normal_(0.0, 0.05)
    model = model.to(torch.bfloat16).eval()
    os.makedirs(OUT, exist_ok=True)
    model.save_pretrained(OUT, safe_serialization=True)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 514, (2, 40), generator=g)
    ids[0, 12] = 514
    ids[1, 30] = 514
    with torch.no_grad():
        logits = model.float()(ids).logits
    np.savez_compressed(os.path.join(OUT, "reference_logits.npz"), ids=ids.numpy(),
                        logits=logits.numpy())
    print("wrote", OUT, sorted(os.listdir(OUT)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/nonexistent")
