"""Benchmark of the Dispatcher-Hybrid B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload prefill|decode]

Workloads (default 292M config, random-init bf16 weights from seed 0,
synthetic uniform token ids):
  prefill  parallel forward of 8 x 4096 tokens per GPU -> logits (configs[1];
           8 rows per GPU, so N=8 is the 64-sequence sharded prefill)
  decode   16 lockstep rows per GPU at context 3900 (one shared prompt, seed
           2), greedy; plus a batch-1 decode line at context 3900 reported in
           the same JSON under "decode_b1"

One JSON line on rank 0.  `value` is the whole-job aggregate tok/s (max of
per-rank device times); `e2e` is the same metric through the public API with
host buffers; `roofline` covers the dominant kernel; `cpu_baseline` is the
reference algorithm (the CPU oracle, a restatement of the reference's eager
path) timed on this host's cores on a bounded sample.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "dispatcher-hybrid-2_b200"))

import torch  # noqa: E402

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- dist
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.distributed.init_process_group(
            "nccl" if torch.cuda.is_available() else "gloo",
            timeout=datetime.timedelta(seconds=300))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------- data
def prompt_ids(n_rows, T, seed, vocab=50257, eot=50256, share=False):
    """Uniform ids; EOT re-drawn from [0, eot) so decode prompts stay one document."""
    g = torch.Generator().manual_seed(seed)
    rows = 1 if share else n_rows
    ids = torch.randint(0, vocab, (rows, T), generator=g)
    bad = ids == eot
    while bad.any():
        ids[bad] = torch.randint(0, eot, (int(bad.sum()),), generator=g)
        bad = ids == eot
    return ids.expand(n_rows, T).contiguous() if share else ids


def decode_bytes_per_step(cfg, batch, ctx):
    """Algorithmic HBM bytes of one decode step: every weight once (tied
    lm_head read in full, embedding one row per token) + per-row state."""
    d, H, L, ff, V = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
    n_attn = len(cfg.attn_slots())
    n_tree = cfg.num_layers - n_attn
    w_tree = (4 * d * d + 3 * L * H * d + 3 * ff * d) * 2 + 3 * L * H * 4
    w_attn = (4 * d * d + 3 * ff * d) * 2
    weights = n_tree * w_tree + n_attn * w_attn + V * d * 2 + (2 * cfg.num_layers + 1) * d * 2
    # per row: tree: B_hist write + 12 reads, ring 12 reads + 12 writes, rg r/w
    tree_row = (d * 2) * (1 + L) + (d * 2) * (2 * L) + L * H * 2 * 2
    win = min(ctx + 1, cfg.attn_window if cfg.attn_window > 0 else ctx + 1)
    attn_row = 2 * win * d * 2 + 2 * d * 2
    state = batch * (n_tree * tree_row + n_attn * attn_row + d * 2)
    return weights + state, weights, state


# ----------------------------------------------------------------- b200 arm
def run_decode(model, cfg, batch, ctx, steps, warmup, seed, world):
    from dispatcher_b200 import FusedGraphedHybridDecoder
    ids = prompt_ids(batch, ctx, seed, cfg.vocab_size, cfg.eot_token, share=True).cuda()
    dec = FusedGraphedHybridDecoder(model)
    logits = dec.prefill(ids)[:, -1]
    nxt = logits.argmax(-1)
    steps = min(steps, cfg.max_len - ctx - warmup)
    for _ in range(warmup):
        nxt = dec.step(nxt).argmax(-1)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        nxt = dec.step(nxt).argmax(-1)
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world)
    return ms / steps, steps, dec


def run_decode_e2e(model, cfg, batch, ctx, steps, seed):
    """Public-API decode with host buffers: per step the host token ids go up
    from pinned memory and the chosen tokens come back."""
    from dispatcher_b200 import FusedGraphedHybridDecoder
    ids = prompt_ids(batch, ctx, seed, cfg.vocab_size, cfg.eot_token, share=True)
    dec = FusedGraphedHybridDecoder(model)
    logits = dec.prefill(ids.cuda())[:, -1]
    host_tok = logits.argmax(-1).cpu().pin_memory()
    steps = min(steps, cfg.max_len - ctx)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        dev_tok = host_tok.to("cuda", non_blocking=True)
        nxt = dec.step(dev_tok).argmax(-1)
        host_tok.copy_(nxt, non_blocking=False)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return batch * steps / dt, host_tok.numel() * 8, host_tok.numel() * 8


def cpu_decode_baseline(cfg, ctx=3900, steps=3):
    """Reference algorithm (oracle restatement of IncrementalDecoder) on the
    host cores, fp32, batch 1: prefill `ctx` tokens untimed, time `steps`."""
    import oracle
    from dispatcher_b200 import make_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    sd = make_state_dict(cfg, seed=0)
    dec = oracle.OracleDecoder(sd, cfg)
    ids = prompt_ids(1, ctx, 1, cfg.vocab_size, cfg.eot_token)
    dec.prefill(ids)
    tok = torch.tensor([11])
    dec.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        dec.step(tok)
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tok/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"oracle IncrementalDecoder restatement, fp32, batch 1, ctx {ctx}, "
                      f"{steps} steps after 1 warm step"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world, rank, local = dist_setup()
    from dispatcher_b200 import DispatcherConfig, DispatcherHybridForCausalLM
    cfg = DispatcherConfig()

    if args.impl == "reference":
        if rank == 0:
            base = cpu_decode_baseline(cfg, steps=max(2, min(args.steps, 5)))
            print(json.dumps({
                "impl": "reference", "metric": "decode tok/s (batch 16 lockstep, ctx 3900)",
                "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "weak", "dtype": "f32", "data": "synthetic",
                "config": {"workload": "decode, batch 1 sample of the 16-row lockstep config"},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tok/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    pk, pk_kind = peaks()
    model = DispatcherHybridForCausalLM(cfg, seed=0).to("cuda", torch.bfloat16).eval()
    clocks = ClockSampler(local)
    B, ctx = 16, 3900
    clocks.start()
    ms16, k16, _ = run_decode(model, cfg, B, ctx, args.steps, args.warmup, seed=2, world=world)
    ms1, k1, _ = run_decode(model, cfg, 1, ctx, args.steps, args.warmup, seed=1, world=world)
    clk = clocks.stop()
    e2e_v, hb, db = run_decode_e2e(model, cfg, B, ctx, min(args.steps, 50), seed=2)
    e2e_v = max_over_ranks(-e2e_v, world) * -1.0  # slowest rank
    tot16, _, _ = decode_bytes_per_step(cfg, B, ctx)
    tot1, _, _ = decode_bytes_per_step(cfg, 1, ctx)
    hbm = pk["hbm_gbs"]
    line = {
        "metric": "decode tok/s (batch 16 lockstep, ctx 3900)",
        "value": world * B * 1000.0 / ms16, "unit": "tok/s", "n_gpus": world,
        "steps": k16, "warmup": args.warmup, "ms_per_step": ms16, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "decode: 16 lockstep rows/GPU, shared 3900-token prompt "
                               "(seed 2), greedy", "model": "dispatcher-hybrid-292m random init",
                   "global_batch": B * world, "seq_len": ctx, "parallelism": f"dp{world}",
                   "l2": "no flush: weights (584 MB) exceed L2 (126 MB)"},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (CUDA graph)",
                     "achieved": tot16 / (ms16 * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": tot16 / (ms16 * 1e-3) / 1e9 / hbm, "traffic": None,
                     "peak_kind": pk_kind},
        "decode_b1": {"value": world * 1000.0 / ms1, "unit": "tok/s", "ms_per_step": ms1,
                      "steps": k1, "roofline_frac": tot1 / (ms1 * 1e-3) / 1e9 / hbm,
                      "vs_a6000_fused_525": world * 1000.0 / ms1 / 525.1},
        "clocks": clk,
        "e2e": {"value": e2e_v * world, "unit": "tok/s", "h2d_bytes_per_step": hb,
                "d2h_bytes_per_step": db},
        "gpu_launches": None,
    }
    n_kernels = 1 + 5 * cfg.num_layers + 2
    line["gpu_launches"] = n_kernels * k16
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_baseline(cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
