"""Benchmark of the Dispatcher-Hybrid B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Primary line: parallel-forward prefill of the
default 292M model (random-init bf16 weights, seed 0) over 8 x 4096 synthetic
token ids per GPU (uniform over the vocabulary, EOT kept so the doc-reset
mask is live) -> logits.  N GPUs each prefill their own 8 sequences (weak
scaling; at N=8 this is the 64-sequence sharded prefill of configs[4]).
`value` is whole-job tok/s (max over ranks of the device time).  Decode
results at context 3900 (16 lockstep rows per GPU, and batch 1) are added
under "decode" in the same JSON line.

`--impl reference` times the reference algorithm on the host CPU (the
oracle: an eager restatement of the reference's own PyTorch code) on a
bounded sample of the same workload.
"""

import argparse
import json
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
PREFILL_B, PREFILL_T = 8, 4096
DECODE_CTX = 3900
METRIC = "prefill tok/s at T=4096 (8 x 4096 per GPU)"
GATE_UP_TRAFFIC = 2 * (65.9e6 + 57.9e6)   # DRAM bytes per gate/up GEMM launch at 8 x 4096


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            return json.load(f), "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


def prefill_flops_per_token(cfg):
    """Algorithmic FLOPs per prefill token: every dense projection (2 per
    MAC, tied lm_head included), the gate readouts of every level, and the
    window attention (average keys per query over T=4096 with window 1024)."""
    d, H, L, ff, V = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
    n_attn = len(cfg.attn_slots())
    n_tree = cfg.num_layers - n_attn
    dense = n_tree * (4 * d * d + 3 * ff * d) + n_attn * (4 * d * d + 3 * ff * d) + V * d
    gates = n_tree * L * 3 * H * d
    T, W = PREFILL_T, cfg.attn_window
    avg_keys = sum(min(t + 1, W) for t in range(T)) / T
    attn = n_attn * 4 * d * avg_keys
    return 2 * dense + 2 * gates + attn


def decode_bytes_per_step(cfg, batch, ctx):
    """Algorithmic HBM bytes of one decode step: every weight once (tied
    lm_head read in full, the embedding one row per token) plus the per-row
    state the step must read/write (ring slots and histories of every level,
    the attention window of K and V)."""
    d, H, L, ff, V = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
    n_attn = len(cfg.attn_slots())
    n_tree = cfg.num_layers - n_attn
    w_tree = (4 * d * d + 3 * L * H * d + 3 * ff * d) * 2 + 3 * L * H * 4
    w_attn = (4 * d * d + 3 * ff * d) * 2
    weights = n_tree * w_tree + n_attn * w_attn + V * d * 2 + (2 * cfg.num_layers + 1) * d * 2
    tree_row = (d * 2) * (1 + L) + (d * 2) * (2 * L) + L * H * 2 * 2
    win = min(ctx + 1, cfg.attn_window if cfg.attn_window > 0 else ctx + 1)
    attn_row = 2 * win * d * 2 + 2 * d * 2
    state = batch * (n_tree * tree_row + n_attn * attn_row + d * 2)
    return weights + state


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev, self.proc, self.lines = device_index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
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
            parts = [x.strip() for x in ln.split(",")]
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
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group(
            "nccl" if torch.cuda.is_available() else "gloo",
            timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    from dispatcher_b200 import sharding
    sharding.barrier(torch.cuda.current_device() if torch.cuda.is_available() else None)


def max_over_ranks(v, world):
    from dispatcher_b200 import sharding
    return sharding.max_over_ranks(v, "cuda" if torch.cuda.is_available() else None)


def prompt_ids(n_rows, T, seed, vocab=50257, eot=50256, keep_eot=False):
    """Uniform ids; unless keep_eot, EOT is re-drawn from [0, eot) so decode
    prompts stay a single document (the decoders reject separators)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (n_rows, T), generator=g)
    if not keep_eot:
        bad = ids == eot
        while bad.any():
            ids[bad] = torch.randint(0, eot, (int(bad.sum()),), generator=g)
            bad = ids == eot
    return ids


# ----------------------------------------------------------------- b200 arm
def run_prefill(engine, ids, steps, warmup, world, logits_buf):
    """Device-timed prefill steps (no instrumentation inside the timed
    region), then the same number of steps again with every launch bracketed
    by CUDA events on the engine's stream, for the per-op split and the
    roofline of the dominant kernel."""
    for _ in range(warmup):
        engine.forward(ids, logits_out=logits_buf)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        engine.forward(ids, logits_out=logits_buf)
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world) / steps
    engine.check_status(sync=True)   # a timed-out wait anywhere in the window raises here
    engine.record_events = []
    for _ in range(steps):
        engine.forward(ids, logits_out=logits_buf)
    torch.cuda.synchronize()
    events, engine.record_events = engine.record_events, None
    per_op = {}
    for name, flops, a, b in events:
        x = per_op.setdefault(name, [0, 0.0, 0.0])
        x[0] += 1
        x[1] += a.elapsed_time(b)
        x[2] += flops
    return ms, per_op


def run_prefill_e2e(model, ids_host, steps, warmup):
    """Public API (`model(input_ids).logits`) with host buffers: each step
    copies the ids up from pinned memory and reads the last-position logits
    (the next-token distribution of every row) back into pinned memory."""
    ids_pin = ids_host.pin_memory()
    out_pin = torch.empty(ids_host.shape[0], model.config.vocab_size, dtype=torch.bfloat16).pin_memory()
    for _ in range(warmup):
        lg = model(ids_pin.to("cuda", non_blocking=True)).logits
        out_pin.copy_(lg[:, -1])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        lg = model(ids_pin.to("cuda", non_blocking=True)).logits
        out_pin.copy_(lg[:, -1])
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / steps
    return ids_host.numel() / dt, ids_pin.numel() * 8, out_pin.numel() * 2


def run_decode(model, cfg, batch, ctx, steps, warmup, seed, world, select=None,
               gather_logits=False):
    """Device-timed lockstep decode after a `ctx`-token prefill.  Each step
    is one CUDA graph replay (FusedGraphedHybridDecoder.lockstep_loop): the
    step's kernels, the token choice on the device (greedy unless `select`
    is given) fed back as the next input, and with N > 1 the NCCL all-gather
    of every rank's tokens.  `steps` counts timed steps after `warmup`
    untimed ones (both within max_len); gather_logits adds one all-gather of
    the last step's logits of every rank after the timed steps, inside the
    timed region."""
    from dispatcher_b200 import FusedGraphedHybridDecoder
    from dispatcher_b200.generation import select_greedy
    torch.cuda.manual_seed(seed)
    ids = prompt_ids(1, ctx, seed, cfg.vocab_size, cfg.eot_token).expand(batch, ctx).contiguous().cuda()
    dec = FusedGraphedHybridDecoder(model)
    dec.prefill(ids)
    loop = dec.lockstep_loop(select or select_greedy)
    warmup = max(0, min(warmup, cfg.max_len - ctx - 1))
    steps = max(1, min(steps, cfg.max_len - ctx - warmup))
    for _ in range(warmup):
        loop.step()
    all_logits = (torch.empty(world * batch, cfg.vocab_size, device="cuda", dtype=torch.bfloat16)
                  if gather_logits and world > 1 else None)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        loop.step()
    if all_logits is not None:
        torch.distributed.all_gather_into_tensor(all_logits, dec.logits_out)
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world) / steps
    loop.finish()
    loop.release()
    return ms, steps, dec.persistent


def run_gate_backward(cfg, steps, warmup):
    """The gate readout's backward (dh_gate_preacts_bwd, the reference op
    gate_preacts_bwd) at one tree layer of the prefill workload: 8 x 4096
    positions, all levels, synthetic bf16 inputs resident in HBM, fp32
    gradient buffers allocated once (the kernel adds into them)."""
    import ctypes
    from dispatcher_b200 import ops
    from dispatcher_b200._lib import call
    b, T, gh, H, L = PREFILL_B, PREFILL_T, cfg.d_model, cfg.num_heads, cfg.levels
    n_lv = min(L, T.bit_length())
    g = torch.Generator(device="cuda").manual_seed(5)
    A = (torch.randn(b, T, gh, device="cuda", generator=g) * 0.5).bfloat16()
    B = (torch.randn(b, T, gh, device="cuda", generator=g) * 0.5).bfloat16()
    W = [(torch.randn(L, H, gh, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(3)]
    dP = [torch.randn(b, T, n_lv, H, device="cuda", generator=g).bfloat16() for _ in range(3)]
    wt = ops.pack_gate_weights_t(*W, n_lv)
    outs = [torch.zeros(b, T, gh, device="cuda") for _ in range(2)]
    outs += [torch.zeros(n_lv, H, gh, device="cuda") for _ in range(3)]
    outs += [torch.zeros(n_lv, H, device="cuda") for _ in range(3)]
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def launch():
        call("dh_gate_preacts_bwd", p(A), gh, p(B), gh, p(wt), None, n_lv, b, T, H, n_lv, gh,
             *(p(x) for x in dP), *(p(x) for x in outs), p(st), stream)

    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    if int(st.item()) != 0:
        raise RuntimeError("gate backward: bounded wait timed out")
    ms = e0.elapsed_time(e1) / steps
    flops = 4.0 * 3 * H * gh * n_lv * b * T   # dh = dP W and dW = dP^T h, 2 flop per MAC
    return ms, flops


def prefill_config(world):
    return {"workload": "configs[1]: parallel-forward prefill, 8 x 4096 tokens per GPU, "
                        "uniform ids (EOT kept, doc-reset mask live)",
            "model": "dispatcher-hybrid-292m random init (seed 0)",
            "global_batch": PREFILL_B * world, "seq_len": PREFILL_T,
            "parallelism": f"dp{world} (batch rows sharded)",
            "l2": "no flush: weights (584 MB) and per-step activations exceed L2 (126 MB)"}


# ----------------------------------------------------------------- CPU legs
def cpu_prefill_sample(cfg, T=1024, steps=1):
    """The reference algorithm (oracle restatement of the reference's eager
    parallel forward), fp32 on the host cores: one sequence of T tokens."""
    import oracle
    from dispatcher_b200 import make_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    sd = make_state_dict(cfg, seed=0)
    ids = prompt_ids(1, T, 0, cfg.vocab_size, cfg.eot_token, keep_eot=True)
    with torch.no_grad():
        oracle.forward(sd, cfg, ids[:, :64])
        t0 = time.perf_counter()
        for _ in range(steps):
            oracle.forward(sd, cfg, ids)
        dt = (time.perf_counter() - t0) / steps
    return {"value": T / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle (eager restatement of the reference forward), fp32, 1 x {T} tokens "
                      f"of the same synthetic distribution, {steps} timed pass(es)"}


def cpu_decode_sample(cfg, prompt=256, steps=8):
    """The reference's incremental decoder (oracle restatement of
    IncrementalDecoder), fp32 on the host cores: batch 1, greedy steps after a
    short prompt.  A step streams every weight once and reads a window of at
    most 1024 keys, so its cost barely depends on the context length."""
    import oracle
    from dispatcher_b200 import make_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    sd = make_state_dict(cfg, seed=0)
    ids = prompt_ids(1, prompt, 1, cfg.vocab_size, cfg.eot_token)
    dec = oracle.OracleDecoder(sd, cfg)
    with torch.no_grad():
        tok = dec.prefill(ids)[:, -1].argmax(-1)
        tok = dec.step(tok).argmax(-1)
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = dec.step(tok).argmax(-1)
        dt = (time.perf_counter() - t0) / steps
    return {"value": 1.0 / dt, "unit": "tok/s", "ms_per_step": dt * 1e3,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle IncrementalDecoder (eager restatement of the reference), fp32, "
                      f"batch 1, {steps} greedy steps after a {prompt}-token prompt"}


def reference_arm(args, world, rank, cfg):
    """The reference's own algorithm on the host cores (the oracle restates the
    reference's eager PyTorch forward op for op): each step is a bounded
    sample (one 1024-token sequence) of the prefill workload."""
    if rank == 0:
        steps = max(1, min(args.steps, 10))
        import oracle
        from dispatcher_b200 import make_state_dict
        torch.set_num_threads(os.cpu_count() or 1)
        sd = make_state_dict(cfg, seed=0)
        ids = prompt_ids(1, 1024, 0, cfg.vocab_size, cfg.eot_token, keep_eot=True)
        with torch.no_grad():
            for _ in range(max(1, min(args.warmup, 2))):
                oracle.forward(sd, cfg, ids[:, :256])
            t0 = time.perf_counter()
            for _ in range(steps):
                oracle.forward(sd, cfg, ids)
            dt = (time.perf_counter() - t0) / steps
        v = 1024 / dt
        sample = (f"oracle eager restatement of the reference forward, fp32, 1 x 1024 tokens per "
                  f"step, {steps} steps")
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": prefill_config(world),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def profile_case(a):
    """A fixed, small workload to run under a profiler (never a bench value):

        python bench.py --profile-case prefill --batch 4 --seq 4096 --iters 1
        python bench.py --profile-case decode --batch 1 --ctx 3900 --iters 3
        python bench.py --profile-case gate_bwd --batch 4 --seq 4096 --iters 2

    Default 292M config, seeded random-init bf16 weights, uniform token ids."""
    from dispatcher_b200 import (DispatcherConfig, DispatcherHybridForCausalLM,
                                 FusedGraphedHybridDecoder, ops)
    from dispatcher_b200.engine import PrefillEngine
    cfg = DispatcherConfig()
    g = torch.Generator().manual_seed(0)
    if a.profile_case == "gate_bwd":  # one tree layer's gate readout backward, all levels
        b, T, gh, H, L = a.batch, a.seq, cfg.d_model, cfg.num_heads, cfg.levels
        n_lv = min(L, T.bit_length())
        A, B = ((torch.randn(b, T, gh, generator=g) * 0.5).bfloat16().cuda() for _ in range(2))
        W = [(torch.randn(L, H, gh, generator=g) * 0.05).bfloat16().cuda() for _ in range(3)]
        dP = [torch.randn(b, T, n_lv, H, generator=g).bfloat16().cuda() for _ in range(3)]
        for _ in range(a.iters):
            ops.gate_preacts_bwd(A, B, *W, *dP, n_lv)
    else:
        model = DispatcherHybridForCausalLM(cfg, seed=0).to("cuda", torch.bfloat16)
        if a.profile_case == "prefill":
            ids = torch.randint(0, cfg.vocab_size, (a.batch, a.seq), generator=g).cuda()
            eng = PrefillEngine(model)
            for _ in range(a.iters):
                eng.forward(ids)
            eng.check_status(sync=True)
        else:
            ids = torch.randint(0, cfg.eot_token, (a.batch, a.ctx), generator=g).cuda()
            dec = FusedGraphedHybridDecoder(model, step_kernel=a.step_kernel)
            tok = dec.prefill(ids)[:, -1].argmax(-1)
            for _ in range(a.iters):
                tok = dec.step(tok).argmax(-1)
            dec.check_status(sync=True)
    torch.cuda.synchronize()
    print("ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", choices=["prefill", "decode", "gate_bwd"],
                    help="run a small fixed workload for a profiler and exit (no JSON line)")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--step-kernel", default="graph")
    args = ap.parse_args()
    if args.profile_case:
        return profile_case(args)
    args.warmup = max(3, args.warmup)

    world, rank, local = dist_setup()
    from dispatcher_b200 import DispatcherConfig, DispatcherHybridForCausalLM
    from dispatcher_b200.engine import PrefillEngine
    cfg = DispatcherConfig()
    if args.impl == "reference":
        return reference_arm(args, world, rank, cfg)

    pk, pk_kind = peaks()
    model = DispatcherHybridForCausalLM(cfg, seed=0).to("cuda", torch.bfloat16).eval()
    model.enable_fused_gates()
    ids_host = prompt_ids(PREFILL_B, PREFILL_T, 1000 * rank, cfg.vocab_size, cfg.eot_token,
                          keep_eot=True)
    ids = ids_host.cuda()
    engine = PrefillEngine(model)
    logits_buf = torch.empty(PREFILL_B * PREFILL_T, (cfg.vocab_size + 7) // 8 * 8, device="cuda",
                             dtype=torch.bfloat16)
    engine.calls = 0
    engine.forward(ids, logits_out=logits_buf)
    launches_per_step = engine.calls

    clocks = ClockSampler(local)
    clocks.start()
    ms, per_op = run_prefill(engine, ids, args.steps, args.warmup, world, logits_buf)
    clk = clocks.stop()
    tokens = PREFILL_B * PREFILL_T
    flop_tok = prefill_flops_per_token(cfg)
    g_n = sum(v[0] for k, v in per_op.items() if k in ("proj3", "qkv", "out", "gate_up", "down", "lm_head"))
    g_ms = sum(v[1] for k, v in per_op.items() if k in ("proj3", "qkv", "out", "gate_up", "down", "lm_head"))
    g_fl = sum(v[2] for k, v in per_op.items() if k in ("proj3", "qkv", "out", "gate_up", "down", "lm_head"))
    peak_t = pk["bf16_tflops_sustained"]
    gemm_tf = g_fl / (g_ms * 1e-3) / 1e12
    e2e_v, h2d, d2h = run_prefill_e2e(model, ids_host, args.steps, 2)
    e2e_v = -max_over_ranks(-e2e_v, world) * world

    # configs[2] (b1: greedy, 196 steps from a 3900 prefill), configs[3] (b16:
    # 16 rows of one 3900 prompt, top-k 50 / T 0.8 sampling, 196 steps) and
    # configs[4] (sharded: 16 rows per GPU, 128 greedy steps from a 3968
    # prefill, tokens gathered every step, logits of the last step gathered)
    from dispatcher_b200.generation import select_top_k
    dec_lines = {}
    legs = (("b16", 16, DECODE_CTX, 2, select_top_k(50, 0.8), False,
             "configs[3]: 16 lockstep rows of one 3900-token prompt, top-k 50 / T 0.8 sampling "
             "(Gumbel-max over the top-k, on the device), 196 steps (to the 4096 context)"),
            ("b1", 1, DECODE_CTX, 1, None, False,
             "configs[2]: batch 1, greedy, 196 steps from a 3900-token prompt"),
            ("sharded", 16, 3968, 3, None, True,
             "configs[4]: 16 rows per GPU, greedy, 128 steps from a 3968-token prompt, "
             "tokens all-gathered every step and the last step's logits all-gathered"))
    for name, batch, ctx, seed, sel, gath, what in legs:
        n_steps = cfg.max_len - ctx - args.warmup
        dms, dsteps, persistent = run_decode(model, cfg, batch, ctx, n_steps, args.warmup, seed,
                                             world, select=sel, gather_logits=gath)
        nbytes = decode_bytes_per_step(cfg, batch, ctx)
        dec_lines[name] = {
            "workload": what,
            "value": world * batch * 1000.0 / dms, "unit": "tok/s", "ms_per_step": dms,
            "steps": dsteps, "warmup": args.warmup, "batch_per_gpu": batch, "ctx": ctx,
            "kernel": "persistent step kernel" if persistent else "per-op kernels in a CUDA graph",
            "roofline": {"bound": "hbm", "achieved": nbytes / (dms * 1e-3) / 1e9,
                         "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": nbytes / (dms * 1e-3) / 1e9 / pk["hbm_gbs"],
                         "bytes_per_step": nbytes}}
    dec_lines["b1"]["vs_reference_a6000_fused_525"] = dec_lines["b1"]["value"] / world / 525.1
    # batch-1 decode cost across context lengths (flatness)
    flat = {}
    for ctx in (256, 1024, 2048):
        fms, _, _ = run_decode(model, cfg, 1, ctx, 64, args.warmup, 1, world)
        flat[str(ctx)] = round(fms, 4)
    flat[str(DECODE_CTX)] = round(dec_lines["b1"]["ms_per_step"], 4)
    dec_lines["b1_ms_per_step_by_ctx"] = flat

    gb_ms, gb_flops = run_gate_backward(cfg, 5, args.warmup)
    gb_tf = gb_flops / (gb_ms * 1e-3) / 1e12

    line = {
        "metric": METRIC, "value": world * tokens * 1000.0 / ms, "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": prefill_config(world),
        "roofline": {"bound": "tensor", "kernel": "gemm_kernel (tcgen05, all prefill projections)",
                     "achieved": gemm_tf, "peak": peak_t, "unit": "TFLOP/s",
                     "frac": gemm_tf / peak_t, "traffic": GATE_UP_TRAFFIC,
                     "traffic_note": "DRAM bytes read + written by one launch of the largest "
                                     "shape (FFN gate/up with the SwiGLU epilogue, M = 8 x 4096): "
                                     "an ncu capture at M = 4 x 4096 (65.9 MB read + 57.9 MB "
                                     "written) scaled by 2, the traffic growing with M; "
                                     "algorithmic bytes of that launch 263 MB (A 67 + W 11.5 + "
                                     "out 184.5); achieved averages all 73 GEMM launches of a step",
                     "peak_kind": f"{pk_kind} sustained",
                     "launches_timed": g_n,
                     "whole_step_tflops": flop_tok * tokens / (ms * 1e-3) / 1e12,
                     "whole_step_frac": flop_tok * tokens / (ms * 1e-3) / 1e12 / peak_t,
                     "algorithmic_flops_per_token": flop_tok},
        "per_op_ms_per_step": {k: round(v[1] / args.steps, 3) for k, v in per_op.items()},
        "decode": dec_lines,
        "gate_backward": {
            "what": "dh_gate_preacts_bwd, one tree layer of the prefill workload (8 x 4096, "
                    "12 levels): dA, dB, dW, db", "ms_per_call": gb_ms,
            "roofline": {"bound": "tensor", "achieved": gb_tf, "peak": peak_t, "unit": "TFLOP/s",
                         "frac": gb_tf / peak_t, "algorithmic_flops": gb_flops}},
        "clocks": clk,
        "e2e": {"value": e2e_v, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_prefill_sample(cfg)
        try:
            line["decode"]["b1"]["cpu_baseline"] = cpu_decode_sample(cfg)
        except Exception as exc:  # a reported baseline: never the reason a bench line is lost
            line["decode"]["b1"]["cpu_baseline"] = {"error": repr(exc)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
