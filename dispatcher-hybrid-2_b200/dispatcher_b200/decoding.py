"""B200 incremental decoder: the drop-in for the reference's
`FusedGraphedHybridDecoder` (dispatcher_hybrid/decoding.py:446-488).

Same public surface as the reference decoders (decoding.py:101-338):

    dec = FusedGraphedHybridDecoder(model)      # model in bfloat16 on CUDA
    logits = dec.prefill(ids)                   # ids (T,) or (B, T)
    logits = dec.step(tokens)                   # scalar / (1,) / (B,)
    dec.t, dec.max_len, dec.batch, dec.caches

and the same cache layouts (B_hist, rg_hist, V_ring with ring offsets and
masks; k/v with RoPE'd keys), so cache contents and slot positions compare
element for element with the reference's eager decoder.

One step is the sequence of C-ABI calls recorded by `_record_step` and
captured once into a CUDA graph; the position lives on the device in
`t_buf` and is advanced inside the graph.  Every kernel of the step is a
hand-written sm_100a kernel of `libdispatcher_b200.so`; there is no other
compute path (construction fails without CUDA or the library).
"""

import math

import torch

from . import _lib
from .packing import PackedModel, config_of
from .status import StatusWord


def _ptr(t):
    return ctypes_void(t.data_ptr()) if t is not None else None


def ctypes_void(p):
    import ctypes
    return ctypes.c_void_p(p)


class TreeLayerCache:
    """Reference `_TreeLayerCache` layout (decoding.py:50-76)."""

    def __init__(self, batch, max_len, gh, L, H, hd, device, dtype):
        self.L, self.H, self.hd = L, H, hd
        d = H * hd
        self.B_hist = torch.zeros(batch, max_len, gh, device=device, dtype=dtype)
        self.rg_hist = torch.zeros(batch, max_len, L, H, device=device, dtype=dtype)
        self.S = 2 ** (L + 1) - 2
        self.V_ring = torch.zeros(batch, self.S, d, device=device, dtype=dtype)
        self.offsets = torch.tensor([2 ** (j + 1) - 2 for j in range(L)], device=device)
        self.masks = torch.tensor([2 ** (j + 1) - 1 for j in range(L)], device=device)


class AttnCache:
    """Reference `_AttnCache` layout (decoding.py:79-86); RoPE tables in fp32."""

    def __init__(self, batch, max_len, H, hd, device, dtype):
        self.k = torch.zeros(batch, max_len, H, hd, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        theta = 10000.0 ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)
        ang = torch.arange(max_len, dtype=torch.float32)[:, None] * theta[None, :]
        self.rope_cos = ang.cos().to(device).contiguous()
        self.rope_sin = ang.sin().to(device).contiguous()


def check_single_document(cfg, ids):
    """decoding.py:89-98: the decoders implement the wrap mask only."""
    if getattr(cfg, "doc_reset", False) and bool((ids == cfg.eot_token).any()):
        raise ValueError(
            f"prompt contains the document separator (token {cfg.eot_token}) and this "
            f"model was trained with doc_reset=True; the incremental decoders assume a "
            f"single document. Remove the separator, or use model.generate().")


class _DirectStep:
    """Stand-in for a captured graph: re-issues the (single-launch) step."""

    def __init__(self, dec):
        self.dec = dec

    def replay(self):
        self.dec._record_step(torch.cuda.current_stream().cuda_stream)


class FusedGraphedHybridDecoder:
    """Exact per-token decoder on B200 kernels, one CUDA-graph replay per token."""

    def __init__(self, model, max_len=None, dtype=None, step_kernel="graph",
                 multi_document=False):
        """step_kernel: "graph" (per-op kernels captured in one CUDA graph) or
        "persistent" (one cooperative kernel per step, batch <= 2).

        multi_document: accept prompts (and generated tokens) that contain the
        document separator of a doc_reset model.  The decoder then keeps each
        row's document id per position and masks every tree level across a
        separator, as the parallel forward does; by default it refuses such
        prompts like the reference's decoders (decoding.py:89-98)."""
        if step_kernel not in ("graph", "persistent"):
            raise ValueError(f"step_kernel must be 'graph' or 'persistent', got {step_kernel!r}")
        if multi_document and step_kernel != "graph":
            raise ValueError("multi_document decoding runs on step_kernel='graph'")
        self.step_kernel = step_kernel
        self.multi_document = bool(multi_document)
        if not torch.cuda.is_available():
            raise RuntimeError("FusedGraphedHybridDecoder requires CUDA")
        param_dtype = next(model.parameters()).dtype
        if dtype is not None and dtype != param_dtype:            # decoding.py:119-122
            raise ValueError(
                f"decoder dtype {dtype} != model dtype {param_dtype}; cast the "
                f"model first, e.g. model.to(torch.bfloat16)")
        _lib.load()                                               # fail now, not mid-step
        self.m = model
        self.cfg = config_of(model)
        self.max_len = max_len or self.cfg.max_len
        if self.max_len > self.cfg.max_len or self.max_len & (self.max_len - 1):
            raise ValueError(f"max_len {self.max_len} must be a power of two <= "
                             f"{self.cfg.max_len}")
        self.dtype = param_dtype
        self.w = PackedModel(model)
        self.device = self.w.device
        self.caches = None
        self.batch = None
        self.graph = None
        self._engine = None
        self.t = 0
        self._squeeze = False

    # ------------------------------------------------------------ buffers
    def _alloc(self, batch):
        if self.caches is not None and self.batch == batch:
            for c in self.caches:          # a new prompt starts from empty caches
                for name in ("B_hist", "rg_hist", "V_ring", "k", "v"):
                    if hasattr(c, name):
                        getattr(c, name).zero_()
            return
        cfg, dev, dt = self.cfg, self.device, self.dtype
        H, d = cfg.num_heads, cfg.d_model
        hd, L = d // H, cfg.levels
        self.batch = batch
        slots = cfg.attn_slots()
        self.caches = [AttnCache(batch, self.max_len, H, hd, dev, dt) if i in slots else
                       TreeLayerCache(batch, self.max_len, d, L, H, hd, dev, dt)
                       for i in range(cfg.num_layers)]
        f32, bf = torch.float32, torch.bfloat16
        self.token_buf = torch.zeros(batch, dtype=torch.long, device=dev)
        # document ids per (row, position) and each row's last token, used
        # only when the decoder tracks documents
        self.doc_hist = (torch.zeros(batch, self.max_len, dtype=torch.int32, device=dev)
                         if self.multi_document else None)
        self.last_tok = torch.zeros(batch, dtype=torch.long, device=dev)
        self.t_buf = torch.zeros(1, dtype=torch.long, device=dev)
        self.logits_out = torch.zeros(batch, cfg.vocab_size, device=dev, dtype=bf)
        self.x = torch.zeros(batch, d, device=dev, dtype=f32)
        self.x_copy = torch.zeros(batch, d, device=dev, dtype=f32)   # input of the fused FFN
        self.v0 = torch.zeros(batch, d, device=dev, dtype=bf)
        self.a = torch.zeros(batch, d, device=dev, dtype=bf)
        self.y = torch.zeros(batch, d, device=dev, dtype=bf)
        self.q = torch.zeros(batch, d, device=dev, dtype=bf)
        self.ig = torch.zeros(batch, L, H, device=dev, dtype=f32)
        self.fg = torch.zeros(batch, L, H, device=dev, dtype=f32)
        sm = torch.cuda.get_device_properties(dev).multi_processor_count
        self.nsplit = max(1, min(16, math.ceil(2 * sm / max(1, min(batch, 16) * H))))
        self.part = torch.zeros(batch, H, self.nsplit, hd + 2, device=dev, dtype=f32)
        self.counters = torch.zeros(H + batch * H, device=dev, dtype=torch.int32)
        # bounded waits and bad token ids report here; read back without a
        # host sync after each call and raised at the next (check_status)
        self.status_word = StatusWord(dev)
        self.status = self.status_word.tensor
        from .step_params import SYNC_WORDS
        self.barrier = torch.zeros(SYNC_WORDS, device=dev, dtype=torch.int64)
        self.graph = None
        # one persistent kernel per step for lockstep batches of up to 2 rows
        # (dh_decode_step); larger batches run the per-op kernels in 16-row chunks
        self.persistent = (self.step_kernel == "persistent" and batch <= 2 and d <= 1024
                           and d % 128 == 0 and hd == 64
                           and cfg.levels * (2 * d + 16) <= 32768)
        # the FFN is one launch per layer, which reads the down projection by
        # rows of its transpose
        if not self.persistent:
            for lay in self.w.layers:
                if "w_downT" not in lay:
                    lay["w_downT"] = lay["w_down"].t().contiguous()
        # tree blocks of 3..16 rows: tensor-core gate readouts over the packed
        # gate rows (all heads of a level at once), pre-activations in fp32
        np_ = ((3 * H + 15) // 16) * 16
        # up to 8 rows: the gate readouts are folded into the W3 GEMV (each
        # tile of A adds its columns' share), then a recurrence kernel; 9-16
        # rows (or more than 16 levels, d above 1024, from 3 rows): the
        # readouts of all heads per level as their own tensor-core launch
        self.gates_fused = (not self.persistent and batch <= 8 and d % 32 == 0 and d <= 1024
                            and hd <= 64 and L <= 16 and 16 * L * np_ * 2 <= 33792)
        self.tree_tc = (not self.persistent and not self.gates_fused and batch > 2
                        and 3 * H <= 48 and d % 32 == 0 and hd <= 64)
        self.pre = None
        if self.tree_tc or self.gates_fused:
            from .ops import pack_gate_weights
            self.pre = torch.zeros(batch, L, np_, device=dev, dtype=f32)
            for lay in self.w.layers:
                if lay["kind"] == "tree" and "w_gates_np" not in lay:
                    lay["w_gates_np"], _, lay["gates_np"] = pack_gate_weights(
                        lay["wi"], lay["wf"], lay["wr"], lay["bi"], lay["bf"], lay["br"])
                if self.gates_fused and lay["kind"] == "tree" and "w_gates_t" not in lay:
                    lay["w_gates_t"] = lay["w_gates_np"].t().contiguous()   # (gh, L * np)
        self._step_params = None
        if self.persistent:
            from .step_params import build_step_params
            self._step_params = build_step_params(self)

    # ------------------------------------------------------------ one step
    def _record_step(self, stream):
        """Issue every kernel of one decode step on `stream` (captured once)."""
        if self.persistent:
            import ctypes
            _lib.call("dh_decode_step", ctypes.byref(self._step_params), ctypes_void(stream))
            return
        cfg, W, B = self.cfg, self.w, self.batch
        d, H, L, ff = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward
        hd = d // H
        V = cfg.vocab_size
        s = ctypes_void(stream)
        P = _ptr
        call = _lib.call
        if self.doc_hist is not None:
            call("dh_decode_doc_step", P(self.token_buf), P(self.t_buf), P(self.doc_hist),
                 P(self.last_tok), cfg.eot_token, B, self.max_len, s)
        call("dh_decode_embed", P(self.token_buf), P(W.emb), P(self.x), B, d, V,
             P(self.status), s)
        tree_ctr = self.counters[:H]
        attn_ctr = self.counters[H:]
        for lay, cache in zip(W.layers, self.caches):
            if lay["kind"] == "tree" and self.gates_fused:
                call("dh_decode_mixer_in_gates", P(self.x), P(lay["norm1"]), P(lay["w3"]),
                     P(self.v0), P(self.a), P(cache.B_hist), P(self.t_buf), self.max_len, B, d,
                     P(lay["w_gates_t"]), lay["gates_np"], L, H, P(self.pre), P(self.doc_hist),
                     P(self.status), s)
                call("dh_decode_tree_recur", P(lay["bi"]), P(lay["bf"]), P(lay["br"]),
                     P(self.t_buf), P(self.pre), lay["gates_np"], P(cache.rg_hist), P(self.v0),
                     P(cache.V_ring), P(self.y), P(self.doc_hist), B, self.max_len, L, H, hd, s)
            elif lay["kind"] == "tree":
                call("dh_decode_mixer_in", P(self.x), P(lay["norm1"]), P(lay["w3"]), P(self.v0),
                     P(self.a), P(cache.B_hist), P(self.t_buf), self.max_len, B, d,
                     P(self.status), s)
                if self.tree_tc:
                    call("dh_decode_tree_step_tc", P(self.a), P(cache.B_hist),
                         P(lay["w_gates_np"]), lay["gates_np"], P(lay["bi"]), P(lay["bf"]),
                         P(lay["br"]), P(self.t_buf), P(self.pre), P(cache.rg_hist),
                         P(self.v0), P(cache.V_ring), P(self.y), P(self.doc_hist), B,
                         self.max_len, L, H, hd, d, s)
                else:
                    call("dh_decode_tree_step", P(self.a), P(cache.B_hist), P(lay["wi"]),
                         P(lay["wf"]), P(lay["wr"]), P(lay["bi"]), P(lay["bf"]), P(lay["br"]),
                         P(self.t_buf), P(self.ig), P(self.fg), P(cache.rg_hist), P(self.v0),
                         P(cache.V_ring), P(self.y), P(tree_ctr), P(self.doc_hist), B,
                         self.max_len, L, H, hd, d, s)
            else:
                call("dh_decode_attn_in", P(self.x), P(lay["norm1"]), P(lay["wqkv"]),
                     P(cache.rope_cos), P(cache.rope_sin), P(self.q), P(cache.k), P(cache.v),
                     P(self.t_buf), self.max_len, B, d, H, P(self.status), s)
                call("dh_decode_attn", P(self.q), P(cache.k), P(cache.v), P(self.y),
                     P(self.t_buf), P(self.part), P(attn_ctr), self.nsplit, B, self.max_len,
                     H, hd, cfg.attn_window, s)
            # output projection + residual (for the fused FFN it also leaves a
            # copy of x, which that kernel reads while it adds into x), then the FFN
            call("dh_decode_linear_residual", P(self.y), P(lay["w_out"]), P(self.x),
                 P(self.x_copy), B, d, d, P(self.status), s)
            call("dh_decode_ffn", P(self.x_copy), P(lay["norm2"]), P(lay["w_gate"]),
                 P(lay["w_up"]), P(lay["w_downT"]), P(self.x), B, d, ff, P(self.status), s)
        call("dh_decode_logits", P(self.x), P(W.norm_out), P(W.lm_head), P(self.logits_out),
             B, d, V, P(self.status), s)
        call("dh_decode_advance", P(self.t_buf), s)

    def _capture(self):
        """decoding.py:317-328: warm up on a side stream, then capture one step."""
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        saved_t = int(self.t)
        with torch.cuda.stream(side):
            self._record_step(side.cuda_stream)   # warm-up: binds lazy attributes
        torch.cuda.current_stream().wait_stream(side)
        try:
            with torch.cuda.graph(g):
                self._record_step(torch.cuda.current_stream().cuda_stream)
        except Exception:
            if not self.persistent:
                raise
            # a single cooperative launch per step: replay it directly when the
            # driver refuses to capture it
            torch.cuda.synchronize()
            g = _DirectStep(self)
        self.t_buf.fill_(saved_t)
        self.graph = g

    # ------------------------------------------------------------ public
    def check_status(self, sync=False):
        """Raise DispatcherB200Error if a kernel of an earlier step or prefill
        reported a failed bounded wait or an out-of-range token; sync=True
        waits for the last call's report."""
        if self.caches is not None:
            self.status_word.check("FusedGraphedHybridDecoder", sync=sync)

    def _prepare_prompt(self, idx):
        self._squeeze = idx.dim() == 1
        ids = idx.view(1, -1) if self._squeeze else idx
        if not self.multi_document:
            check_single_document(self.cfg, ids)
        T = ids.shape[1]
        if T > self.max_len:
            raise ValueError(f"prompt of {T} exceeds max_len {self.max_len}")
        if T < 1:
            raise ValueError("empty prompt")
        ids = ids.to(self.device)
        self.check_status()
        self._alloc(ids.shape[0])
        return ids, T

    @torch.no_grad()
    def prefill(self, idx):
        """idx: (T,) or (B, T) token ids -> (T, vocab) / (B, T, vocab) logits.

        Runs the parallel forward on the B200 prefill engine, which also fills
        B_hist, rg_hist (all levels), every level's ring slab and the
        attention caches (decoding.py:143-185, 225-245), then captures the
        step graph at position T."""
        ids, T = self._prepare_prompt(idx)
        if self.graph is None:
            # the capture's warm-up step writes position 0, which the
            # prefill below overwrites; no cache slot keeps a stray value
            self.t = 0
            self.t_buf.zero_()
            self._capture()
        if self._engine is None:
            from .engine import PrefillEngine
            self._engine = PrefillEngine(self.m, packed=self.w)
        out = self._engine.forward(ids, caches=self.caches)
        if self.doc_hist is not None:
            # exclusive count of separators before each position (the
            # forward's doc_id); later positions come from the step kernels
            sep = (ids == self.cfg.eot_token).to(torch.int32)
            self.doc_hist[:, :T] = torch.cumsum(sep, 1, dtype=torch.int32) - sep
            self.last_tok.copy_(ids[:, T - 1])
        self.t = T
        self.t_buf.fill_(T)
        self.logits_out.copy_(out[:, -1])   # the latest logits, as after a step
        self.status_word.arm()
        return out[0] if self._squeeze else out

    @torch.no_grad()
    def prefill_stepwise(self, idx):
        """Same contract as prefill(), but the prompt runs through the captured
        step one position at a time (an independent route to the same caches)."""
        ids, T = self._prepare_prompt(idx)
        self.t = 0
        self.t_buf.zero_()
        if self.graph is None:
            self._capture()
        out = torch.empty(self.batch, T, self.cfg.vocab_size, device=self.device,
                          dtype=self.logits_out.dtype)
        for p in range(T):
            self.token_buf.copy_(ids[:, p])
            self.graph.replay()
            out[:, p].copy_(self.logits_out)
        self.t = T
        self.status_word.arm()
        return out[0] if self._squeeze else out

    @torch.no_grad()
    def step(self, tokens):
        """tokens: scalar / (1,) / (B,) -> (vocab,) or (B, vocab)."""
        if self.graph is None:
            raise RuntimeError("call prefill() before step()")
        if self.t >= self.max_len:                                 # decoding.py:289-290
            raise ValueError(f"context exhausted at max_len {self.max_len}")
        toks = tokens.view(-1)
        if toks.shape[0] != self.batch:
            raise ValueError(f"got {toks.shape[0]} tokens for batch {self.batch}")
        self.check_status()
        self.token_buf.copy_(toks)
        self.graph.replay()
        self.t += 1
        out = self.logits_out.clone()
        self.status_word.arm()
        return out[0] if self._squeeze else out

    def lockstep_loop(self, select, group=None):
        """A CUDA graph of one whole lockstep step, token choice included:
        the step's kernels, then `select(logits) -> (B,) int64` (device ops
        only: argmax, top-k with Gumbel noise, ...), whose tokens become the
        next step's input on the device, then (with a process group of more
        than one rank) an NCCL all-gather of every rank's tokens, all in the
        same graph.  Call after prefill(); run steps with .step().  The
        reference's loop (modeling_dispatcher.py:421-442) takes the same
        decisions on the host between graph replays."""
        return _LockstepLoop(self, select, group)


def select_greedy(logits):
    """Token choice for lockstep_loop: argmax per row (the loop runs it as
    one device kernel, dh_decode_argmax, that also feeds the next step)."""
    return logits.argmax(-1)


class _LockstepLoop:
    ARM_EVERY = 16   # steps between read-backs of the (sticky) status word

    def __init__(self, dec, select, group):
        import torch.distributed as dist
        if dec.graph is None:
            raise RuntimeError("call prefill() before lockstep_loop()")
        self.dec, self.select, self.group = dec, select, group
        world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.world = world
        B = dec.batch
        self.tokens = torch.zeros(world * B, dtype=torch.long, device=dec.device)
        self.local = torch.zeros(B, dtype=torch.long, device=dec.device)
        self._n = 0
        # first token from the latest logits (the prefill's last position, or
        # the last step's), outside the graph
        dec.token_buf.copy_(select(dec.logits_out))
        # warm the selection and the collective up outside the capture
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            select(dec.logits_out.clone())
            if world > 1:
                dist.all_gather_into_tensor(self.tokens, dec.token_buf.clone(), group=group)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = None
        if isinstance(dec.graph, _DirectStep):
            # a cooperative step the driver would not capture: issue it
            # directly, selection and collective after it
            return
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            dec._record_step(torch.cuda.current_stream().cuda_stream)
            self._choose()
        self.graph = g

    def _choose(self):
        """Token choice, feed-back and gather, on the current stream."""
        import torch.distributed as dist
        dec = self.dec
        stream = ctypes_void(torch.cuda.current_stream().cuda_stream)
        out = self.tokens if self.world == 1 else self.local
        if self.select is select_greedy:
            _lib.call("dh_decode_argmax", _ptr(dec.logits_out), _ptr(dec.token_buf), _ptr(out),
                      dec.batch, dec.cfg.vocab_size, stream)
            tok = out
        elif getattr(self.select, "top_k", None) is not None:   # generation.select_top_k
            sel = self.select
            _lib.call("dh_decode_sample_top_k", _ptr(dec.logits_out), _ptr(dec.token_buf),
                      _ptr(out), dec.batch, dec.cfg.vocab_size, sel.top_k, sel.temperature,
                      sel.seed, _ptr(dec.t_buf), stream)
            tok = out
        else:
            tok = self.select(dec.logits_out)
            dec.token_buf.copy_(tok)
            if self.world == 1:
                self.tokens.copy_(tok)
        if self.world > 1:
            dist.all_gather_into_tensor(self.tokens, tok, group=self.group)

    def step(self):
        """One step: feeds the tokens chosen last (the prefill's for the
        first call); afterwards .tokens holds this step's tokens of every
        rank (rank-major) and the decoder's logits buffer this step's logits."""
        dec = self.dec
        if dec.t >= dec.max_len:
            raise ValueError(f"context exhausted at max_len {dec.max_len}")
        dec.check_status()
        if self.graph is None:
            dec._record_step(torch.cuda.current_stream().cuda_stream)
            self._choose()
        else:
            self.graph.replay()
        dec.t += 1
        self._n += 1
        if self._n % self.ARM_EVERY == 0:
            dec.status_word.arm()
        return self.tokens

    def finish(self):
        """Wait for the steps issued so far and raise if any kernel of them
        reported a failure (the status word is sticky)."""
        self.dec.status_word.arm()
        self.dec.check_status(sync=True)

    def release(self):
        """Drop the graph (before destroying a process group it holds)."""
        self.graph = None


# the reference's name for the graphed decoder without fused kernels maps to
# the same implementation: on B200 every decoder runs the fused step
GraphedHybridDecoder = FusedGraphedHybridDecoder
