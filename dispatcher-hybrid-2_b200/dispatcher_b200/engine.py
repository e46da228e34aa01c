"""Parallel-forward (prefill) engine on the B200 kernels.

`PrefillEngine(model).forward(ids)` computes the logits of
`DispatcherHybridForCausalLM.forward` (modeling_dispatcher.py:325-351) with
every op on this package's sm_100a kernels:

    embedding gather -> per block: RMSNorm -> fused projection GEMM
      tree block:  [V0|A|B] = h W3^T; gates (tcgen05, hidden built in smem);
                   level sweep; x += V W_out^T (GEMM with residual epilogue)
      attn block:  [q|k|v] = h Wqkv^T; RoPE; window attention;
                   x += Y W_out^T
      FFN:         RMSNorm -> GEMM with SwiGLU epilogue -> GEMM + residual
    -> RMSNorm -> logits GEMM (tied embedding)

With `caches=` (a decoder's cache list) it also fills the decoder state
exactly as the reference's eager prefill does (decoding.py:143-185,
225-245): B_hist, rg_hist for all levels, every level's ring slab, and the
RoPE'd keys / raw values of the attention layers.
"""

import ctypes
import math

import torch

from . import _lib
from .ops import interleave_swiglu
from .packing import PackedModel, config_of
from .status import StatusWord


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def n_levels(L, T):
    """modeling_dispatcher.py:76 (and decoding.py:152)."""
    return min(L, int(math.log2(T)) + 1) if T > 1 else 1


class PrefillEngine:
    def __init__(self, model, packed=None):
        _lib.load()
        self.model = model
        self.cfg = cfg = config_of(model)
        self.w = packed if packed is not None else PackedModel(model)
        self.device = self.w.device
        d, H, L = cfg.d_model, cfg.num_heads, cfg.levels
        self.NP = ((3 * H + 15) // 16) * 16
        for lay in self.w.layers:
            if "w_gu" not in lay:
                lay["w_gu"] = interleave_swiglu(lay["w_gate"], lay["w_up"])
            if lay["kind"] == "tree" and "wg" not in lay:
                wg = torch.zeros(L, self.NP, d, device=self.device, dtype=torch.bfloat16)
                bias = torch.zeros(L, self.NP, device=self.device, dtype=torch.float32)
                for gi, g in enumerate("ifr"):
                    wg[:, gi * H:(gi + 1) * H] = lay["w" + g]
                    bias[:, gi * H:(gi + 1) * H] = lay["b" + g]
                lay["wg"] = wg.reshape(L * self.NP, d).contiguous()
                lay["bias_np"] = bias.contiguous()
        hd = d // H
        theta = 10000.0 ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)
        ang = torch.arange(cfg.max_len, dtype=torch.float32)[:, None] * theta[None, :]
        self.rope_cos = ang.cos().to(self.device).contiguous()
        self.rope_sin = ang.sin().to(self.device).contiguous()
        self._bufs = {}
        # every kernel's bounded waits report here; read back without a host
        # sync after each forward and raised at the next one (check_status)
        self.status_word = StatusWord(self.device)
        self.status = self.status_word.tensor
        self.record_events = None   # optional list collecting (name, start, end) events
        self.calls = 0              # C-ABI launches issued (each starts one kernel)

    def stale(self):
        return self.w.stale()

    def check_status(self, sync=False):
        """Raise DispatcherB200Error if a kernel of an earlier forward reported
        a failed bounded wait or a bad input; sync=True waits for the last one."""
        self.status_word.check("PrefillEngine.forward", sync=sync)

    def _buffers(self, B, T):
        key = (B, T)
        if key not in self._bufs:
            cfg, dev, bf = self.cfg, self.device, torch.bfloat16
            d, H, L, ff = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward
            M = B * T
            self._bufs.clear()
            self._bufs[key] = dict(
                x=torch.empty(M, d, device=dev, dtype=bf),
                h=torch.empty(M, d, device=dev, dtype=bf),
                P=torch.empty(M, 3 * d, device=dev, dtype=bf),
                V=torch.empty(M, d, device=dev, dtype=bf),
                U=torch.empty(M, ff, device=dev, dtype=bf),
                gates=torch.empty(B, H, L, T, 4, device=dev, dtype=bf),
                mask=torch.empty(B, T, L, device=dev, dtype=torch.uint8))
        return self._bufs[key]

    def _timed(self, name, flops, fn, *args):
        """Run one C-ABI call; with `record_events` set (a list), bracket it
        with CUDA events on the current stream for per-op timing."""
        ev = self.record_events
        self.calls += 1
        if ev is None:
            return _lib.call(fn, *args)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.call(fn, *args)
        e1.record()
        ev.append((name, flops, e0, e1))

    def _gemm(self, name, a, w, out, epi=0, residual=None, s=None):
        M, K = a.shape
        N = w.shape[0]
        self._timed(name, 2.0 * M * N * K, "dh_gemm_bf16", _p(a), a.stride(0), _p(w), w.stride(0),
                    _p(out), out.stride(0), _p(residual),
                    residual.stride(0) if residual is not None else 0, M, N, K, epi,
                    _p(self.status), s)

    @torch.no_grad()
    def forward(self, ids, caches=None, logits_out=None):
        """ids (B, T) int64 -> logits (B, T, vocab) bf16."""
        if ids.dim() == 1:
            ids = ids.view(1, -1)
        ids = ids.to(self.device, torch.long).contiguous()
        self.check_status()
        cfg, W = self.cfg, self.w
        B, T = ids.shape
        if T > cfg.max_len:
            raise ValueError(f"sequence length {T} exceeds max_len {cfg.max_len}")
        d, H, L, ff, Vv = cfg.d_model, cfg.num_heads, cfg.levels, cfg.dim_feedforward, cfg.vocab_size
        hd = d // H
        M = B * T
        buf = self._buffers(B, T)
        x, h, P, Vb, U, gates, mask = (buf[k] for k in ("x", "h", "P", "V", "U", "gates", "mask"))
        s = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        def call(*a):
            self.calls += 1
            return _lib.call(*a)
        n_lv = n_levels(L, T)
        call("dh_embed_bf16", _p(ids), _p(W.emb), _p(x), M, d, Vv, _p(self.status), s)
        use_mask = bool(cfg.doc_reset)
        if use_mask:
            call("dh_tree_mask", _p(ids), B, T, L, int(cfg.eot_token), 1, _p(mask), s)
        for i, lay in enumerate(W.layers):
            cache = caches[i] if caches is not None else None
            self._timed("rmsnorm", 0.0, "dh_rmsnorm_bf16", _p(x), d, _p(lay["norm1"]), _p(h), d,
                        M, d, s)
            if lay["kind"] == "tree":
                self._gemm("proj3", h, lay["w3"], P, s=s)
                A, Bs = P[:, d:2 * d], P[:, 2 * d:]
                if cache is not None:
                    mlen = cache.B_hist.shape[1]
                    call("dh_copy_rows", _p(Bs), 3 * d, _p(cache.B_hist), d, mlen * d, B, T, d, s)
                self._timed("gates", 2.0 * M * (L if cache is not None else n_lv) * 3 * H * d,
                            "dh_mixer_gates", _p(A), 3 * d, _p(Bs), 3 * d, _p(lay["wg"]),
                            _p(lay["bias_np"]), _p(mask) if use_mask else None, B, T, H, L,
                            self.NP, d, n_lv, _p(gates),
                            _p(cache.rg_hist) if cache is not None else None,
                            cache.rg_hist.shape[1] if cache is not None else 0,
                            _p(self.status), s)
                self._timed("scan", 0.0, "dh_level_scan", _p(P), 3 * d, _p(gates), _p(Vb), d, B,
                            T, H, hd, L, n_lv, _p(cache.V_ring) if cache is not None else None, s)
            else:
                self._gemm("qkv", h, lay["wqkv"], P, s=s)
                call("dh_rope_qk", _p(P), 3 * d, M, T, d, hd, _p(self.rope_cos),
                     _p(self.rope_sin), s)
                if cache is not None:
                    mlen = cache.k.shape[1]
                    call("dh_copy_rows", _p(P[:, d:2 * d]), 3 * d, _p(cache.k), d, mlen * d, B, T, d, s)
                    call("dh_copy_rows", _p(P[:, 2 * d:]), 3 * d, _p(cache.v), d, mlen * d, B, T, d, s)
                self._timed("attn", 0.0, "dh_window_attn_prefill_tc", _p(P), 3 * d, _p(Vb), d, B,
                            T, H, hd, cfg.attn_window, _p(self.status), s)
            self._gemm("out", Vb, lay["w_out"], x, epi=1, residual=x, s=s)
            call("dh_rmsnorm_bf16", _p(x), d, _p(lay["norm2"]), _p(h), d, M, d, s)
            self._gemm("gate_up", h, lay["w_gu"], U, epi=2, s=s)
            self._gemm("down", U, lay["w_down"], x, epi=1, residual=x, s=s)
        call("dh_rmsnorm_bf16", _p(x), d, _p(W.norm_out), _p(h), d, M, d, s)
        # logits rows are padded to a multiple of 8 columns so every row starts
        # 16-byte aligned (full-width vector stores); the result is a view
        vp = ((Vv + 7) // 8) * 8
        if logits_out is None:
            logits_out = torch.empty(M, vp, device=self.device, dtype=torch.bfloat16)
        lo = logits_out.view(M, -1)
        if lo.shape[1] < Vv:
            raise ValueError(f"logits_out has {lo.shape[1]} columns, need {Vv}")
        M_, N_, K_ = M, Vv, h.shape[1]
        self._timed("lm_head", 2.0 * M_ * N_ * K_, "dh_gemm_bf16", _p(h), h.stride(0),
                    _p(W.lm_head), W.lm_head.stride(0), _p(lo), lo.stride(0), None, 0, M_, N_,
                    K_, 0, _p(self.status), s)
        self.status_word.arm()
        return lo.view(B, T, lo.shape[1])[..., :Vv]
