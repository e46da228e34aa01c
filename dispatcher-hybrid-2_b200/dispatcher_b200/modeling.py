"""Module tree mirror of `DispatcherHybridForCausalLM`
(dispatcher_hybrid/modeling_dispatcher.py:36-442) for hosts without the
reference package.

The classes hold the reference's parameters under the reference's names,
so state dicts move between the two unchanged.  They contain no eager
arithmetic: `forward` runs the B200 parallel-forward engine and
`fast_generate` the B200 decoder.  A reference model object can use the
same backend directly (see `dispatcher_b200.integration`).
"""

from collections import namedtuple

import torch
import torch.nn as nn

from .config import DispatcherConfig
from .weights import make_state_dict

CausalLMOutput = namedtuple("CausalLMOutput", ["loss", "logits", "hidden_states"])


class DispatcherMixer(nn.Module):
    def __init__(self, config):
        super().__init__()
        d, H, L = config.d_model, config.num_heads, config.levels
        self.embed_dim, self.num_heads, self.head_dim, self.levels = d, H, d // H, L
        self.use_fused_gates = True
        self.linear_in = nn.Linear(d, d, bias=False)
        self.gate_hidden = nn.Linear(d, d, bias=False)
        self.gate_hidden_src = nn.Linear(d, d, bias=False)
        self.gate_out = nn.Parameter(torch.empty(L, H, d))
        self.gate_out_bias = nn.Parameter(torch.full((L, H), float(config.gate_bias_flat)))
        self.forget_out = nn.Parameter(torch.empty(L, H, d))
        self.forget_out_bias = nn.Parameter(torch.full((L, H), float(config.gate_fbias_flat)))
        self.reset_out = nn.Parameter(torch.empty(L, H, d))
        self.reset_out_bias = nn.Parameter(torch.full((L, H), 2.0))
        self.linear_out = nn.Linear(d, d, bias=False)


class WindowAttention(nn.Module):
    def __init__(self, config):
        super().__init__()
        d, H = config.d_model, config.num_heads
        self.embed_dim, self.num_heads, self.head_dim = d, H, d // H
        self.window = config.attn_window
        self.linear_q = nn.Linear(d, d, bias=False)
        self.linear_k = nn.Linear(d, d, bias=False)
        self.linear_v = nn.Linear(d, d, bias=False)
        self.linear_out = nn.Linear(d, d, bias=False)


class SwiGLU(nn.Module):
    def __init__(self, config):
        super().__init__()
        d, ff = config.d_model, config.dim_feedforward
        self.linear_gate = nn.Linear(d, ff, bias=False)
        self.linear_up = nn.Linear(d, ff, bias=False)
        self.linear_down = nn.Linear(ff, d, bias=False)


class DispatcherBlock(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.mixer = DispatcherMixer(config)
        self.ffn = SwiGLU(config)
        self.norm1 = nn.RMSNorm(config.d_model)
        self.norm2 = nn.RMSNorm(config.d_model)


class AttentionBlock(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.attn = WindowAttention(config)
        self.ffn = SwiGLU(config)
        self.norm1 = nn.RMSNorm(config.d_model)
        self.norm2 = nn.RMSNorm(config.d_model)


class DispatcherHybridForCausalLM(nn.Module):
    """Parameter container with the reference's module tree; compute is B200-only.

    The weights are filled with `weights.make_state_dict(config, seed)`."""

    main_input_name = "input_ids"

    def __init__(self, config=None, seed=0, nondegenerate=False):
        super().__init__()
        config = config or DispatcherConfig()
        self.config = config
        slots = config.attn_slots()
        self.embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.blocks = nn.ModuleList(
            AttentionBlock(config) if i in slots else DispatcherBlock(config)
            for i in range(config.num_layers))
        self.norm_out = nn.RMSNorm(config.d_model)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight                  # tied (:265)
        self._engine = None
        self.load_state_dict(make_state_dict(config, seed, nondegenerate), strict=True)

    # ------------------------------------------------------------ loading
    @classmethod
    def from_pretrained(cls, path, dtype=None, device=None):
        """A released model directory: config.json + model.safetensors (or
        sharded / pytorch_model.bin), the layout the reference's
        save_pretrained and scripts/convert_checkpoint.py write."""
        from .checkpoint import load_pretrained
        cfg, sd = load_pretrained(path)
        return cls._with_weights(cfg, sd, dtype, device)

    @classmethod
    def from_research_checkpoint(cls, path, dtype=None, device=None):
        """A research training checkpoint, remapped as the reference's converter
        does (scripts/convert_checkpoint.py:25-57)."""
        from .checkpoint import load_research_checkpoint
        cfg, sd = load_research_checkpoint(path)
        return cls._with_weights(cfg, sd, dtype, device)

    @classmethod
    def _with_weights(cls, cfg, sd, dtype, device):
        from .checkpoint import check_keys
        model = check_keys(cls(cfg), sd)
        if dtype is not None or device is not None:
            model = model.to(device=device, dtype=dtype)
        return model.eval()

    # ------------------------------------------------------------ reference API
    def enable_fused_gates(self, enabled=True):
        """modeling_dispatcher.py:365-377.  The B200 engine is the only compute
        path of this mirror; enabling checks that it can load now."""
        if enabled:
            from . import _lib
            _lib.load()
        for blk in self.blocks:
            if hasattr(blk, "mixer"):
                blk.mixer.use_fused_gates = enabled
        return self

    def forward(self, input_ids=None, **kwargs):
        if input_ids is None:
            raise ValueError("DispatcherHybridForCausalLM requires input_ids "
                             "(the tree mask is built from token identities)")
        if input_ids.size(1) > self.config.max_len:
            raise ValueError(f"sequence length {input_ids.size(1)} exceeds max_len "
                             f"{self.config.max_len}")
        from .engine import PrefillEngine
        if self._engine is None or self._engine.stale():
            self._engine = PrefillEngine(self)
        logits = self._engine.forward(input_ids)
        return CausalLMOutput(loss=None, logits=logits, hidden_states=None)

    @torch.no_grad()
    def fast_generate(self, input_ids, max_new_tokens=50, do_sample=False, temperature=1.0,
                      top_k=None, eos_token_id=None, num_return_sequences=1, decoder="auto"):
        from .generation import fast_generate
        return fast_generate(self, input_ids, max_new_tokens, do_sample, temperature, top_k,
                             eos_token_id, num_return_sequences, decoder)
