"""Model configuration mirror.

Same constructor arguments, defaults and validation as the reference
`DispatcherConfig` (dispatcher_hybrid/configuration_dispatcher.py:35-82), as a
plain Python object so the B200 backend runs without `transformers`.  A
reference config object can be passed anywhere this one is accepted: the
backend reads only the attributes listed here.
"""

import math


class DispatcherConfig:
    model_type = "dispatcher-hybrid"

    def __init__(self, vocab_size=50257, d_model=1024, num_heads=16,
                 dim_feedforward=2816, num_layers=18, max_len=4096,
                 attn_layers=(8, 17), attn_window=1024, gate_bias_flat=-2.0,
                 gate_fbias_flat=2.0, doc_reset=True, eot_token=50256,
                 tie_word_embeddings=True, use_cache=False, bos_token_id=50256,
                 eos_token_id=50256, **kwargs):
        # configuration_dispatcher.py:55-58
        if max_len & (max_len - 1):
            raise ValueError(f"max_len must be a power of two, got {max_len}")
        if d_model % num_heads:
            raise ValueError("d_model must be divisible by num_heads")
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.num_heads = num_heads
        self.dim_feedforward = dim_feedforward
        self.num_layers = num_layers
        self.max_len = max_len
        self.attn_layers = tuple(attn_layers)
        self.attn_window = attn_window
        self.gate_bias_flat = gate_bias_flat
        self.gate_fbias_flat = gate_fbias_flat
        self.doc_reset = doc_reset
        self.eot_token = eot_token
        self.tie_word_embeddings = tie_word_embeddings
        self.use_cache = use_cache
        self.bos_token_id = bos_token_id
        self.eos_token_id = eos_token_id
        for k, v in kwargs.items():
            setattr(self, k, v)

    @property
    def levels(self):
        # configuration_dispatcher.py:80-82
        return int(math.log2(self.max_len))

    @property
    def head_dim(self):
        return self.d_model // self.num_heads

    def attn_slots(self):
        """0-indexed block positions that hold window attention
        (modeling_dispatcher.py:270-275: 1-indexed `attn_layers`, disabled
        when `attn_window` is 0)."""
        if self.attn_window <= 0:
            return set()
        return {i - 1 for i in self.attn_layers}

    def to_dict(self):
        keys = ("vocab_size", "d_model", "num_heads", "dim_feedforward",
                "num_layers", "max_len", "attn_layers", "attn_window",
                "gate_bias_flat", "gate_fbias_flat", "doc_reset", "eot_token")
        return {k: getattr(self, k) for k in keys}

    def __repr__(self):
        return f"DispatcherConfig({self.to_dict()})"


def small_config(**overrides):
    """A reduced shape used by the parity tests: every kernel path (tree and
    attention blocks, level masking, window clipping, vocab tails) is live,
    at sizes the CPU oracle finishes in well under a second."""
    kw = dict(vocab_size=515, d_model=128, num_heads=2, dim_feedforward=384,
              num_layers=4, max_len=256, attn_layers=(2,), attn_window=64,
              eot_token=514, bos_token_id=514, eos_token_id=514)
    kw.update(overrides)
    return DispatcherConfig(**kw)
