"""dispatcher_b200 — B200 (sm_100a) backend for the Dispatcher-Hybrid mixer.

Hand-written CUDA kernels behind a C ABI (include/dispatcher_b200.h,
`lib/libdispatcher_b200.so`), driven from Python through ctypes:

    from dispatcher_b200 import DispatcherHybridForCausalLM, FusedGraphedHybridDecoder
    model = DispatcherHybridForCausalLM(seed=0).to("cuda", torch.bfloat16)
    dec = FusedGraphedHybridDecoder(model)
    logits = dec.prefill(ids); logits = dec.step(tok)

There is no CPU path: without a CUDA device or the built library every
entry point raises.
"""

from .config import DispatcherConfig, small_config  # noqa: F401
from .weights import make_state_dict  # noqa: F401
from .modeling import DispatcherHybridForCausalLM  # noqa: F401
from .decoding import FusedGraphedHybridDecoder, GraphedHybridDecoder  # noqa: F401
from .fused_gates import fused_gate_preacts  # noqa: F401

__version__ = "0.1.0"
