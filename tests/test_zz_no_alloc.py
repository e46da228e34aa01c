"""dh_decode_attn_noalloc (split-window attention with the library's own
static scratch) against dh_decode_attn (caller scratch) on the same inputs.

The file name sorts last so that the suite runs it after every other test;
it must also pass alone in a fresh process."""

import ctypes

import pytest
import torch

from dispatcher_b200._lib import DispatcherB200Error, call

pytestmark = pytest.mark.gpu

TOL = 1e-2  # bf16 output of one attention read-out; the two entries run the same arithmetic


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(batch, H, max_len, t, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    d = H * 64
    q = torch.randn(batch, d, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(batch, max_len, H, 64, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(batch, max_len, H, 64, device="cuda", generator=g).to(torch.bfloat16)
    t_buf = torch.tensor([t], device="cuda", dtype=torch.int64)
    return q, k, v, t_buf


def _with_scratch(q, k, v, t_buf, nsplit, batch, max_len, H, window):
    y = torch.empty(batch, H * 64, device="cuda", dtype=torch.bfloat16)
    part = torch.zeros(batch, H, nsplit, 66, device="cuda", dtype=torch.float32)
    counters = torch.zeros(batch * H, device="cuda", dtype=torch.int32)
    call("dh_decode_attn", _p(q), _p(k), _p(v), _p(y), _p(t_buf), _p(part), _p(counters),
         nsplit, batch, max_len, H, 64, window, _stream())
    return y


def _no_alloc(q, k, v, t_buf, nsplit, batch, max_len, H, window):
    y = torch.empty(batch, H * 64, device="cuda", dtype=torch.bfloat16)
    call("dh_decode_attn_noalloc", _p(q), _p(k), _p(v), _p(y), _p(t_buf), nsplit, batch,
         max_len, H, 64, window, _stream())
    return y


@pytest.mark.parametrize("batch,H,max_len,t,window,nsplit", [
    (1, 16, 4096, 3899, 1024, 16),   # default config, one row, the decoder's split
    (16, 16, 4096, 3899, 1024, 2),   # sixteen lockstep rows
    (3, 2, 512, 200, 64, 5),         # small config, ragged split of the window
    (20, 16, 1024, 700, 0, 4),       # full causal span, batch over one launch chunk
])
def test_no_alloc_matches_caller_scratch(batch, H, max_len, t, window, nsplit):
    q, k, v, t_buf = _inputs(batch, H, max_len, t, seed=batch * 31 + nsplit)
    want = _with_scratch(q, k, v, t_buf, nsplit, batch, max_len, H, window)
    first = _no_alloc(q, k, v, t_buf, nsplit, batch, max_len, H, window)
    second = _no_alloc(q, k, v, t_buf, nsplit, batch, max_len, H, window)
    torch.cuda.synchronize()
    assert (first.float() - want.float()).abs().max().item() <= TOL
    assert (second.float() - want.float()).abs().max().item() <= TOL


def test_no_alloc_rejects_oversize():
    q, k, v, t_buf = _inputs(2, 16, 256, 100, seed=7)
    # 64 rows x 16 heads x 16 splits x 66 floats > 131072
    with pytest.raises(DispatcherB200Error, match="exceeds the built-in scratch"):
        call("dh_decode_attn_noalloc", _p(q), _p(k), _p(v), _p(q), _p(t_buf), 16, 64, 256, 16,
             64, 0, _stream())
    # 80 rows x 16 heads = 1280 counters > 1024 (one split keeps the partials small)
    with pytest.raises(DispatcherB200Error, match="counters"):
        call("dh_decode_attn_noalloc", _p(q), _p(k), _p(v), _p(q), _p(t_buf), 1, 80, 256, 16,
             64, 0, _stream())
