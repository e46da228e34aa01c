"""CPU-side checks of the C ABI and the host logic (no GPU needed)."""

import ctypes
import os
import re

import pytest
import torch

from dispatcher_b200 import _lib, build


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    decl = _lib.parse_header()
    assert len(decl) >= 10
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert b"sm_100a" in lib.dh_version()


def test_header_declarations_cover_all_exports():
    """Every exported dh_* symbol is declared in the public header."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (dh_\w+)", out))
    assert exported == set(_lib.parse_header()), exported ^ set(_lib.parse_header())


def test_errors_are_reported_not_trapped():
    """Argument validation fails with a status and a message, on the host."""
    with pytest.raises(_lib.DispatcherB200Error, match="null pointer"):
        _lib.call("dh_decode_advance", None, None)
    lib = _lib.load()
    rc = lib.dh_decode_attn(None, None, None, None, None, None, None, 1, 1, 16, 2, 64, 0, None)
    assert rc == 2 and b"null" in lib.dh_last_error()


def _status_entry_points():
    return [(n, args) for n, (res, args) in _lib.parse_header().items()
            if res is ctypes.c_int and ctypes.c_void_p in args]


def test_wait_limit_setting_needs_no_device():
    """dh_set_wait_limit only records a host-side value for later launches."""
    lib = _lib.load()
    assert lib.dh_set_wait_limit(12345) == 0
    assert lib.dh_set_wait_limit(-1) == 0


@pytest.mark.parametrize("name,args", _status_entry_points(), ids=lambda v: v if isinstance(v, str) else "")
def test_every_entry_point_rejects_null_pointers_on_the_host(name, args):
    """With every pointer null (sizes 1), each status-returning entry point
    answers DH_ERR_ARG with a message naming itself, before any CUDA call,
    so the check is safe on a machine with or without a GPU."""
    lib = _lib.load()
    vals = [None if a is ctypes.c_void_p else 1 for a in args]
    rc = getattr(lib, name)(*vals)
    assert rc == 2, (name, rc)
    msg = lib.dh_last_error()
    assert msg.startswith(name.encode()) and b"null" in msg, msg


def test_library_is_built_for_sm100a_only():
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert os.path.exists(build.LIB_PATH)


def test_decoder_refuses_without_cuda():
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    from dispatcher_b200 import FusedGraphedHybridDecoder, DispatcherHybridForCausalLM, small_config
    m = DispatcherHybridForCausalLM(small_config())
    with pytest.raises(RuntimeError, match="requires CUDA"):
        FusedGraphedHybridDecoder(m)


def test_ring_layout_constants():
    """Ring j: 2^(j+1) slots at offset 2^(j+1)-2; S = 2^(L+1)-2 (8190 at L=12)."""
    import oracle
    L = 12
    offs = oracle.RING_OFFSETS(L)
    assert offs[-1] + 2 ** L == 2 ** (L + 1) - 2 == 8190
    for j in range(L):
        slots = {oracle.ring_slot(j, t) for t in range(5000, 5000 + 2 ** (j + 1))}
        assert slots == set(range(offs[j], offs[j] + 2 ** (j + 1)))


def test_step_params_layout_matches_header(tmp_path):
    """ctypes mirrors of dh_layer_params / dh_step_params have the C layout."""
    import subprocess
    from dispatcher_b200.step_params import LayerParams, StepParams
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "dispatcher_b200.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu\\n", sizeof(dh_layer_params), '
        'sizeof(dh_step_params), offsetof(dh_step_params, tokens), '
        'offsetof(dh_step_params, layers), offsetof(dh_step_params, status));return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", build.INCLUDE, str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(LayerParams), ctypes.sizeof(StepParams), StepParams.tokens.offset,
            StepParams.layers.offset, StepParams.status.offset]
    assert got == want


@pytest.mark.skipif(torch.cuda.is_available(), reason="host-only argument checks; run without a GPU")
def test_shape_errors_are_reported_before_any_launch():
    """Sizes a kernel cannot take are refused with DH_ERR_SHAPE on the host.
    The pointers are never dereferenced (the checks run first), and the test
    is skipped where a GPU is present."""
    lib = _lib.load()
    buf = ctypes.create_string_buffer(1 << 12)
    p = ctypes.cast(buf, ctypes.c_void_p)
    # gate pre-activations: 12 levels computed over a mask that holds 3 per position
    rc = lib.dh_gate_preacts_fwd(p, 1024, p, 1024, p, p, p, 3, 1, 128, 16, 12, 48, 1024, 12,
                                 p, p, p, None, None)
    assert rc == 1 and b"mask has 3 levels" in lib.dh_last_error()
    # more levels than the layer has, empty batch
    rc = lib.dh_mixer_gates(p, 3072, p, 3072, p, p, p, 1, 128, 16, 4, 48, 1024, 12, p, p, 4096,
                            None, None)
    assert rc == 1 and b"level counts" in lib.dh_last_error()
    rc = lib.dh_mixer_gates(p, 3072, p, 3072, p, p, None, 0, 128, 16, 12, 48, 1024, 12, p,
                            None, 0, None, None)
    assert rc == 1 and b"batch=0" in lib.dh_last_error()
    for args in ((0, 128, 16, 64, 12, 12), (1, 128, 0, 64, 12, 12), (1, 128, 16, 64, 0, 0),
                 (1, 128, 16, 64, 12, 13), (1, 128, 16, 60, 12, 12)):
        batch, T, H, hd, L, n_lv = args
        rc = lib.dh_level_scan(p, 3072, p, p, 1024, batch, T, H, hd, L, n_lv, None, None)
        assert rc == 1 and b"dh_level_scan" in lib.dh_last_error(), args


@pytest.mark.parametrize("batch,L,H,np_,d", [
    (9, 12, 16, 48, 1024),    # the W3 GEMV with the readouts takes one 8-row tile
    (1, 17, 16, 48, 1024),    # at most 16 levels
    (1, 16, 32, 96, 1024),    # 16 rows of the transposed gate weights exceed one ring slot
    (1, 12, 16, 48, 2048),    # d above 1024
    (1, 12, 16, 40, 1024),    # np not a multiple of 16
])
def test_mixer_in_gates_rejects_unsupported_sizes_on_the_host(batch, L, H, np_, d):
    """dh_decode_mixer_in_gates validates its sizes before any CUDA call:
    DH_ERR_SHAPE with its name in the message (non-null dummy pointers, never
    dereferenced)."""
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    rc = lib.dh_decode_mixer_in_gates(p, p, p, p, p, p, p, 4096, batch, d, p, np_, L, H, p, None,
                                      None, None)
    assert rc == 1, rc
    assert lib.dh_last_error().startswith(b"dh_decode_mixer_in_gates")


def test_tree_recur_rejects_unsupported_sizes_on_the_host():
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    for L, H, hd, np_ in ((17, 16, 64, 48), (12, 16, 65, 48), (12, 16, 64, 32)):
        rc = lib.dh_decode_tree_recur(p, p, p, p, p, np_, p, p, p, p, None, 1, 4096, L, H, hd, None)
        assert rc == 1, (L, H, hd, np_, rc)
        assert lib.dh_last_error().startswith(b"dh_decode_tree_recur")
