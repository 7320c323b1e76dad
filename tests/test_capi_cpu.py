"""CPU-only checks of the C ABI boundary: the library loads, exports every
entry point include/*.h declares, and rejects bad arguments before touching
the device (no compute call runs here)."""
import ctypes
import glob
import os
import re

import pytest

from freeml_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"^FML_API\s+[\w\s\*]+?\b(fml_\w+)\s*\(", txt, re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 30
    assert "fml_lm_step" in names and "fml_matmul" in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_every_declared_symbol():
    missing = [n for n in declared_functions() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_null_pointer_rejected_without_device():
    lib = _lib.load()
    rc = lib.fml_layernorm(None, None, None, None, None, 4, 8, ctypes.c_float(1e-5), None)
    assert rc == 1
    assert b"fml_layernorm" in lib.fml_last_error()
    with pytest.raises(_lib.FmlError) as e:
        _lib.call("fml_softmax", None, None, 3, 0, None)
    assert e.value.status == 1


def test_engine_config_validation_without_device():
    cfg = _lib.LMConfig(256, 128, 96, 4, 4, 1)  # head dim 24: unsupported
    h = ctypes.c_void_p()
    rc = _lib.load().fml_lm_create(ctypes.byref(cfg), 0, ctypes.byref(h))
    assert rc == 4 and not h.value
    cfg = _lib.LMConfig(256, 128, 130, 4, 4, 1)  # d % H != 0
    assert _lib.load().fml_lm_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == 1
    with pytest.raises(_lib.FmlError):
        _lib.call("fml_set_math_mode", 7)


def test_param_count_matches_oracle_layout():
    from freeml_b200.lm import NanoLLMShape
    from oracle import oracle as O
    cfg = _lib.LMConfig(4096, 512, 512, 8, 8, 32)
    n = int(_lib.load().fml_lm_param_count(ctypes.byref(cfg)))
    assert n == NanoLLMShape(4096, 512, 512, 8, 8).param_count() == O.weight_count(O.LMShape(4096, 512, 512, 8, 8))


def test_zero_size_ops_are_noops():
    # n == 0 returns before any launch
    assert _lib.call("fml_add", None, None, None, 0, None) == 0
    assert _lib.call("fml_gelu", None, None, 0, None) == 0


def _flag_reached(epoch, slot, nslot, flag):
    r = ctypes.c_int(-1)
    _lib.call("fml_tp_flag_check", epoch, slot, nslot, flag, ctypes.byref(r))
    return bool(r.value)


@pytest.mark.parametrize("n_layer", [1, 8, 32, 64, 100])
def test_tp_flag_tags_are_ordered_across_steps_and_the_wrap(n_layer):
    """The peer all-reduce's flags: a waiter passes on its own tag or a later
    one and waits on every earlier one -- also for models of 64 layers and
    more, and where epoch * slots wraps past 2^32."""
    nslot = 2 * n_layer
    M = 1 << 32
    wrap_epoch = M // nslot  # the first step whose tags wrap
    for epoch in (0, 1, 5, wrap_epoch - 1, wrap_epoch, wrap_epoch + 1, (M - 1) // nslot):
        for slot in (0, 1, nslot - 1):
            tag = (epoch * nslot + slot + 1) % M
            assert _flag_reached(epoch, slot, nslot, tag)
            assert _flag_reached(epoch, slot, nslot, (tag + 1) % M)  # a peer one use ahead
            assert not _flag_reached(epoch, slot, nslot, (tag - 1) % M)  # the previous use
            prev_step = ((epoch - 1) * nslot + slot + 1) % M  # the same slot one step earlier
            assert not _flag_reached(epoch, slot, nslot, prev_step)
            # the last slot of the previous step never satisfies slot 0 of this one
            if slot == 0:
                assert not _flag_reached(epoch, 0, nslot, ((epoch - 1) * nslot + nslot) % M)
