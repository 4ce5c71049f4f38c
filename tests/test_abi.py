"""CPU checks of the C ABI: the library loads and exports every entry point the
header declares; status strings resolve. No kernel is launched."""
import re
from pathlib import Path

import pytest

from theorem_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "theorem_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(thm_[A-Za-z0-9_]+)\s*\(", text)))


def test_library_is_built():
    assert _lib.LIB_PATH.exists(), "run python -m theorem_b200.build"


def test_every_declared_symbol_is_exported():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 7
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/theorem_b200.h but not exported"


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.exported_symbols())


@pytest.mark.parametrize("code", range(0, 8))
def test_status_strings(code):
    s = _lib.status_string(code)
    assert s.startswith("THM_")


def test_status_mapping_raises_reference_exception_classes():
    with pytest.raises(AssertionError):
        _lib.check(_lib.THM_ERR_INVALID, "x")
    with pytest.raises(AssertionError):
        _lib.check(_lib.THM_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.THM_ERR_TIMEOUT, "x")
    _lib.check(_lib.THM_OK, "x")


def test_invalid_arguments_rejected_without_gpu():
    """Argument validation happens on the host before any CUDA call."""
    lib = _lib.load()
    # W = 0 is invalid; empty tensors are a no-op that never touches the device.
    assert lib.thm_causal_conv1d_fwd(None, None, None, None, 1, 1, 1, 0, 0, 0, 0, 0, None) == _lib.THM_ERR_INVALID
    assert lib.thm_causal_conv1d_fwd(None, None, None, None, 0, 8, 8, 4, 0, 0, 0, 0, None) == _lib.THM_OK
    assert lib.thm_causal_conv1d_fwd(None, None, None, None, 1, 8, 8, 4, 7, 0, 0, 0, None) == _lib.THM_ERR_INVALID


def test_conv_pair_rejects_arguments_without_gpu():
    """thm_causal_conv1d_pair_fwd checks its arguments on the host, before any CUDA
    call; an empty problem is a no-op."""
    lib = _lib.load()
    f = lib.thm_causal_conv1d_pair_fwd
    fake = 1 << 20  # never dereferenced: every case returns before touching memory
    p8 = [fake] * 8
    assert f(*p8, 1, 8, 8, 0, 1, 1, 0, None) == _lib.THM_ERR_INVALID          # W = 0
    assert f(*([None] * 8), 0, 8, 8, 4, 1, 1, 0, None) == _lib.THM_OK         # empty batch
    assert f(*([None] * 8), 1, 8, 8, 4, 1, 1, 0, None) == _lib.THM_ERR_INVALID  # null pointers
    assert f(*p8, 1, 8, 8, 4, 1, 7, 0, None) == _lib.THM_ERR_INVALID          # unknown activation
    assert f(*p8, 1, 8, 8, 4, 9, 1, 0, None) == _lib.THM_ERR_INVALID          # unknown dtype
    assert f(*p8, 1, 6, 8, 4, 1, 1, 0, None) == _lib.THM_ERR_UNSUPPORTED      # D % 4 != 0
    assert f(*p8, 1, 8, 8, 65, 1, 1, 0, None) == _lib.THM_ERR_UNSUPPORTED     # W > 64
    assert f(*p8, 1, 8, 8, 4, 1, 1, 16, None) == _lib.THM_ERR_INVALID         # group does not divide D
    assert f(*p8, 1, 48, 8, 4, 1, 1, 24, None) == _lib.THM_ERR_UNSUPPORTED    # group size not built
    bad = [fake + 4] + [fake] * 7
    assert f(*bad, 1, 8, 8, 4, 1, 1, 0, None) == _lib.THM_ERR_ALIGNMENT       # x0 not 16-byte aligned


def test_conv_folded_recompute_w_u_rejects_arguments_without_gpu():
    """thm_recompute_w_u_conv_fwd checks its arguments on the host, before any CUDA call:
    only an in-kernel A (a_mode +1 / -1), a known activation, T % 64 == 0, and conv
    width 4 with K, V in {64, 128}; an empty problem is a no-op."""
    lib = _lib.load()
    f = lib.thm_recompute_w_u_conv_fwd
    fake = 1 << 20  # never dereferenced: every case returns before touching memory
    p9 = [fake] * 9
    ok_shape = (1, 64, 1, 128, 128, 4, 1)  # B, T, H, K, V, width, activation
    assert f(*p9, *ok_shape, 0, None) == _lib.THM_ERR_INVALID          # a_mode 0: A is not taken
    assert f(*p9, 1, 65, 1, 128, 128, 4, 1, 1, None) == _lib.THM_ERR_INVALID  # T % 64 != 0
    assert f(*p9, 1, 64, 1, 128, 128, 4, 7, 1, None) == _lib.THM_ERR_INVALID  # unknown activation
    assert f(*([None] * 9), *ok_shape, 1, None) == _lib.THM_ERR_INVALID       # null pointers
    assert f(*([None] * 9), 0, 64, 1, 128, 128, 4, 1, 1, None) == _lib.THM_OK  # empty batch
    assert f(*p9, 1, 64, 1, 128, 128, 3, 1, 1, None) == _lib.THM_ERR_UNSUPPORTED  # conv width 3
    assert f(*p9, 1, 64, 1, 96, 128, 4, 1, -1, None) == _lib.THM_ERR_UNSUPPORTED  # K = 96
