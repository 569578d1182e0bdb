"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/vvq2_capi.h declares, and refuses compute without an sm_100 device."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "vvq2_capi.h"


def declared_functions():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vvq2_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("vvq2_init", "vvq2_forward", "vvq2_kv_init", "vvq2_set_layer", "vvq2_decode_step"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import vvq2
    lib = vvq2.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_device_is_an_error_not_a_fallback():
    import vvq2
    if vvq2.lib().vvq2_device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(vvq2.VVQ2Error) as e:
        vvq2.Engine(dict(hidden=128, n_heads=4, n_kv_heads=2, head_dim=64, ffn=384, n_layers=1))
    assert e.value.rc in (-10, -9)
    with pytest.raises(vvq2.VVQ2Error):
        vvq2.rope_neox(__import__("numpy").zeros((1, 1, 64), "float32"), [0], 1e6)


def test_backend_selection_env(monkeypatch):
    import vvq2
    monkeypatch.setenv("VIBEVOICE_BACKEND", "cpu")
    assert vvq2.lib().vvq2_backend_selected() == 0
    monkeypatch.setenv("VIBEVOICE_BACKEND", "B200")
    assert vvq2.lib().vvq2_backend_selected() == (1 if vvq2.lib().vvq2_device_count() > 0 else 0)


def test_version_string():
    import vvq2
    assert b"sm_100a" in vvq2.lib().vvq2_version()


def test_null_context_is_an_argument_error():
    """Every context entry point reports a null context as VVQ2_ERR_INVALID_ARG
    (-2) instead of dereferencing it (checked for the per-frame heads, the
    stack step and the lm_head)."""
    import numpy as np

    import vvq2
    lib = vvq2.lib()
    x = np.zeros((1, 896), np.float32)
    y = np.zeros((1, 896), np.float32)
    assert lib.vvq2_set_connector(None, None, None, None, None, None) == -2
    assert lib.vvq2_connector(None, x.ctypes.data, 1, y.ctypes.data, None) == -2
    assert lib.vvq2_set_eos(None, None, None, None, None) == -2
    assert lib.vvq2_eos(None, x.ctypes.data, 1, y.ctypes.data, None) == -2
    assert lib.vvq2_lm_head(None, 1, x.ctypes.data, None, None, None) == -2
