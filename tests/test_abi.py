"""The C-ABI library loads and exports every symbol include/tenzor_cuda.h declares; argument
validation and the no-GPU failure path work without launching anything.  CPU only."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "tenzor_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tz_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from tenzor_b200 import _lib
    assert os.path.exists(_lib.LIB_PATH), "run python -m tenzor_b200.build"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    declared = header_functions()
    missing = [f for f in declared if f not in syms]
    assert not missing, missing
    assert sorted(_lib.EXPORTS) == declared  # the Python binding covers exactly the header


def test_library_loads_and_binds():
    from tenzor_b200 import _lib
    L = _lib.lib()
    assert L.tz_version().decode().startswith("tenzor_b200")
    for name in _lib.EXPORTS:
        assert getattr(L, name) is not None


def test_argument_validation_without_device():
    from tenzor_b200 import _lib
    L = _lib.lib()
    assert L.tz_layernorm_last_dim(None, None, None, None, None, 4, 384, 1e-12, None) == _lib.TZ_EINVAL
    assert "bad arguments" in L.tz_get_last_error().decode()
    assert L.tz_gemm_i8_i32(None, None, None, None, 1, 16, 16, None) == _lib.TZ_EINVAL
    assert L.tz_arctic_forward(None, None, None, 1, None) == _lib.TZ_EINVAL
    assert L.tz_arctic_load(None, None, 0, None) == _lib.TZ_EINVAL
    assert L.tz_arctic_load_safetensors(None, b"/nonexistent", 0, None) == _lib.TZ_EINVAL


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from tenzor_b200 import TenzorError
    from tenzor_b200.runtime import Context
    with pytest.raises(TenzorError):
        Context(0)


def test_missing_library_raises(monkeypatch, tmp_path):
    from tenzor_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "libtenzor_cuda.so"))
    with pytest.raises(ImportError):
        _lib.lib()
