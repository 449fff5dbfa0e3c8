"""The C ABI library loads and exports every entry point include/recavsr_b200.h
declares (CPU: no compute calls)."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    with open(os.path.join(ROOT, "include", "recavsr_b200.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"^(?:int|long long) (rc_\w+)\(", src, flags=re.M)))


def test_header_symbols_exported():
    from recavsr_b200 import _lib
    lib = _lib.library()
    names = declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.rc_abi_version() == 1


def test_bindings_cover_header():
    from recavsr_b200 import _lib
    assert set(declared()) <= set(_lib._SIGNATURES), set(declared()) - set(_lib._SIGNATURES)


def test_dynamic_symbols_are_c_abi():
    so = os.path.join(ROOT, "recavsr_b200", "librecavsr_b200.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T rc_" in l}
    assert set(declared()) <= exported


def test_argument_errors_raise_valueerror_without_gpu():
    """Invalid sizes are rejected before any device work (no GPU needed)."""
    import pytest
    from recavsr_b200 import _lib
    with pytest.raises(ValueError, match="multiple of 16"):
        _lib.call("rc_nvfp4_quantize", None, 4, 15, 15, 1.0, None, None, None)
    with pytest.raises(ValueError):
        _lib.call("rc_kv_commit", None, None, 0, None, None, 0, 24, 1, 9, None, None, None)
