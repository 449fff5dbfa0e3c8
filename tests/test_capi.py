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


def test_session_and_commit_entry_points_reject_bad_arguments():
    """The session-glue entry points and the planned KV commit reject invalid
    geometry and strides on the host, before any device work (every call
    here fails validation, most with null pointers, so nothing is launched)."""
    import pytest
    from recavsr_b200 import _lib
    with pytest.raises(ValueError, match="bad geometry"):          # cin % 8
        _lib.call("rc_conv3d_im2col", None, 0, 0, 0, 0, 0, 12, 10, 4, 4, 2, 1, 4, None, 0, None)
    with pytest.raises(ValueError, match="bad geometry"):          # unshuffle not a multiple of 8
        _lib.call("rc_conv3d_im2col", None, 0, 0, 0, 0, 4, 768, 10, 4, 4, 2, 1, 4, None, 0, None)
    with pytest.raises(ValueError, match="need 10 input frames"):  # (4 - 1) * 2 + 4 > 9
        _lib.call("rc_conv3d_im2col", None, 0, 0, 0, 0, 16, 768, 9, 4, 4, 2, 1, 4, None, 0, None)
    with pytest.raises(ValueError, match="16-byte aligned"):       # null source
        _lib.call("rc_conv3d_im2col", None, 8, 8, 8, 8, 0, 64, 10, 4, 4, 2, 1, 4, None, 2304, None)
    with pytest.raises(ValueError, match="bad shape"):             # C > 8192
        _lib.call("rc_channel_rmsnorm_silu", None, 16384, 4, 16384, None, 1e-6, None, 16384, None)
    with pytest.raises(ValueError, match="bad shape"):             # C % 8
        _lib.call("rc_channel_rmsnorm_silu", None, 12, 4, 12, None, 1e-6, None, 12, None)
    with pytest.raises(ValueError, match="bad shape"):             # H % ph
        _lib.call("rc_patchify", None, 0, 1, 1, 1, 16, 2, 5, 6, 2, 2, None, 64, None)
    with pytest.raises(ValueError, match="bad shape"):             # recycle_frames > F
        _lib.call("rc_unpatchify_residual", None, 64, None, None, None, 16, 2, 4, 6, 2, 2, 3, None)
    with pytest.raises(ValueError, match="row stride below row_bytes"):
        _lib.call("rc_kv_commit_planned", 4096, 4096, 16, 32, 4096, 4096, 32, 32, 24, 2, 2, 4096, None)
    with pytest.raises(ValueError, match="bad shape"):             # row_bytes % 16
        _lib.call("rc_kv_commit_planned", None, None, 0, 0, None, None, 0, 24, 1, 2, 2, None, None)


def test_decoder_pipeline_colorfix_entry_points_reject_bad_arguments():
    """The FlashDecoder, frame-preparation and colour-correction entry points
    validate on the host before any device work (every call fails validation)."""
    import ctypes as C

    import pytest
    from recavsr_b200 import _lib
    st9 = (C.c_longlong * 9)(*([64] * 9))
    with pytest.raises(ValueError, match="head_dim 32"):
        _lib.call("rc_local_gqa_attention", None, None, None, st9, 1, 8, 2, 4, 8, 6, 20, 32, 4, 8, 4, 2, 0, None,
                  None, None)
    with pytest.raises(ValueError, match="alignment"):       # HQ % HK
        _lib.call("rc_local_gqa_attention", None, None, None, st9, 1, 6, 4, 4, 8, 6, 20, 64, 4, 8, 4, 2, 0, None,
                  None, None)
    with pytest.raises(ValueError, match="alignment"):       # odd window
        _lib.call("rc_local_gqa_attention", None, None, None, st9, 1, 8, 2, 4, 8, 6, 20, 64, 3, 8, 4, 2, 0, None,
                  None, None)
    with pytest.raises(ValueError, match="missing pointer"):
        _lib.call("rc_local_gqa_attention", None, None, None, st9, 1, 8, 2, 4, 8, 6, 20, 64, 4, 8, 4, 2, 0, None,
                  None, None)
    with pytest.raises(ValueError, match="bad arguments"):
        _lib.call("rc_fd_kv_norm", None, 768, 10, 512, 2, None, None, 1e-5, None, None, 640, 0, None)
    with pytest.raises(ValueError, match="bad arguments"):   # nf < cur
        _lib.call("rc_fd_rope_gather", None, 768, 8, 2, 4, 0, 2, 0, 8, 4, 6, None, None, 0, None, 8, None, None,
                  None, None)
    with pytest.raises(ValueError, match="bad arguments"):   # H % 8
        _lib.call("rc_fd_silu", None, 4, 12, 0, None, None)
    with pytest.raises(ValueError, match="bad arguments"):   # f0 + frames > 4
        _lib.call("rc_fd_pixel_shuffle", None, 768, 3, 2, 4, 4, 6, None, None)
    with pytest.raises(ValueError, match="bad arguments"):
        _lib.call("rc_fd_lr_group", None, 48, 24, 0, None, None, None)
    with pytest.raises(ValueError, match="bad arguments"):
        _lib.call("rc_cf_adain", None, 0, None, 0, 3, 100, None, 0, None, None)
    with pytest.raises(ValueError, match="bad arguments"):   # radius 0
        _lib.call("rc_cf_wavelet_level", None, 0, None, None, None, None, None, None, 1, 8, 8, 0, 1, 0, None)
    with pytest.raises(ValueError, match="bad arguments"):
        _lib.call("rc_cf_bicubic_u8", None, 1, 4, 4, 16, 16, None, None)
    with pytest.raises(ValueError, match="missing pointer"):
        _lib.call("rc_enlarge_block", None, 0, 0, 1, 8, 4, 4, 16, 16, 0, None, None)
    with pytest.raises(ValueError, match="bad shape"):       # no strips
        _lib.call("rc_strip_blend", 0, None, None, None, None, None, None, 8, 8, None, 24, None)
    assert _lib.library().rc_cf_adain_workspace(6, 100000) == 6 * 7 * 4 * 8
