"""The FlashDecoder drop-in's argument checks, on the CPU: the reference's
messages (flashdecoder_wan22.py:25-35 and :38-80) for bad windows, grids,
head counts and temporal groups, and a loud refusal of CPU tensors (the
reference's CPU fallback is not part of the product)."""
import pytest
import torch

from recavsr_b200.runtime.flashdecoder import local_attention, validate_spatial_window


def _qkv(hq=4, hk=2, qf=2, nf=4, n=12, d=64):
    return torch.zeros(1, hq, qf * n, d), torch.zeros(1, hk, nf * n, d), torch.zeros(1, hk, nf * n, d)


@pytest.mark.parametrize("window", [(3, 4), (0, 2), (2,), None, (True, 2), (2.0, 2)])
def test_bad_windows(window):
    with pytest.raises(ValueError, match="two positive even integers"):
        validate_spatial_window(window)


def test_argument_errors():
    q, k, v = _qkv()
    kw = dict(height=3, width=4, window=(2, 2), group_size=2, temporal_window=1)
    with pytest.raises(ValueError, match="must be positive"):
        local_attention(q, k, v, **{**kw, "group_size": 0})
    with pytest.raises(ValueError, match="Expected 4D"):
        local_attention(q, k[0], v[0], **kw)
    with pytest.raises(ValueError, match="Invalid local grid"):
        local_attention(q, k, v, **{**kw, "width": 5})
    with pytest.raises(ValueError, match="Invalid local grid"):
        local_attention(*_qkv(hq=3), **kw)
    with pytest.raises(ValueError, match="Invalid local grid"):
        local_attention(*_qkv(qf=3, nf=6), **kw)
    with pytest.raises(ValueError, match="CUDA fp16 / bf16"):
        local_attention(q, k, v, **kw)


def test_decoder_session_rejects_unsupported_layouts():
    from recavsr_b200.runtime.decoder import DecoderSession
    with pytest.raises(ValueError, match="64-dimensional heads"):
        DecoderSession({}, height=2, width=2, mean=[0.0] * 48, std=[1.0] * 48, dim=384, num_heads=8)
    with pytest.raises(ValueError, match="two positive even integers"):
        DecoderSession({}, height=2, width=2, mean=[0.0] * 48, std=[1.0] * 48, window=(3, 4))
    with pytest.raises(ValueError, match="CUDA device"):
        DecoderSession({}, height=2, width=2, mean=[0.0] * 48, std=[1.0] * 48, device="cpu")
