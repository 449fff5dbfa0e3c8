"""Host logic of the session glue (recavsr_b200/runtime/session.py) on CPU:
the streaming causal-convolution frame bookkeeping must pick exactly the frames
CausalConv3d.forward_streaming (recavsr_infer/models/lq_proj.py:80-139) feeds
its convolution, with the history and first-frame replication, for the
prefix / body block schedule of both LQ projector convolutions."""
import pytest
import torch

from oracle import session as osess
from recavsr_b200.runtime.session import ConvStreamState, conv_input, streaming_window


def _labels(t, frame_dim):
    """The label (first element) of every frame along frame_dim."""
    return t.movedim(frame_dim, 0).reshape(t.shape[frame_dim], -1)[:, 0].tolist()


@pytest.mark.parametrize("frame_dim", [0, 1])
def test_conv_input_frames_follow_the_reference(frame_dim):
    # conv1 (stride 2) over RGB chunks 21, 8, 8 and conv2 (stride 2) over the
    # conv1 outputs 11, 4, 4: the frames fed to the convolution, by label
    cases = {(21, 8, 8): [[0, 0, 0] + list(range(21)), list(range(19, 29)), list(range(27, 37))],
             (11, 4, 4): [[0, 0, 0] + list(range(11)), list(range(9, 15)), list(range(13, 19))]}
    for chunks, expect in cases.items():
        state, start = ConvStreamState(), 0
        for chunk, frames in zip(chunks, expect):
            lab = torch.arange(start, start + chunk, dtype=torch.float32)
            shape = [1, 1]
            shape[frame_dim] = chunk
            x = lab.reshape(*shape) if frame_dim == 0 else lab.reshape(1, chunk)
            x = x.unsqueeze(-1).expand(*x.shape, 3).contiguous()
            inp, n_out = conv_input(x, state, frame_dim, stride=2)
            assert _labels(inp, frame_dim) == [float(v) for v in frames]
            assert n_out == (len(frames) - 4) // 2 + 1
            assert n_out == osess.streaming_window(start, chunk, 2)[3]
            start += chunk
        assert state.seen_frames == sum(chunks)
        assert _labels(state.history, frame_dim) == [float(v) for v in range(start - 3, start)]


def test_streaming_window_matches_oracle_and_rejects_short_chunks():
    for seen, chunk in ((0, 21), (21, 8), (29, 8), (0, 1), (5, 3)):
        assert streaming_window(seen, chunk, 2) == osess.streaming_window(seen, chunk, 2)
    with pytest.raises(ValueError):
        streaming_window(21, 1, 2)
    with pytest.raises(ValueError):
        streaming_window(0, 0, 2)
    state = ConvStreamState()
    conv_input(torch.zeros(1, 21, 2), state, 1, 2)
    with pytest.raises(ValueError):
        conv_input(torch.zeros(1, 8, 3), state, 1, 2)     # history shape changed
