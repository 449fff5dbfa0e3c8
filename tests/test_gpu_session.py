"""Session glue on the GPU (recavsr_b200/runtime/session.py, csrc/session.cu)
against the oracle and the reference's own TransformerSession.step
(tests/golden/session_outputs.npz): the LQ projector's streaming output over a
prefix and two body blocks, the embedding entering the first DiT block, the
output head, and a whole StreamingSession (FusedBlock layer loop included)."""
import os

import numpy as np
import pytest
import torch

from oracle import session as osess
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes
from tests.test_oracle_session import session_setup
from tests.util import assert_no_device_error, dev_bf16, host

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# bf16 convolutions / linears against the oracle's float64 accumulation with
# the same bf16 rounding points: a bf16 ulp or two
STAGE_REL, STAGE_L2 = 2e-2, 1e-2


@pytest.fixture(scope="module")
def sgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "session_outputs.npz"))


def _check(got, ref, what, rel=STAGE_REL, l2=STAGE_L2):
    mx = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    r2 = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert mx < rel and r2 < l2, f"{what}: max {mx:.3e}, rel L2 {r2:.3e}"


def _glue(p):
    from recavsr_b200.runtime.session import SessionGlue
    return SessionGlue({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in p.items()}, "cuda")


def test_lq_projector_matches_oracle_and_reference(sgold):
    p, steps = session_setup(sgold["session_meta"])
    glue = _glue(p)
    state, ostate = glue.lq.create_streaming_state(), osess.new_lq_state()
    for i, (video, _) in enumerate(steps):
        got = host(glue.lq.forward_streaming(dev_bf16(video), state))
        _check(got, osess.lq_project_stream(video[0], ostate, p), f"block {i} vs oracle")
        _check(got, bf16_from_bits(sgold[f"session_step{i}_lqproj"])[0], f"block {i} vs reference")
    assert_no_device_error()


def test_embedding_and_head_match_reference(sgold):
    p, steps = session_setup(sgold["session_meta"])
    glue = _glue(p)
    state = glue.lq.create_streaming_state()
    for i, (video, noise) in enumerate(steps):
        if i == 0:
            rec = torch.zeros(noise.shape, dtype=torch.bfloat16, device="cuda")
        else:
            rec = dev_bf16(sgold[f"session_step{i - 1}_result"][:, :, -2:])
        nz = torch.from_numpy(noise).cuda()
        hidden = glue.embed(nz, dev_bf16(video), rec, state)
        _check(host(hidden), bf16_from_bits(sgold[f"session_step{i}_hidden_in"])[0], f"embed {i}")
        result, recycle = glue.head(dev_bf16(bf16_from_bits(sgold[f"session_step{i}_hidden_out"])[0]), nz)
        got, ref = host(result)[0], sgold[f"session_step{i}_result"][0]
        _check(noise[0] - got, noise[0] - ref, f"head {i} prediction")
        np.testing.assert_array_equal(host(recycle)[0], bf16_round(got[:, -2:]))
    assert_no_device_error()


@pytest.mark.parametrize("graphs", [False, True])
def test_streaming_session_matches_reference(sgold, graphs):
    """Prefix + two body blocks through the whole step: embedding, the FusedBlock
    layer loop with the static router, head. The layers run NVFP4 linears, so
    the bound is the block-level one of the layer-stack tests."""
    from recavsr_b200.runtime.block import FusedBlock, LayerStack, rope_tables
    from recavsr_b200.runtime.session import StreamingSession
    dim, heads, ffn, channels, height, width, h1, h2, enc_len = (int(v) for v in sgold["session_meta"])
    p, steps = session_setup(sgold["session_meta"])
    H, W = height // 32, width // 32
    tables = rope_tables(dim // heads, H, W, "cuda")
    bp = [recipes.block_params(dim, heads, ffn, enc_len=enc_len, seed=70 + i) for i in range(2)]
    blocks = []
    for b in bp:
        w = {k: dev_bf16(v) for k, v in b.items()}
        w["timestep_proj"], w["encoder"] = dev_bf16(bp[0]["timestep_proj"]), dev_bf16(bp[0]["encoder"])
        w["heads"] = heads
        blocks.append(FusedBlock(w, H, W, tables))
    session = StreamingSession(LayerStack(blocks, ["recent_2", "none"]), _glue(p), height, width,
                               graphs=graphs)
    for i, (video, noise) in enumerate(steps):
        result = session.step(dev_bf16(video), noise=torch.from_numpy(noise).cuda())
        got, ref = host(result)[0], sgold[f"session_step{i}_result"][0]
        _check(noise[0] - got, noise[0] - ref, f"step {i} prediction", rel=0.15, l2=0.06)
    with pytest.raises(ValueError):
        session.step(dev_bf16(steps[1][0][:, :, :4]))
    assert_no_device_error()


def test_step_host_matches_step(sgold):
    """The pinned-host streaming entry (copies on a side stream, double-buffered
    staging) returns exactly what step() returns while the caller refills one
    pinned input buffer after each step's input_consumed event."""
    from recavsr_b200.runtime.block import FusedBlock, LayerStack, rope_tables
    from recavsr_b200.runtime.session import StreamingSession
    dim, heads, ffn, channels, height, width, h1, h2, enc_len = (int(v) for v in sgold["session_meta"])
    p, steps = session_setup(sgold["session_meta"])
    H, W = height // 32, width // 32
    tables = rope_tables(dim // heads, H, W, "cuda")
    bp = [recipes.block_params(dim, heads, ffn, enc_len=enc_len, seed=70 + i) for i in range(2)]

    def make():
        blocks = []
        for b in bp:
            w = {k: dev_bf16(v) for k, v in b.items()}
            w["heads"] = heads
            blocks.append(FusedBlock(w, H, W, tables))
        return StreamingSession(LayerStack(blocks, ["recent_2", "none"]), _glue(p), height, width,
                                seed=7, graphs=True)
    a, b = make(), make()
    rs = np.random.RandomState(9)
    lq = [steps[0][0]] + [bf16_round(rs.uniform(-1, 1, steps[1][0].shape).astype(np.float32))
                          for _ in range(5)]
    want = [host(a.step(dev_bf16(x)))[0] for x in lq]
    # One pinned input buffer per block shape, refilled as soon as the previous
    # step has consumed it (HostStep.input_consumed), the way a streaming
    # decoder reuses its frame buffer; each output read after output_ready.
    outs, handles, bufs = [], [], {}
    for x in lq:
        hin = bufs.get(x.shape)
        if hin is None:
            hin = bufs[x.shape] = torch.empty(x.shape, dtype=torch.bfloat16).pin_memory()
        elif handles:
            handles[-1].input_consumed.synchronize()
        hin.copy_(torch.from_numpy(x))
        shape = (1, channels, 6 if not outs else 2, height // 16, width // 16)
        outs.append(torch.empty(shape, dtype=torch.float32).pin_memory())
        handles.append(b.step_host(hin, outs[-1]))
    for i, (o, h, w_) in enumerate(zip(outs, handles, want)):
        h.output_ready.synchronize()
        np.testing.assert_array_equal(o.numpy()[0], w_, err_msg=f"block {i}")
    b.sync_host()
    assert_no_device_error()
