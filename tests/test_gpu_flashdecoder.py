"""FlashDecoder's local grouped-query attention on the device
(rc_local_gqa_attention through recavsr_b200.runtime.flashdecoder.local_attention)
against the oracle (pinned to the reference's CPU path and its Triton forward)
and against the reference's own fixtures: the two fixture geometries with
head_dim 64 in fp16 and bf16 (GQA 8:2 and 4:1, temporal groups of 4 and 1
frames), strided K / V views of a cache, and the decoder's own geometry
(8:2 heads, 24 x 24 window, groups of 4 frames over a window of 2 groups) at a
44 x 80 latent grid on sampled query rows.

Tolerances: the kernel rounds P to the input type for the P.V product and the
output to it; the oracle is float64. fp16: |err| <= 4e-3 * max(1, |out|max);
bf16: <= 2.5e-2 * max(1, |out|max)."""
import os

import numpy as np
import pytest
import torch

from oracle import flashdecoder as ofd
from tests.golden import recipes
from tests.util import assert_no_device_error

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "flashdecoder_outputs.npz")
TOL = {torch.float16: 4e-3, torch.bfloat16: 2.5e-2}


def _rounded(x, dtype):
    return torch.from_numpy(x).to(dtype)


def _check(got, ref, dtype):
    ref = np.asarray(ref, np.float32)
    err = np.abs(got.float().cpu().numpy() - ref).max()
    assert err <= TOL[dtype] * max(1.0, np.abs(ref).max()), err


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("tag", ["a", "b"])
def test_fixture_cases_match_oracle(tag, dtype):
    from recavsr_b200.runtime.flashdecoder import local_attention
    b, hq, hk, d, h, w, win, grp, tw, qf, nf = recipes.LOCAL_GQA_CASES[tag]
    q, k, v = (_rounded(x, dtype) for x in recipes.local_gqa_inputs(tag))
    ref = ofd.local_gqa_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), h, w, win, grp, tw)
    got = local_attention(q.cuda(), k.cuda(), v.cuda(), height=h, width=w, window=win, group_size=grp,
                          temporal_window=tw)
    assert got.dtype == dtype and tuple(got.shape) == (b, hq, qf * h * w, d)
    _check(got, ref, dtype)
    assert_no_device_error()


def test_matches_reference_fixtures():
    """The reference's CPU path (fp32 inputs, compared after the kernel's fp16
    rounding) and its Triton forward in fp16, case a."""
    from recavsr_b200.runtime.flashdecoder import local_attention
    fg = np.load(GOLDEN)
    for tag in ("a", "b"):
        _, _, _, _, h, w, win, grp, tw, _, _ = recipes.LOCAL_GQA_CASES[tag]
        q, k, v = (_rounded(x, torch.float16).cuda() for x in recipes.local_gqa_inputs(tag))
        got = local_attention(q, k, v, height=h, width=w, window=win, group_size=grp, temporal_window=tw)
        # fp16 input rounding moves the fp32 reference by up to ~1e-3 as well
        _check(got, fg[f"fd_{tag}_out"], torch.float16)
        if tag == "a":
            _check(got, fg["fd_a_triton_fp16"], torch.float16)
    assert_no_device_error()


def test_strided_cache_views_and_kv_dtype_cast():
    """K / V as views of a larger [B, HK, T, D] cache (the decoder's rolling
    KV buffer) in fp32, cast to the query type as the reference does."""
    from recavsr_b200.runtime.flashdecoder import local_attention
    b, hq, hk, d, h, w, win, grp, tw, qf, nf = recipes.LOCAL_GQA_CASES["a"]
    q, k, v = recipes.local_gqa_inputs("a")
    n = h * w
    cache = torch.zeros(2, b, hk, (nf + 3) * n, d, dtype=torch.bfloat16, device="cuda")
    cache[0, :, :, 3 * n:] = torch.from_numpy(k).to(torch.bfloat16).cuda()
    cache[1, :, :, 3 * n:] = torch.from_numpy(v).to(torch.bfloat16).cuda()
    kv, vv = cache[0, :, :, 3 * n:], cache[1, :, :, 3 * n:]
    assert not kv.is_contiguous()
    qb = _rounded(q, torch.bfloat16).cuda()
    got = local_attention(qb, kv, vv, height=h, width=w, window=win, group_size=grp, temporal_window=tw)
    ref = ofd.local_gqa_attention(qb.float().cpu().numpy(), kv.float().cpu().numpy(), vv.float().cpu().numpy(),
                                  h, w, win, grp, tw)
    _check(got, ref, torch.bfloat16)
    got32 = local_attention(qb, kv.float(), vv.float(), height=h, width=w, window=win, group_size=grp,
                            temporal_window=tw)
    assert torch.equal(got32, got)
    assert_no_device_error()


@pytest.mark.parametrize("qf,nf", [(4, 8), (1, 2), (1, 1)])
def test_decoder_geometry_sampled(qf, nf):
    """flashdecoder_wan22.py's decoder attention (:448-454, :655-675): 8 query
    heads on 2 KV heads, head_dim 64, window (24, 24), on a 44 x 80 latent grid
    (a 704 x 1280 frame / 16). The backbone appends 1 frame to a 2-frame
    window (group 1, temporal window 2; the first call has no history), the
    temporal refinement 4 frames to an 8-frame window (group 4, window 2)."""
    from recavsr_b200.runtime.flashdecoder import local_attention
    h, w, hq, hk, d, win = 44, 80, 8, 2, 64, (24, 24)
    grp = qf
    tw = (2 * qf) // qf
    n = h * w
    g = torch.Generator().manual_seed(5 + qf)
    q = torch.randn(1, hq, qf * n, d, generator=g).to(torch.bfloat16)
    k = torch.randn(1, hk, nf * n, d, generator=g).to(torch.bfloat16)
    v = torch.randn(1, hk, nf * n, d, generator=g).to(torch.bfloat16)
    got = local_attention(q.cuda(), k.cuda(), v.cuda(), height=h, width=w, window=win, group_size=grp,
                          temporal_window=tw).cpu()
    rows = np.random.RandomState(qf).choice(qf * n, 160, replace=False)
    rows = np.concatenate([rows, [0, w - 1, n - 1, qf * n - 1, (qf - 1) * n + 11 * w + 40]])
    ref = ofd.local_gqa_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), h, w, win, grp, tw,
                                  query_rows=rows)
    _check(got[:, :, rows], ref, torch.bfloat16)
    assert_no_device_error()


def test_unsupported_head_dim_raises():
    from recavsr_b200.runtime.flashdecoder import local_attention
    q, k, v = (torch.from_numpy(x).half().cuda() for x in recipes.local_gqa_inputs("c"))
    _, _, _, _, h, w, win, grp, tw, _, _ = recipes.LOCAL_GQA_CASES["c"]
    with pytest.raises(ValueError, match="head_dim 64"):
        local_attention(q, k, v, height=h, width=w, window=win, group_size=grp, temporal_window=tw)
