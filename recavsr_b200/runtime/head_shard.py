"""Head-sharded single stream: one high-resolution stream over P ranks.

The reference scales out by independent streams or spatial strips
(recavsr_infer/strips.py:24-45), each a full TransformerSession; a single
stream runs the layer loop of transformer.py:311-318 on one device. For one
stream too large for one GPU's time budget (3840x2176 output: 120x68 latent
tokens per frame, 16320 query tokens per 2-frame block) this module splits the
same layer loop over a process group, one GPU per rank, Ulysses-style:

* token shard (rank r holds tokens [r*N/P, (r+1)*N/P) of the block): the three
  LayerNorm + AdaLN passes, every NVFP4 linear, RMSNorm across heads, spatial
  RoPE (each rank reads the spatial-table rows of its own tokens), the cross
  attention (its 512 prompt K/V replicated) and the FFN -- everything of
  PreparedBlock.forward (transformer.py:81-134) that is per token;
* head shard (rank r holds heads [r*heads/P, (r+1)*heads/P) of every token):
  the routed self-attention (temporal RoPE, cache planes by slot id, local
  windows) and the KV cache of those heads, so cache traffic never crosses GPUs;
* two all-to-alls per layer between them: q / k / v (token -> head shard)
  before the attention, its output (head -> token shard) after it.

Every rank runs the same FixedKVCache router (cache.py:31-133; deterministic
host bookkeeping), so the routing needs no communication. The exchange is a
callable (recv, send) with send / recv shaped [P, ...] (chunk j goes to /
comes from rank j); the default is torch.distributed.all_to_all_single (NCCL
over NVLink on GPUs). Results equal the unsharded LayerStack's: every kernel
computes a token row or an attention head independently of the others.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _lib
from .block import LayerStack, Workspace


def token_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first token, token count) of rank's shard of an n-token block."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if n % world:
        raise ValueError(f"{n} tokens do not split evenly over {world} ranks.")
    per = n // world
    return rank * per, per


def local_spatial_tables(cos: torch.Tensor, sin: torch.Tensor, span: int, start: int, count: int):
    """Spatial rotary rows of tokens [start, start + count) of a block whose
    token t sits at spatial position t % span (rope.py:57-82 tables [span, d]),
    as (cos, sin, count) for a kernel that indexes row % count."""
    rows = (torch.arange(start, start + count, device=cos.device) % span)
    return cos.index_select(0, rows).contiguous(), sin.index_select(0, rows).contiguous(), count


def pack_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, send: torch.Tensor) -> None:
    """q, k, v [n_local, heads*d] (row-strided views allowed) -> send
    [P, 3, n_local, E]: chunk j holds the E = heads/P*d columns of head group j."""
    world, _, n_loc, e = send.shape
    for i, x in enumerate((q, k, v)):
        if x.shape != (n_loc, world * e):
            raise ValueError(f"pack_heads: tensor {i} is {tuple(x.shape)}, expected {(n_loc, world * e)}")
        send[:, i].copy_(x.unflatten(1, (world, e)).transpose(0, 1))


def unpack_heads(recv: torch.Tensor, out: torch.Tensor) -> None:
    """recv [P, 3, n_local, E] (chunk j from rank j = tokens of shard j) ->
    out [3, P*n_local, E]: q, k, v of this rank's heads for every token in order."""
    world, three, n_loc, e = recv.shape
    out.view(three, world, n_loc, e).copy_(recv.transpose(0, 1))


def unpack_tokens(recv: torch.Tensor, out: torch.Tensor) -> None:
    """recv [P, n_local, E] (chunk j = head group j of this rank's tokens) ->
    out [n_local, P*E] in head order."""
    world, n_loc, e = recv.shape
    out.view(n_loc, world, e).copy_(recv.transpose(0, 1))


class AllToAll:
    """recv[j] <- rank j's send[me] over a torch.distributed group (NCCL on
    GPUs, gloo on CPU ranks)."""

    def __init__(self, group=None):
        self.group = group

    def __call__(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        import torch.distributed as dist
        dist.all_to_all_single(recv, send, group=self.group)


def local_exchange(recv: torch.Tensor, send: torch.Tensor) -> None:
    """The exchange of a group of one rank."""
    recv.copy_(send)


class ShardWorkspace:
    """Buffers of one rank for an n-token block: the token-shard workspace of
    FusedBlock (n/P rows), the exchange buffers and the head-shard attention."""

    def __init__(self, stack: "HeadShardedStack", n: int, frames: int):
        blk = stack.blocks[0]
        dev, dim, hd = stack.device, stack.dim, stack.head_dim
        world, hl = stack.world, stack.heads_local
        start, n_loc = token_shard(n, world, stack.rank)
        e = hl * hd
        self.n, self.n_loc, self.e = n, n_loc, e
        self.tok = Workspace(blk, n_loc, attention=False)
        bf = lambda *s: torch.empty(s, dtype=torch.bfloat16, device=dev)
        self.send, self.recv = bf(world, 3, n_loc, e), bf(world, 3, n_loc, e)
        self.qkv_h = bf(3, n, e)
        self.attn_h = bf(n, e)
        self.back = bf(world, n_loc, e)
        self.attn_tok = bf(n_loc, dim)
        ws = _lib.library().rc_paired_attention_workspace(1, frames, max(stack.max_cap, 1), blk.height,
                                                          blk.width, hl, hd)
        if ws < 0:
            raise ValueError(_lib.last_error())
        self.attn_ws = torch.empty((ws,), dtype=torch.uint8, device=dev)
        self.spatial = local_spatial_tables(blk.tables["spatial_cos"], blk.tables["spatial_sin"],
                                            stack.span, start, n_loc)


class HeadShardedStack(LayerStack):
    """The 30-layer loop of one stream split over `world` ranks (module
    docstring). step(hidden_local, frames) takes this rank's token shard of the
    block's hidden state [N/P, dim] and updates it in place; every rank calls
    it with the same frames, in the same order (the exchanges are collective)."""

    def __init__(self, blocks, actions, *, rank: int, world: int, exchange=None, **router):
        heads = blocks[0].heads
        if world <= 0 or heads % world:
            raise ValueError(f"{heads} heads do not split evenly over {world} ranks.")
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside a group of {world}")
        self.rank, self.world = rank, world
        self.heads_local = heads // world
        self.cache_heads = self.heads_local
        if exchange is None:
            exchange = AllToAll() if world > 1 else local_exchange
        self.exchange = exchange
        self._sws: dict[int, ShardWorkspace] = {}
        super().__init__(blocks, actions, **router)

    def shard_workspace(self, n: int, frames: int) -> ShardWorkspace:
        if n not in self._sws:
            self._sws[n] = ShardWorkspace(self, n, frames)
        return self._sws[n]

    def step(self, hidden: torch.Tensor, frames: int, *, graphs: bool = False) -> torch.Tensor:
        if graphs:
            raise ValueError("HeadShardedStack runs eagerly (graphs=False).")
        n = self.plan_block(hidden.shape[0], frames)
        self._layers(hidden, n, frames)
        return hidden

    def plan_block(self, n_local: int, frames: int) -> int:
        """Route the next block of `frames` latent frames (host router, one
        routing-table upload) and return its token count; step() calls it, a
        driver that runs the layer phases itself calls it once per block."""
        n = n_local * self.world
        if n != frames * self.span:
            raise ValueError("the shards must hold `frames` complete planes together.")
        self._plan(frames)
        self._upload_route()
        return n

    def step_host(self, *args, **kwargs):
        raise NotImplementedError("HeadShardedStack has no graph-replay host streaming path.")

    def capture(self, *args, **kwargs):
        raise NotImplementedError("HeadShardedStack runs eagerly.")

    # --------------------------------------------------------- per layer
    def _layers(self, h, n, frames):
        sw = self.shard_workspace(n, frames)
        for i in range(len(self.blocks)):
            self.layer_pre(i, h, sw)
            self.exchange(sw.recv, sw.send)
            self.layer_attend(i, sw, frames)
            self.exchange(sw.back, sw.attn_h.view(self.world, sw.n_loc, sw.e))
            self.layer_post(i, h, sw)

    def layer_pre(self, i: int, h: torch.Tensor, sw: ShardWorkspace) -> None:
        """Token shard: LN1 + AdaLN, QKV GEMM, RMSNorm + spatial RoPE; q/k/v packed
        by head group into sw.send."""
        blk, t = self.blocks[i], sw.tok
        lib, st = _lib.library(), _lib.stream(self.device)
        blk.pre_attention(lib, h, t, st, spatial=sw.spatial)
        pack_heads(t.q_rot, t.k_rot, t.qkv[:, 2 * self.dim:], sw.send)

    def layer_attend(self, i: int, sw: ShardWorkspace, frames: int) -> None:
        """Head shard: routed attention of this rank's heads over every token of
        the block (output sw.attn_h [N, E]), then the KV commit of those heads."""
        blk, c = self.blocks[i], self.caches[i]
        lib, st = _lib.library(), _lib.stream(self.device)
        unpack_heads(sw.recv, sw.qkv_h)
        q, k, v = sw.qkv_h[0], sw.qkv_h[1], sw.qkv_h[2]
        hd, e, hl = self.head_dim, sw.e, self.heads_local
        cap = c.capacity
        rd = self.route_dev
        o = i * self._row
        qpos = rd[len(self.blocks) * self._row:]
        pk, pv = self.cache_k[i], self.cache_v[i]
        kv_tok = pk.stride(1) if cap else 0
        strides = (C.c_longlong * 15)(0, e, hd, 0, e, hd, 0, e, hd, 0, kv_tok, hd, 0, kv_tok, hd)
        wh, ww = (blk.height, blk.width) if not blk.local else blk.window
        _lib.check(lib.rc_paired_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), pk.data_ptr() if cap else None,
            pv.data_ptr() if cap else None, strides, rd[o:].data_ptr() if cap else None,
            rd[o + 8:].data_ptr() if cap else None, qpos.data_ptr(),
            blk.tables["temporal_cos"].data_ptr(), blk.tables["temporal_sin"].data_ptr(),
            1, frames, cap, blk.height, blk.width, hl, hd, blk.tables["temporal_cos"].shape[1] * 2,
            wh, ww, sw.attn_ws.data_ptr(), sw.attn_ws.numel(), sw.attn_h.data_ptr(), e, None, None, st),
            "attention")
        if cap:
            row = e * 2
            _lib.check(lib.rc_kv_commit_planned(
                k.data_ptr(), v.data_ptr(), row, row, pk.data_ptr(), pv.data_ptr(), row, row,
                self.span, frames, cap, rd[o + 16:].data_ptr(), st), "kv_commit")

    def layer_post(self, i: int, h: torch.Tensor, sw: ShardWorkspace) -> None:
        """Token shard: the attention output of every head for this rank's tokens
        (sw.back, by head group) -> NVFP4 -> o-proj, cross attention, FFN."""
        blk, t = self.blocks[i], sw.tok
        lib, st = _lib.library(), _lib.stream(self.device)
        unpack_tokens(sw.back, sw.attn_tok)
        _lib.check(lib.rc_nvfp4_quantize(sw.attn_tok.data_ptr(), sw.n_loc, self.dim, self.dim, 1.0,
                                         t.a_codes.data_ptr(), t.a_scales.data_ptr(), st),
                   "nvfp4_quantize")
        blk.post_attention(lib, h, t, st)
