"""Multi-GPU windowed attention: one process per GPU over torch.distributed.

Prefill shards the *queries*: the sequence is cut into 2G blocks (G ranks) and
rank i computes blocks i and 2G-1-i (zig-zag causal balance) against
replicated K/V. Each block is a bottom-right-aligned chunk (q_offset = block
start), so windows use global positions and, with block starts on the 128-row
tile grid, every output row is bit-identical to the single-GPU run. There is no
collective on this path (an optional all-gather of the output is separate).

Decode shards the *KV sequence*: rank r holds keys [start_r, end_r) of every
request in its own paged cache, runs the split-KV decode with global key
positions (kv_pos0 = start_r) and the global query position, and returns a
partial (O, LSE). One all-gather of (O fp32, LSE) over the group and an LSE merge
give the result.

The reference has no multi-GPU code (it is batch-1, single GPU); this module is
the build's sharding of the same computation.
"""
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

TILE = 128


def zigzag_bounds(seqlen: int, world: int, align: int = TILE, zhi: Optional[Sequence[int]] = None) -> List[int]:
    """2*world+1 block boundaries, interior ones on multiples of `align`.

    Without a window table the blocks have equal rows: under a causal mask the
    work of a block grows linearly with its position, so blocks i and
    2*world-1-i always add up to the same work. With a window (`zhi`, the
    16-snap levels) a far key tile costs less than a near one and the work of a
    row grows more slowly than its length, so equal rows would leave the ranks
    holding the first blocks with the most work. Then the first half of the
    sequence keeps equal-row blocks and the second half is cut so that every
    rank's pair of blocks carries the same work, in the windowed FLOP model of
    the kernel: a (query tile, key tile) step costs D_eff + head_dim."""
    nb = 2 * world
    equal = [0]
    for i in range(1, nb):
        x = int(round(i * seqlen / nb / align)) * align
        equal.append(min(max(x, equal[-1]), seqlen))
    equal.append(seqlen)
    if zhi is None or world == 1:
        return equal
    cum = _cumulative_tile_work(seqlen, zhi, align)  # cum[t]: work of rows [0, t * align)
    nt = len(cum) - 1
    half = int(round(nt / 2))
    b = [0] + [int(round(i * half / world)) for i in range(1, world)] + [half]
    target = cum[nt] / world
    tail = [nt]
    for r in range(world - 1):  # rank r's far block ends where rank r-1's starts
        want = target - (cum[b[r + 1]] - cum[b[r]])
        lo_val = cum[tail[-1]] - want
        t = int(np.searchsorted(cum, lo_val))
        if t > 0 and abs(cum[t - 1] - lo_val) < abs(cum[t] - lo_val):
            t -= 1
        tail.append(min(max(t, half), tail[-1]))
    tail.append(half)
    b = [min(x * align, seqlen) for x in b[:-1] + tail[::-1]]
    # the cuts sit on whole tiles, so keep whichever split is closer to even
    return b if _max_pair_work(b, cum, world, align) < _max_pair_work(equal, cum, world, align) else equal


def _max_pair_work(b, cum, world, align):
    t = [(x + align - 1) // align for x in b]
    return max((cum[t[r + 1]] - cum[t[r]]) + (cum[t[2 * world - r]] - cum[t[2 * world - 1 - r]])
               for r in range(world))


def _cumulative_tile_work(seqlen: int, zhi: Sequence[int], tile: int = TILE, head_dim: int = 128):
    """Windowed work of the rows [0, t * tile) for every t (causal prefill, one head)."""
    levels = np.asarray(list(zhi), dtype=np.int64)
    nt = (seqlen + tile - 1) // tile
    work = np.zeros(nt + 1, dtype=np.float64)
    n0 = np.arange(nt, dtype=np.int64) * tile
    for t in range(nt):
        q0 = t * tile
        z = np.maximum(0, q0 - (n0[:t + 1] + tile - 1))
        L = np.maximum(1, (levels[None, :] >= z[:, None]).sum(axis=1))
        work[t + 1] = work[t] + float((16 * L + head_dim).sum())
    return work


def zigzag_blocks(seqlen: int, world: int, rank: int, align: int = TILE,
                  zhi: Optional[Sequence[int]] = None) -> List[Tuple[int, int]]:
    """The two [start, end) query blocks of `rank`: blocks rank and 2*world-1-rank
    (of zigzag_bounds, balanced for the window when `zhi` is given)."""
    b = zigzag_bounds(seqlen, world, align, zhi)
    i, j = rank, 2 * world - 1 - rank
    return [(b[i], b[i + 1]), (b[j], b[j + 1])]


def causal_pairs(s: int, e: int) -> int:
    """Query-key pairs of rows [s, e) under a causal mask (work of one block)."""
    return (e * (e + 1) - s * (s + 1)) // 2


def kv_shard_range(seqlen: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Contiguous key range of `rank` when the KV sequence is split evenly."""
    per = -(-seqlen // world)
    per = -(-per // align) * align
    return min(seqlen, rank * per), min(seqlen, (rank + 1) * per)


def _rank_world(group) -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def sharded_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, group=None,
                    rank: Optional[int] = None, world: Optional[int] = None,
                    window_table=None, causal: bool = True, softmax_scale=None,
                    qk_layout: str = "sorted_pair", gather: bool = False,
                    prefill_fn: Optional[Callable] = None):
    """This rank's zig-zag share of a causal prefill over the full q/k/v.

    Returns [(start, end, out_block)] for the rank's two blocks, or with
    gather=True the full (B, S, Hq, D) output assembled by an all-gather."""
    if prefill_fn is None:
        from .prefill import prefill_fwd as prefill_fn
    r0, w0 = _rank_world(group)
    rank = r0 if rank is None else rank
    world = w0 if world is None else world
    S = q.shape[1]
    if k.shape[1] != S:
        raise ValueError("sharded prefill expects seqlen_q == seqlen_k")
    zhi = getattr(window_table, "zhi16", None) if causal else None
    outs = []
    for (s, e) in zigzag_blocks(S, world, rank, zhi=zhi):
        if e <= s:
            outs.append((s, e, q.new_empty((q.shape[0], 0, q.shape[2], q.shape[3]))))
            continue
        o = prefill_fn(q[:, s:e], k[:, :e] if causal else k, v[:, :e] if causal else v,
                       causal=causal, softmax_scale=softmax_scale, window_table=window_table,
                       qk_layout=qk_layout, q_offset=s if causal else 0)
        outs.append((s, e, o))
    if not gather:
        return outs
    return gather_zigzag(outs, S, world, group, zhi=zhi)


def gather_zigzag(outs, seqlen: int, world: int, group=None, zhi: Optional[Sequence[int]] = None) -> torch.Tensor:
    """All-gather every rank's two blocks into the full output (rows in order).
    `zhi` must be the window levels the blocks were cut with (None: equal rows)."""
    bounds = zigzag_bounds(seqlen, world, zhi=zhi)
    maxlen = max(bounds[i + 1] - bounds[i] for i in range(2 * world))
    ref = outs[0][2]
    B, _, H, D = ref.shape
    send = ref.new_zeros((2, B, maxlen, H, D))
    for t, (s, e, o) in enumerate(outs):
        send[t, :, : e - s] = o
    recv = ref.new_empty((world, 2, B, maxlen, H, D))
    dist.all_gather_into_tensor(recv.view(-1), send.view(-1), group=group)
    full = ref.new_empty((B, seqlen, H, D))
    for r in range(world):
        for t, (s, e) in enumerate(zigzag_blocks(seqlen, world, r, zhi=zhi)):
            full[:, s:e] = recv[r, t, :, : e - s]
    return full


def _gather_and_merge(pack, B, H, D, group, world, merge_fn, out_dtype):
    """All-gather one flat fp32 buffer per rank ([B*H*D] O, then [B*H] LSE, padded to
    a multiple of 4 floats) and merge the ranks' states in place."""
    n = pack.numel()
    allp = pack.new_empty((world * n,))
    dist.all_gather_into_tensor(allp, pack, group=group)
    po = allp.as_strided((world, B, H, D), (n, H * D, D, 1))
    pl = allp.as_strided((world, B, H), (n, H, 1), B * H * D)
    if merge_fn is None:
        from .decode import lse_merge
        return lse_merge(po, pl, lse_log2=False, out_dtype=out_dtype, return_lse=True)
    return merge_fn(po, pl)


def _pack_views(B, H, D, device):
    n_o, n_l = B * H * D, (B * H + 3) // 4 * 4
    pack = torch.empty((n_o + n_l,), dtype=torch.float32, device=device)
    return pack, pack[:n_o].view(B, H, D), pack[n_o:n_o + B * H].view(B, H)


def merge_partials(o_local: torch.Tensor, lse_local: torch.Tensor, group=None,
                   merge_fn: Optional[Callable] = None, out_dtype=torch.bfloat16):
    """All-gather per-rank partial states (O fp32 (B,H,D), LSE natural (B,H)) and
    merge them: LSE = log sum exp LSE_r, O = sum exp(LSE_r - LSE) O_r."""
    _, world = _rank_world(group)
    B, H, D = o_local.shape
    if world == 1:
        po, pl = o_local.float()[None], lse_local.float()[None]
        if merge_fn is None:
            from .decode import lse_merge
            return lse_merge(po, pl, lse_log2=False, out_dtype=out_dtype, return_lse=True)
        return merge_fn(po, pl)
    pack, o_view, l_view = _pack_views(B, H, D, o_local.device)
    o_view.copy_(o_local)
    l_view.copy_(lse_local)
    return _gather_and_merge(pack, B, H, D, group, world, merge_fn, out_dtype)


def sharded_decode(q: torch.Tensor, wrapper, paged_kv_cache, *, q_pos: torch.Tensor,
                   kv_pos0: torch.Tensor, group=None, out_dtype=torch.bfloat16):
    """Decode with this rank's KV shard; `wrapper` is planned over the rank's local
    pages. q_pos: global query position per request; kv_pos0: global position of
    this rank's first key per request. Returns (out, lse) merged over the group."""
    _, world = _rank_world(group)
    if world == 1:
        # one shard: the decode's own split merge is already the result
        return wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0, return_lse=True,
                           out_dtype=out_dtype)
    # the local state goes straight into the buffer that is all-gathered
    B, H, D = q.shape
    pack, o_view, l_view = _pack_views(B, H, D, q.device)
    wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0, out=o_view, lse=l_view, return_lse=True,
                out_dtype=torch.float32)
    return _gather_and_merge(pack, B, H, D, group, world, None, out_dtype)


class ShardedDecodeStep:
    """A KV-sharded decode step with fixed buffers, replayed from CUDA graphs.

    This rank's split-KV decode (and its own merge) is captured as one graph and
    the cross-rank LSE merge as another. The NCCL all-gather between them runs
    eagerly on the same stream, so no collective is captured in a graph. The
    caller writes each step's query into ``self.q`` (a copy of `q`, made at
    construction); `q_pos` / `kv_pos0` must be device tensors and may also be
    updated in place. Calling the object runs one step and returns (out, lse),
    tensors that later steps overwrite. The result equals ``sharded_decode`` on
    the same inputs bit for bit.
    """

    def __init__(self, q: torch.Tensor, wrapper, paged_kv_cache, *, q_pos: torch.Tensor,
                 kv_pos0: torch.Tensor, group=None, out_dtype=torch.bfloat16):
        if not (q_pos.is_cuda and kv_pos0.is_cuda):
            raise ValueError("q_pos and kv_pos0 must be CUDA tensors (they are read by the replayed graph)")
        _, self.world = _rank_world(group)
        self.group = group
        self.q = q.clone()
        self.q_pos, self.kv_pos0 = q_pos, kv_pos0
        B, H, D = q.shape
        self.B, self.H, self.D = B, H, D
        self.pack, self.o_view, self.l_view = _pack_views(B, H, D, q.device)
        n = self.pack.numel()
        self.allp = self.pack.new_empty((self.world * n,))
        from .decode import lse_merge

        def local():
            if self.world == 1:
                return wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0, return_lse=True,
                                   out_dtype=out_dtype)
            wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0, out=self.o_view, lse=self.l_view,
                        return_lse=True, out_dtype=torch.float32)
            return None

        def merge():
            po = self.allp.as_strided((self.world, B, H, D), (n, H * D, D, 1))
            pl = self.allp.as_strided((self.world, B, H), (n, H, 1), B * H * D)
            return lse_merge(po, pl, lse_log2=False, out_dtype=out_dtype, return_lse=True)

        # one eager step first (library load, lazy allocations), then the captures
        local()
        if self.world > 1:
            dist.all_gather_into_tensor(self.allp, self.pack, group=group)
            merge()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(q.device)
        side.wait_stream(torch.cuda.current_stream())
        self.g_local = torch.cuda.CUDAGraph()
        self.g_merge = None
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.g_local):
                res = local()
            if self.world > 1:
                self.g_merge = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.g_merge):
                    res = merge()
        torch.cuda.current_stream().wait_stream(side)
        self.out, self.lse = res

    def __call__(self):
        self.g_local.replay()
        if self.world > 1:
            dist.all_gather_into_tensor(self.allp, self.pack, group=self.group)
            self.g_merge.replay()
        return self.out, self.lse

    def release(self):
        """Free the graphs (before the process group is destroyed)."""
        self.g_local = None
        self.g_merge = None

