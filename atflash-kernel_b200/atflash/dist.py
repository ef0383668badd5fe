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
import functools
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

TILE = 128


def zigzag_bounds(seqlen: int, world: int, align: int = TILE, zhi: Optional[Sequence[int]] = None) -> List[int]:
    """2*world+1 query block boundaries (see _zigzag_bounds); cached per shape."""
    return list(_zigzag_bounds(int(seqlen), int(world), int(align), None if zhi is None else tuple(int(x) for x in zhi)))


@functools.lru_cache(maxsize=64)
def _zigzag_bounds(seqlen: int, world: int, align: int, zhi: Optional[Tuple[int, ...]]) -> Tuple[int, ...]:
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
        return tuple(equal)
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
    return tuple(b if _max_pair_work(b, cum, world, align) < _max_pair_work(equal, cum, world, align) else equal)


def _max_pair_work(b, cum, world, align):
    t = [(x + align - 1) // align for x in b]
    return max((cum[t[r + 1]] - cum[t[r]]) + (cum[t[2 * world - r]] - cum[t[2 * world - 1 - r]])
               for r in range(world))


def _cumulative_tile_work(seqlen: int, zhi: Sequence[int], tile: int = TILE, head_dim: int = 128):
    """Windowed work of the rows [0, t * tile) for every t (causal prefill, one head).

    Query tile t meets key tiles n = 0..t; the pair's smallest distance
    z = max(0, (t - n - 1) * tile + 1) depends on d = t - n only, so the work of
    query tile t is the prefix sum over d <= t of 16 L(d) + head_dim."""
    levels = np.asarray(list(zhi), dtype=np.int64)
    nt = (seqlen + tile - 1) // tile
    d = np.arange(nt, dtype=np.int64)
    z = np.maximum(0, (d - 1) * tile + 1)
    L = np.maximum(1, (levels[None, :] >= z[:, None]).sum(axis=1))
    per_tile = np.cumsum((16 * L + head_dim).astype(np.float64))  # work of query tile t
    work = np.zeros(nt + 1, dtype=np.float64)
    work[1:] = np.cumsum(per_tile)
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
    gather=True the full (B, S, Hq, D) output assembled by an all-gather.

    Both blocks go out as one kernel launch over the full q/k/v (the kernel's
    row ranges), so they share one launch tail; the blocks are views of one
    (B, S, Hq, D) buffer whose other rows are left unwritten. A custom
    `prefill_fn` (a host-side model of the kernel, say) is called per block."""
    r0, w0 = _rank_world(group)
    rank = r0 if rank is None else rank
    world = w0 if world is None else world
    S = q.shape[1]
    if k.shape[1] != S:
        raise ValueError("sharded prefill expects seqlen_q == seqlen_k")
    zhi = getattr(window_table, "zhi16", None) if causal else None
    blocks = zigzag_blocks(S, world, rank, zhi=zhi)
    if prefill_fn is None:
        from .prefill import prefill_fwd
        live = [(s, e) for (s, e) in blocks if e > s]
        full = q.new_empty(q.shape)
        if live:
            prefill_fwd(q, k, v, causal=causal, softmax_scale=softmax_scale, window_table=window_table,
                        qk_layout=qk_layout, q_offset=0, out=full, row_ranges=live)
        outs = [(s, e, full[:, s:e]) for (s, e) in blocks]
        if not gather:
            return outs
        return gather_zigzag(outs, S, world, group, zhi=zhi)
    outs = []
    for (s, e) in blocks:
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
    `zhi` must be the window levels the blocks were cut with (None: equal rows).

    Every rank writes its blocks into its own slot of one padded receive buffer
    and the all-gather runs in place, so the only copies besides the gather are
    this rank's blocks going in and every block going to its rows in the output."""
    bounds = zigzag_bounds(seqlen, world, zhi=zhi)
    maxlen = max(bounds[i + 1] - bounds[i] for i in range(2 * world))
    ref = outs[0][2]
    B, _, H, D = ref.shape
    rank, _ = _rank_world(group)
    recv = ref.new_empty((world, 2, B, maxlen, H, D))
    for t, (s, e, o) in enumerate(outs):
        if e > s:
            recv[rank, t, :, : e - s].copy_(o)
    dist.all_gather_into_tensor(recv.view(-1), recv[rank].view(-1), group=group)
    full = ref.new_empty((B, seqlen, H, D))
    for r in range(world):
        for t, (s, e) in enumerate(zigzag_blocks(seqlen, world, r, zhi=zhi)):
            if e > s:
                full[:, s:e].copy_(recv[r, t, :, : e - s])
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


class StateExchange:
    """Cross-rank merge of partial attention states without a collective library
    (atf_state_push / atf_state_merge): every rank writes its (O, LSE) state into
    every peer's exchange region with NVLink peer stores and merges once every
    peer's push of the step has arrived. The result is bit-identical to
    all-gathering the states and merging them with lse_merge.

    The exchange region is one zeroed device buffer per rank, mapped into the
    peers' processes through CUDA IPC at construction (a collective setup step:
    every rank of `group` constructs its StateExchange together). The step
    counter lives on the device, so a step can be replayed from a CUDA graph.
    """

    def __init__(self, batch: int, num_heads: int, group=None, device=None, *, _emulate=None):
        import ctypes
        from . import _ffi
        self.B, self.H = int(batch), int(num_heads)
        self.rank, self.world = _rank_world(group) if _emulate is None else _emulate
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _ffi.load()
        nbytes = int(lib.atf_exchange_region_bytes(self.B, self.H, self.world))
        if nbytes <= 0:
            raise ValueError("unsupported exchange shape")
        self._region = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
        self.base = (self._region.data_ptr() + 255) // 256 * 256
        self._opened = []
        self.peer_base = None
        self._emulated = _emulate is not None
        if _emulate is not None:
            return  # peers are set by emulated()
        ptrs = [self.base]
        if self.world > 1:
            handle = (ctypes.c_char * _ffi.ATF_IPC_HANDLE_BYTES)()
            off = ctypes.c_int64(0)
            with torch.cuda.device(self.device):
                _ffi.check("atf_ipc_export", lib.atf_ipc_export(self.base, handle, ctypes.byref(off)))
            torch.cuda.synchronize(self.device)  # the zeroed region is in place before any peer maps it
            everyone = [None] * self.world
            dist.all_gather_object(everyone, (bytes(handle), int(off.value)), group=group)
            ptrs = []
            for q, (h, o) in enumerate(everyone):
                if q == self.rank:
                    ptrs.append(self.base)
                    continue
                ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _ffi.check("atf_ipc_import", lib.atf_ipc_import(h, o, ctypes.byref(ptr), ctypes.byref(base)))
                self._opened.append(base.value)
                ptrs.append(ptr.value)
            self.group = group
        self._set_peers(ptrs)

    def _set_peers(self, ptrs):
        self.peer_base = torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    @staticmethod
    def emulated(batch: int, num_heads: int, world: int, device=None) -> List["StateExchange"]:
        """`world` exchanges in one process on one GPU, wired with plain
        pointers (no IPC): the ranks' pushes, then their merges, in that order,
        reproduce a multi-GPU step on one device (tests)."""
        xs = [StateExchange(batch, num_heads, device=device, _emulate=(r, world)) for r in range(world)]
        for x in xs:
            x._set_peers([y.base for y in xs])
        return xs

    def _params(self, o, lse):
        from . import _ffi
        if o.dtype != torch.float32 or tuple(o.shape) != (self.B, self.H, 128) or o.stride(2) != 1:
            raise ValueError("the state must be fp32 (B, H, 128) with a contiguous head dim")
        if lse.dtype != torch.float32 or tuple(lse.shape) != (self.B, self.H) or not lse.is_contiguous():
            raise ValueError("the LSE must be a contiguous fp32 (B, H) tensor")
        from . import _runtime
        p = _ffi.AtfExchangeParams()
        p.o, p.lse = o.data_ptr(), lse.data_ptr()
        p.o_stride_b, p.o_stride_h = o.stride(0), o.stride(1)
        p.batch, p.num_heads, p.world, p.rank = self.B, self.H, self.world, self.rank
        p.peer_base, p.base = self.peer_base.data_ptr(), self.base
        p.error_flag = _runtime.error_flag(self.device).data_ptr()
        return p

    def _fused_params(self, device):
        """The exchange fields atf_decode_run_exchange reads. Emulated ranks share
        one GPU, and a fused step waits inside its kernel for the other ranks'
        kernels, which on one GPU need not run at the same time: refused."""
        from . import _ffi, _runtime
        if self._emulated:
            raise RuntimeError("an emulated exchange runs push() and merge() as separate steps; the fused "
                               "decode step needs every rank on its own GPU")
        if torch.device(device) != self.device:
            raise ValueError("the decode runs on another device than the exchange region")
        p = _ffi.AtfExchangeParams()
        p.batch, p.num_heads, p.world, p.rank = self.B, self.H, self.world, self.rank
        p.peer_base, p.base = self.peer_base.data_ptr(), self.base
        p.error_flag = _runtime.error_flag(self.device).data_ptr()
        return p

    def push(self, o: torch.Tensor, lse: torch.Tensor) -> None:
        """Send this rank's state (O fp32 (B, H, 128), LSE natural log (B, H))."""
        import ctypes
        from . import _ffi, _runtime
        p = self._params(o, lse)
        with torch.cuda.device(self.device):
            _ffi.check("atf_state_push", _ffi.load().atf_state_push(ctypes.byref(p), _runtime.stream_handle(self.device)))

    def merge(self, o: torch.Tensor, lse: torch.Tensor, out=None, lse_out=None, out_dtype=torch.bfloat16):
        """Merge every rank's state of this step into `out` (B, H, 128) and the
        natural-log `lse_out` (B, H); o / lse are this rank's pushed state."""
        import ctypes
        from . import _ffi, _runtime
        p = self._params(o, lse)
        if out is None:
            out = torch.empty((self.B, self.H, 128), dtype=out_dtype, device=self.device)
        if lse_out is None:
            lse_out = torch.empty((self.B, self.H), dtype=torch.float32, device=self.device)
        p.out, p.out_stride_b, p.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
        p.out_dtype = _ffi.ATF_DTYPE_F32 if out.dtype == torch.float32 else _ffi.ATF_DTYPE_BF16
        p.lse_out = lse_out.data_ptr()
        with torch.cuda.device(self.device):
            _ffi.check("atf_state_merge",
                       _ffi.load().atf_state_merge(ctypes.byref(p), _runtime.stream_handle(self.device)))
        return out, lse_out

    def close(self) -> None:
        """Unmap the peers' regions (after every rank has finished its last step)."""
        from . import _ffi
        lib = _ffi.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for b in self._opened:
                lib.atf_ipc_release(b)
        self._opened = []


def sharded_decode(q: torch.Tensor, wrapper, paged_kv_cache, *, q_pos: torch.Tensor,
                   kv_pos0: torch.Tensor, group=None, out_dtype=torch.bfloat16,
                   exchange: Optional[StateExchange] = None, enable_pdl: bool = False):
    """Decode with this rank's KV shard; `wrapper` is planned over the rank's local
    pages. q_pos: global query position per request; kv_pos0: global position of
    this rank's first key per request. Returns (out, lse) merged over the group:
    through `exchange` (peer stores, no collective) when given, else with one
    all-gather of the ranks' states. enable_pdl: the decode's launch as in
    BatchDecodeWithPagedKVCacheWrapper.run."""
    _, world = _rank_world(group)
    if exchange is not None:
        if not exchange._emulated:
            # one kernel after the decode merges, exchanges and merges again
            return wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                               enable_pdl=enable_pdl, return_lse=True,
                               out_dtype=out_dtype, exchange=exchange)
        B, H, D = q.shape
        o = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
        lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
        wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                    enable_pdl=enable_pdl, out=o, lse=lse, return_lse=True,
                    out_dtype=torch.float32)
        exchange.push(o, lse)
        return exchange.merge(o, lse, out_dtype=out_dtype)
    if world == 1:
        # one shard: the decode's own split merge is already the result
        return wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0, enable_pdl=enable_pdl, return_lse=True,
                           out_dtype=out_dtype)
    # the local state goes straight into the buffer that is all-gathered
    B, H, D = q.shape
    pack, o_view, l_view = _pack_views(B, H, D, q.device)
    wrapper.run(q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                enable_pdl=enable_pdl, out=o_view, lse=l_view, return_lse=True,
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
    the same inputs bit for bit. With a StateExchange the whole step (decode,
    push, merge) is one graph and no collective runs at all.
    """

    def __init__(self, q: torch.Tensor, wrapper, paged_kv_cache, *, q_pos: torch.Tensor,
                 kv_pos0: torch.Tensor, group=None, out_dtype=torch.bfloat16,
                 exchange: Optional["StateExchange"] = None, enable_pdl: bool = False):
        if not (q_pos.is_cuda and kv_pos0.is_cuda):
            raise ValueError("q_pos and kv_pos0 must be CUDA tensors (they are read by the replayed graph)")
        _, self.world = _rank_world(group)
        self.group = group
        self.q = q.clone()
        self.q_pos, self.kv_pos0 = q_pos, kv_pos0
        B, H, D = q.shape
        self.B, self.H, self.D = B, H, D
        self.exchange = exchange
        self.pack, self.o_view, self.l_view = _pack_views(B, H, D, q.device)
        n = self.pack.numel()
        self.allp = self.pack.new_empty((self.world * n,))
        from .decode import lse_merge

        def local():
            if exchange is not None and not exchange._emulated:
                # the whole step in one graph: the decode and one kernel that
                # merges its split, exchanges with the peers and merges again
                return wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                                   enable_pdl=enable_pdl, return_lse=True,
                                   out_dtype=out_dtype, exchange=exchange)
            if exchange is not None:
                # the whole step (decode, push to the peers, merge) in one graph:
                # no collective library call, the step counter is on the device
                wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                            enable_pdl=enable_pdl, out=self.o_view, lse=self.l_view,
                            return_lse=True, out_dtype=torch.float32)
                exchange.push(self.o_view, self.l_view)
                return exchange.merge(self.o_view, self.l_view, out_dtype=out_dtype)
            if self.world == 1:
                return wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                                   enable_pdl=enable_pdl, return_lse=True,
                                   out_dtype=out_dtype)
            wrapper.run(self.q, paged_kv_cache, q_pos=q_pos, kv_pos0=kv_pos0,
                        enable_pdl=enable_pdl, out=self.o_view, lse=self.l_view,
                        return_lse=True, out_dtype=torch.float32)
            return None

        def merge():
            po = self.allp.as_strided((self.world, B, H, D), (n, H * D, D, 1))
            pl = self.allp.as_strided((self.world, B, H), (n, H, 1), B * H * D)
            return lse_merge(po, pl, lse_log2=False, out_dtype=out_dtype, return_lse=True)

        # one eager step first (library load, lazy allocations), then the captures
        local()
        if self.world > 1 and exchange is None:
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
            if self.world > 1 and exchange is None:
                self.g_merge = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.g_merge):
                    res = merge()
        torch.cuda.current_stream().wait_stream(side)
        self.out, self.lse = res

    def __call__(self):
        self.g_local.replay()
        if self.world > 1 and self.exchange is None:
            dist.all_gather_into_tensor(self.allp, self.pack, group=self.group)
            self.g_merge.replay()
        return self.out, self.lse

    def release(self):
        """Free the graphs (before the process group is destroyed)."""
        self.g_local = None
        self.g_merge = None

