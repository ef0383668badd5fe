"""Host logic of the multi-GPU paths on CPU: zig-zag query partition, KV shard
ranges, and two gloo ranks (world size 2) running the sharded prefill (with the
oracle as the per-block compute) and the KV-sharded decode merge (all-gather of
partial (O, LSE) states + LSE merge) against single-process oracle results."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atflash import dist as AD


def test_zigzag_partition_covers_and_balances():
    for N in (4096, 131072, 524288, 1000, 128 * 37):
        for world in (1, 2, 4, 8):
            seen = np.zeros(N, dtype=np.int32)
            work = []
            for r in range(world):
                w = 0
                for (s, e) in AD.zigzag_blocks(N, world, r):
                    assert s % 128 == 0 and (e % 128 == 0 or e == N)
                    seen[s:e] += 1
                    w += AD.causal_pairs(s, e)
                work.append(w)
            assert (seen == 1).all()
            if N >= 128 * 16 * world and N % (256 * world) == 0:
                # zig-zag pairs give exactly equal causal work when blocks are equal
                assert max(work) - min(work) <= 0.02 * max(work), (N, world, work)


@pytest.mark.parametrize("N", [131072, 524288, 4096 + 384])
def test_windowed_zigzag_split_covers_and_is_not_less_even(N):
    """With a window table the blocks are cut by windowed work (the kernel's
    tile schedule); every row is covered once, every cut sits on the 128-row
    tile grid, and the largest rank's work is never above the equal-row split's."""
    from atflash import window_table as WT
    zhi = WT.WindowTable(128, 1e7, 2.0).zhi16
    cum = AD._cumulative_tile_work(N, zhi)
    for world in (2, 4, 8):
        seen = np.zeros(N, dtype=np.int32)
        for r in range(world):
            for (s, e) in AD.zigzag_blocks(N, world, r, zhi=zhi):
                assert s % 128 == 0 and (e % 128 == 0 or e == N)
                seen[s:e] += 1
        assert (seen == 1).all()
        bal = AD._max_pair_work(AD.zigzag_bounds(N, world, zhi=zhi), cum, world, 128)
        eq = AD._max_pair_work(AD.zigzag_bounds(N, world), cum, world, 128)
        assert bal <= eq
    if N == 524288:  # far from even with equal rows at 512K, close to even after the cut
        assert AD._max_pair_work(AD.zigzag_bounds(N, 8, zhi=zhi), cum, 8, 128) <= 1.003 * cum[-1] / 8


def test_kv_shard_ranges():
    for N in (1048576, 1000, 77):
        for world in (1, 2, 4, 8):
            rng = [AD.kv_shard_range(N, world, r, align=64) for r in range(world)]
            assert rng[0][0] == 0 and rng[-1][1] == N
            for a, b in zip(rng, rng[1:]):
                assert a[1] == b[0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_prefill(q, k, v, causal=True, softmax_scale=None, window_table=None, qk_layout="sorted_pair",
                    q_offset=0):
    from oracle import attention as OA
    from oracle import window_table as OWT
    w = OWT.wavelengths_sorted(128, window_table[0], window_table[1])
    o = OA.ref_window_attn(q.transpose(1, 2).float().numpy(), k.transpose(1, 2).float().numpy(),
                           v.transpose(1, 2).float().numpy(), w, phase="prefill", block_m=128, block_n=128,
                           q_offset=q_offset)
    return torch.from_numpy(o).transpose(1, 2).contiguous()


def _inputs(N=1024, hq=6, hkv=2):
    g = torch.Generator().manual_seed(4)
    q = torch.randn((1, N, hq, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, N, hkv, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, N, hkv, 128), generator=g).to(torch.bfloat16)
    return q, k, v


def _decode_partial(q, k, v, lo, hi, base, kr):
    """Oracle partial state of keys [lo, hi) at global positions; q at N-1."""
    from oracle import window_table as OWT
    N = k.shape[1]
    w = OWT.wavelengths_sorted(128, base, kr)
    zhi = OWT.zhi_table(w, 128, N)
    hq, hkv = q.shape[0], k.shape[0]
    G = hq // hkv
    o = np.zeros((hq, 128), dtype=np.float32)
    lse = np.full((hq,), -np.inf, dtype=np.float32)
    for h in range(hq):
        kk = k[h // G, lo:hi].astype(np.float32)
        vv = v[h // G, lo:hi].astype(np.float32)
        s = np.empty(hi - lo, dtype=np.float32)
        for n in range(lo, hi):
            z = (N - 1) - n
            deff = 16 * max(1, sum(1 for x in zhi if x >= z))
            s[n - lo] = q[h, :deff] @ kk[n - lo, :deff]
        s = s / np.sqrt(128.0)
        m = s.max()
        e = np.exp(s - m)
        o[h] = (e / e.sum()) @ vv
        lse[h] = m + np.log(e.sum())
    return o, lse


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__)))]
        q, k, v = _inputs()
        full = AD.sharded_prefill(q, k, v, rank=rank, world=world, window_table=(1e4, 2.0),
                                  prefill_fn=_oracle_prefill, gather=True)
        ref = _oracle_prefill(q, k, v, window_table=(1e4, 2.0))
        ok_prefill = torch.equal(full, ref)
        # KV-sharded decode: rank r holds keys of its shard, merged by LSE
        g = np.random.default_rng(1)
        N, hq, hkv = 700, 6, 2
        qd = g.standard_normal((hq, 128)).astype(np.float32)
        kd = g.standard_normal((hkv, N, 128)).astype(np.float32)
        vd = g.standard_normal((hkv, N, 128)).astype(np.float32)
        lo, hi = AD.kv_shard_range(N, world, rank)
        o, l = _decode_partial(qd, kd, vd, lo, hi, 1e4, 2.0)

        def merge_fn(po, pl):
            from oracle import attention as OA
            mo, ml = OA.merge_states(po.numpy(), pl.numpy())
            return torch.from_numpy(mo), torch.from_numpy(ml)
        mo, ml = AD.merge_partials(torch.from_numpy(o)[None], torch.from_numpy(l)[None], merge_fn=merge_fn)
        fo, fl = _decode_partial(qd, kd, vd, 0, N, 1e4, 2.0)
        ok_decode = float(np.abs(mo[0].numpy() - fo).max()) < 1e-5 and float(np.abs(ml[0].numpy() - fl).max()) < 1e-5
        results[rank] = (bool(ok_prefill), bool(ok_decode))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_sharded_prefill_and_decode_merge():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: (True, True), 1: (True, True)}


def _worker_lost_peer(rank, world, port, results):
    """Rank 1 leaves before the decode merge's all-gather; rank 0 must get an
    error from the collective within the process-group timeout, not hang."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results[rank] = "left"
        os._exit(0)  # leaves between steps, with no collective in flight
    o = torch.zeros((1, 4, 128))
    lse = torch.zeros((1, 4))
    t0 = time.time()
    try:
        AD.merge_partials(o, lse, merge_fn=lambda po, pl: (po[0], pl[0]))
        results[rank] = "no error"
    except Exception as e:  # gloo reports the lost peer or the timeout
        results[rank] = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"


def test_gloo_lost_rank_fails_the_collective_within_the_timeout():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_worker_lost_peer, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert results.get(1) == "left"
    msg = results.get(0, "hung")
    assert msg.startswith("error after"), msg
    assert float(msg.split()[2].rstrip("s:")) < 60, msg


class _FakeWrapper:
    """Records the keyword arguments of each run() call (host routing only)."""

    def __init__(self):
        self.calls = []

    def run(self, q, kv, **kw):
        self.calls.append(kw)
        B, H, D = q.shape
        out = torch.zeros((B, H, D), dtype=kw.get("out_dtype") or torch.bfloat16)
        lse = torch.zeros((B, H), dtype=torch.float32)
        if kw.get("out") is not None:
            return kw["out"], kw["lse"]
        return out, lse


class _FakeExchange:
    def __init__(self, emulated):
        self._emulated = emulated
        self.pushed = self.merged = 0

    def push(self, o, lse):
        self.pushed += 1

    def merge(self, o, lse, out_dtype=torch.bfloat16):
        self.merged += 1
        return o.to(out_dtype), lse


def test_sharded_decode_routes_exchange_and_programmatic_launch():
    """One rank, no process group: enable_pdl reaches the decode call; a real
    exchange runs as the decode's own fused step (exchange= passed to run), an
    emulated one as the decode followed by separate push and merge."""
    from atflash import dist as adist
    q = torch.zeros((1, 4, 128), dtype=torch.bfloat16)
    pos = torch.tensor([9], dtype=torch.int64)
    for pdl in (False, True):
        w = _FakeWrapper()
        adist.sharded_decode(q, w, (None, None), q_pos=pos, kv_pos0=pos, enable_pdl=pdl)
        assert w.calls[-1]["enable_pdl"] is pdl and "exchange" not in w.calls[-1]
        ex = _FakeExchange(emulated=False)
        adist.sharded_decode(q, w, (None, None), q_pos=pos, kv_pos0=pos, exchange=ex, enable_pdl=pdl)
        assert w.calls[-1]["exchange"] is ex and w.calls[-1]["enable_pdl"] is pdl
        assert ex.pushed == 0 and ex.merged == 0
        ex = _FakeExchange(emulated=True)
        adist.sharded_decode(q, w, (None, None), q_pos=pos, kv_pos0=pos, exchange=ex, enable_pdl=pdl)
        assert "exchange" not in w.calls[-1] and w.calls[-1]["out_dtype"] == torch.float32
        assert ex.pushed == 1 and ex.merged == 1
