"""The cross-rank state exchange (atf_state_push / atf_state_merge) emulated on
one GPU: W ranks' exchange regions live in one process, wired with plain
pointers, and each step runs every rank's push, then every rank's merge (the
merges find the pushes already done, so nothing waits on a later launch).

The fused step (atf_decode_run_exchange: the decode's split merge, the push and
the exchange merge in one kernel) waits inside its kernel for the other ranks'
kernels, so several ranks of it cannot share one GPU: here it runs as a single
rank, which waits for no peer, and the emulated exchanges refuse it. Its
multi-rank form is checked on two GPUs (test_gpu_multi.py) and by bench.py's
KV-sharded decode parity at N > 1.

Each rank's merged output must equal lse_merge of the same W states bit for
bit (the NCCL all-gather path merges with the same kernel) and match the
one-GPU decode of the whole cache within tolerance, over several steps (the
buffer parity and the device step counter cycle). A rank whose peer never
pushes gives up after the wait limit and reports through the error flag."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _states(dev, world, seed, N=65536, hq=28, hkv=4, page=64):
    """A 1-request paged cache cut into `world` contiguous shards: every rank's
    fp32 (O, LSE) state for a fresh query, and the one-GPU decode."""
    import atflash
    g = torch.Generator(device=dev).manual_seed(seed)
    npg = N // page
    kc = torch.randn((npg, page, hkv, 128), generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn((npg, page, hkv, 128), generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((1, hq, 128), generator=g, device=dev).to(torch.bfloat16)
    wt = atflash.WindowTable(128, 1e7, 64.0)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
    w.plan(torch.tensor([0, npg], dtype=torch.int32), torch.arange(npg, dtype=torch.int32),
           torch.tensor([page], dtype=torch.int32), hq, hkv, 128, page, window_table=wt)
    full = w.run(q, (kc, vc), out_dtype=torch.float32)
    states = []
    for r in range(world):
        p0, p1 = r * npg // world, (r + 1) * npg // world
        wr = atflash.BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=dev), "NHD")
        wr.plan(torch.tensor([0, p1 - p0], dtype=torch.int32), torch.arange(p0, p1, dtype=torch.int32),
                torch.tensor([page], dtype=torch.int32), hq, hkv, 128, page, window_table=wt)
        o, l = wr.run(q, (kc, vc), q_pos=torch.tensor([N - 1]), kv_pos0=torch.tensor([p0 * page]),
                      return_lse=True, out_dtype=torch.float32)
        states.append((o, l))
    torch.cuda.synchronize()
    return states, full


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_emulated_equals_gather_merge(cuda_device, world):
    import atflash
    xs = atflash.dist.StateExchange.emulated(1, 28, world, device=cuda_device)
    for step in range(3):
        states, full = _states(cuda_device, world, seed=100 + step)
        ref_o, ref_l = atflash.lse_merge(torch.stack([o for o, _ in states]), torch.stack([l for _, l in states]),
                                         out_dtype=torch.float32, return_lse=True)
        for r, x in enumerate(xs):
            x.push(*states[r])
        outs = [x.merge(*states[r], out_dtype=torch.float32) for r, x in enumerate(xs)]
        torch.cuda.synchronize()
        assert atflash.check_device_errors() == 0
        for o, l in outs:
            assert torch.equal(o, ref_o) and torch.equal(l, ref_l), step
        assert (outs[0][0] - full).abs().max().item() < 4e-3


def test_exchange_reports_a_missing_peer(cuda_device):
    """Rank 0 of an emulated pair merges although rank 1 never pushed: the
    bounded wait gives up after its limit (about 2 s) and sets the error flag;
    the context stays usable."""
    import atflash
    xs = atflash.dist.StateExchange.emulated(1, 28, 2, device=cuda_device)
    states, _ = _states(cuda_device, 2, seed=7, N=8192)
    xs[0].push(*states[0])
    xs[0].merge(*states[0])
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 1
    x = torch.ones(4, device=cuda_device)
    assert float((x * 2).sum().item()) == 8.0


def test_fused_exchange_single_rank(cuda_device):
    """atf_decode_run_exchange with one rank, over several steps (the buffer
    parity and the step counter cycle), eagerly and replayed from a CUDA graph:
    bit-identical to the decode's own merge followed by atf_state_push and
    atf_state_merge, the separate-kernel path."""
    import atflash
    g = torch.Generator(device=cuda_device).manual_seed(5)
    N, hq, hkv, page = 16384, 28, 4, 64
    npg = N // page
    kc = torch.randn((npg, page, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    vc = torch.randn((npg, page, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=cuda_device),
                                                   "NHD")
    w.plan(torch.tensor([0, npg], dtype=torch.int32), torch.randperm(npg).to(torch.int32),
           torch.tensor([page], dtype=torch.int32), hq, hkv, 128, page,
           window_table=atflash.WindowTable(128, 1e7, 64.0))
    q_pos = torch.tensor([N - 1], dtype=torch.int64, device=cuda_device)
    kv_pos0 = torch.tensor([0], dtype=torch.int64, device=cuda_device)
    fused = atflash.dist.StateExchange(1, hq, device=cuda_device)
    separate = atflash.dist.StateExchange(1, hq, device=cuda_device)

    def reference(q):
        o, l = w.run(q, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0, return_lse=True, out_dtype=torch.float32)
        separate.push(o, l)
        return separate.merge(o, l, out_dtype=torch.float32)

    for step in range(3):
        q = torch.randn((1, hq, 128), generator=g, device=cuda_device).to(torch.bfloat16)
        ref_o, ref_l = reference(q)
        fo, fl = atflash.dist.sharded_decode(q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0,
                                             out_dtype=torch.float32, exchange=fused)
        torch.cuda.synchronize()
        assert torch.equal(fo, ref_o) and torch.equal(fl, ref_l), step
    gstep = atflash.dist.ShardedDecodeStep(q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0, out_dtype=torch.float32,
                                           exchange=fused)
    for step in range(3):
        gstep.q.copy_(torch.randn((1, hq, 128), generator=g, device=cuda_device).to(torch.bfloat16))
        og, lg = gstep()
        ref_o, ref_l = reference(gstep.q)
        torch.cuda.synchronize()
        assert torch.equal(og, ref_o) and torch.equal(lg, ref_l), step
    gstep.release()
    assert atflash.check_device_errors() == 0


def test_fused_exchange_refused_when_emulated(cuda_device):
    """Emulated ranks share one GPU: the fused step is refused on the host
    before anything is launched."""
    import atflash
    xs = atflash.dist.StateExchange.emulated(1, 28, 2, device=cuda_device)
    with pytest.raises(RuntimeError):
        xs[0]._fused_params(cuda_device)
