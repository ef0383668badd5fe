"""Two-GPU runs of the sharded paths over NCCL (skipped with fewer than two GPUs).

Zig-zag prefill: each rank computes its two query blocks against replicated
K/V; the gathered rows must equal a one-GPU run bit for bit. KV-sharded decode:
each rank decodes its contiguous shard of every request with global positions,
the partial (O, LSE) are all-gathered and merged; the result must match the
one-GPU decode of the whole cache (same kernels, different split points, so a
tolerance rather than bit equality). The NVLink state exchange (peer stores, no
collective) must equal the all-gather path bit for bit, eagerly and replayed
from a CUDA graph, both as the fused step (atf_decode_run_exchange) and as the
decode's merge followed by separate push and merge kernels."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq):
    import datetime
    import sys
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "atflash-kernel_b200")]
    try:
        import atflash
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        g = torch.Generator(device="cpu").manual_seed(31)
        # --- zig-zag prefill
        N, hq, hkv = 1536, 6, 2
        q = torch.randn((1, N, hq, 128), generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn((1, N, hkv, 128), generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn((1, N, hkv, 128), generator=g).to(torch.bfloat16).to(dev)
        wt = atflash.WindowTable(128, 1e4, 2.0)
        full = atflash.dist.sharded_prefill(q, k, v, window_table=wt, gather=True)
        single = atflash.prefill_fwd(q, k, v, causal=True, window_table=wt)
        torch.cuda.synchronize()
        assert torch.equal(full, single), "zig-zag rows differ from the one-GPU run"
        # --- KV-sharded decode: 3 requests, page 16, every rank holds a contiguous key range
        lens = [4096, 2048, 1040]
        page, hq, hkv = 16, 24, 8
        qd = torch.randn((len(lens), hq, 128), generator=g).to(torch.bfloat16).to(dev)
        ks = [torch.randn((n, hkv, 128), generator=g).to(torch.bfloat16) for n in lens]
        vs = [torch.randn((n, hkv, 128), generator=g).to(torch.bfloat16) for n in lens]

        def paged(kl, vl):
            pages, indptr, lpl, kp, vp = [], [0], [], [], []
            for kk, vv in zip(kl, vl):
                n = kk.shape[0]
                npg = (n + page - 1) // page
                pad = npg * page - n
                kk = torch.cat([kk, kk.new_zeros((pad, hkv, 128))]).view(npg, page, hkv, 128)
                vv = torch.cat([vv, vv.new_zeros((pad, hkv, 128))]).view(npg, page, hkv, 128)
                kp.append(kk)
                vp.append(vv)
                indptr.append(indptr[-1] + npg)
                lpl.append(n - (npg - 1) * page)
            kc = torch.cat(kp).to(dev)
            vc = torch.cat(vp).to(dev)
            idx = torch.arange(indptr[-1], dtype=torch.int32)
            return kc, vc, torch.tensor(indptr, dtype=torch.int32), idx, torch.tensor(lpl, dtype=torch.int32)

        ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
        kc, vc, indptr, idx, lpl = paged(ks, vs)
        w1 = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w1.plan(indptr, idx, lpl, hq, hkv, 128, page, window_table=wt)
        ref = w1.run(qd, (kc, vc), out_dtype=torch.float32)
        # this rank's contiguous shard of every request, cut at page boundaries
        kl, vl, pos0 = [], [], []
        for kk, vv, n in zip(ks, vs, lens):
            npg = (n + page - 1) // page
            cut = [min(n, ((npg * r) // world) * page) for r in range(world + 1)]
            kl.append(kk[cut[rank]:cut[rank + 1]])
            vl.append(vv[cut[rank]:cut[rank + 1]])
            pos0.append(cut[rank])
        assert all(x.shape[0] > 0 for x in kl)
        kc2, vc2, indptr2, idx2, lpl2 = paged(kl, vl)
        ws2 = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
        w2 = atflash.BatchDecodeWithPagedKVCacheWrapper(ws2, "NHD")
        w2.plan(indptr2, idx2, lpl2, hq, hkv, 128, page, window_table=wt)
        q_pos = torch.tensor([n - 1 for n in lens], dtype=torch.int64, device=dev)
        kv_pos0 = torch.tensor(pos0, dtype=torch.int64, device=dev)
        out, lse = atflash.dist.sharded_decode(qd, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                               out_dtype=torch.float32)
        torch.cuda.synchronize()
        err = (out - ref).abs().max().item()
        assert err < 2e-3, f"sharded decode differs from the one-GPU decode by {err}"
        # the same step replayed from CUDA graphs (the all-gather stays eager)
        step = atflash.dist.ShardedDecodeStep(qd, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                              out_dtype=torch.float32)
        for _ in range(2):
            o_g, l_g = step()
        torch.cuda.synchronize()
        assert torch.equal(o_g, out) and torch.equal(l_g, lse), "graph step differs from sharded_decode"
        step.q.copy_(torch.randn(qd.shape, generator=g).to(torch.bfloat16).to(dev))
        o_g, l_g = step()
        out2, lse2 = atflash.dist.sharded_decode(step.q, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                                 out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(o_g, out2) and torch.equal(l_g, lse2), "graph step on a new query differs"
        step.release()
        # the same step through the NVLink state exchange (peer stores, no
        # collective): bit-identical to the all-gather path, over several steps
        # and from a CUDA graph
        ex = atflash.dist.StateExchange(len(lens), hq)
        for _ in range(3):
            ox, lx = atflash.dist.sharded_decode(step.q, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                                 out_dtype=torch.float32, exchange=ex)
            torch.cuda.synchronize()
            assert torch.equal(ox, out2) and torch.equal(lx, lse2), "exchange differs from the all-gather path"
        gstep = atflash.dist.ShardedDecodeStep(step.q, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                               out_dtype=torch.float32, exchange=ex)
        for _ in range(3):
            og, lg = gstep()
        torch.cuda.synchronize()
        assert torch.equal(og, out2) and torch.equal(lg, lse2), "graph-replayed exchange step differs"
        gstep.release()
        # each decode launched as a programmatic dependent of the previous exchange kernel
        pstep = atflash.dist.ShardedDecodeStep(step.q, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                               out_dtype=torch.float32, exchange=ex, enable_pdl=True)
        for _ in range(3):
            op, lp = pstep()
        torch.cuda.synchronize()
        assert torch.equal(op, out2) and torch.equal(lp, lse2), "programmatic-launch exchange step differs"
        pstep.release()
        # the separate-kernel path on the same exchange (decode merge, push,
        # merge): the same bits, and the step protocol carries on between the two
        for _ in range(2):
            o_s, l_s = w2.run(step.q, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0, return_lse=True,
                              out_dtype=torch.float32)
            ex.push(o_s, l_s)
            os_, ls_ = ex.merge(o_s, l_s, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(os_, out2) and torch.equal(ls_, lse2), "push / merge kernels differ"
            ox, lx = atflash.dist.sharded_decode(step.q, w2, (kc2, vc2), q_pos=q_pos, kv_pos0=kv_pos0,
                                                 out_dtype=torch.float32, exchange=ex)
            torch.cuda.synchronize()
            assert torch.equal(ox, out2) and torch.equal(lx, lse2), "fused step after push / merge differs"
        assert atflash.check_device_errors() == 0
        dist.barrier()
        ex.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_two_gpu_zigzag_prefill_and_sharded_decode():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not msgs, "; ".join(msgs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
