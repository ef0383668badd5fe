"""The paged decode replays from a CUDA graph: with a fixed plan and fixed
input/output buffers, run() captured once and replayed on new queries gives
the same outputs as eager runs (FlashInfer's use_cuda_graph contract)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_decode_run_replays_from_a_cuda_graph():
    import atflash
    from test_gpu_decode import make_paged
    dev = torch.device("cuda:0")
    lens, hq, hkv, page = [3000, 517, 1200], 24, 8, 16
    q, kc, vc, indptr, indices, lpl, _, _ = make_paged(lens, hq, hkv, page, 21)
    kc, vc = kc.to(dev), vc.to(dev)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD", use_cuda_graph=True)
    assert w.is_cuda_graph_enabled
    w.plan(indptr, indices, lpl, hq, hkv, 128, page, window_table=atflash.WindowTable(128, 1e4, 2.0))
    q_buf = q.to(dev).clone()
    out_buf = torch.empty((len(lens), hq, 128), dtype=torch.bfloat16, device=dev)
    w.run(q_buf, (kc, vc), out=out_buf)  # warm-up outside the capture (library load, attributes)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            w.run(q_buf, (kc, vc), out=out_buf)
    torch.cuda.current_stream().wait_stream(s)
    gen = torch.Generator(device=dev).manual_seed(5)
    for _ in range(3):
        qn = torch.randn(q_buf.shape, generator=gen, device=dev).to(torch.bfloat16)
        q_buf.copy_(qn)
        g.replay()
        torch.cuda.synchronize()
        ref = w.run(qn, (kc, vc))
        torch.cuda.synchronize()
        assert torch.equal(out_buf, ref)
    assert atflash.check_device_errors() == 0
    del g


def test_sharded_decode_step_one_rank_replays():
    """ShardedDecodeStep on one rank (no process group): the replayed decode equals
    sharded_decode bit for bit, also after the query buffer is rewritten."""
    import atflash
    from test_gpu_decode import make_paged
    dev = torch.device("cuda:0")
    lens, hq, hkv, page = [5000], 28, 4, 64
    q, kc, vc, indptr, indices, lpl, _, _ = make_paged(lens, hq, hkv, page, 22)
    kc, vc = kc.to(dev), vc.to(dev)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
    w.plan(indptr, indices, lpl, hq, hkv, 128, page, window_table=atflash.WindowTable(128, 1e7, 64.0))
    q_pos = torch.tensor([lens[0] - 1], dtype=torch.int64, device=dev)
    kv_pos0 = torch.zeros(1, dtype=torch.int64, device=dev)
    q = q.to(dev)
    step = atflash.dist.ShardedDecodeStep(q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0)
    gen = torch.Generator(device=dev).manual_seed(6)
    for _ in range(3):
        out, lse = step()
        ref, ref_lse = atflash.dist.sharded_decode(step.q, w, (kc, vc), q_pos=q_pos, kv_pos0=kv_pos0)
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
        step.q.copy_(torch.randn(q.shape, generator=gen, device=dev).to(torch.bfloat16))
    step.release()
    assert atflash.check_device_errors() == 0

