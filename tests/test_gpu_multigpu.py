"""Multi-GPU decode (fable_attn.multigpu.decode_kv_split) on 2 GPUs over NCCL: each rank holds
its contiguous chunk of every sequence's context and decodes against it; the all-gathered
partials merged by flash_attn_combine equal single-GPU decode over the whole context within the
bf16 tolerance.  Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ret):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import fable_attn as fa
        from fable_attn import multigpu as M
        dev = torch.device("cuda", rank)
        B, H, Hk, D, page = 4, 16, 4, 128, 64
        rng = np.random.default_rng(0)              # the same global cache on every rank
        lens = np.array([3000, 640, 1999, 129])
        nper = int((lens.max() + page - 1) // page)
        kc = torch.from_numpy(rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)).to(dev, torch.bfloat16)
        vc = torch.from_numpy(rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)).to(dev, torch.bfloat16)
        bt = torch.from_numpy(rng.permutation(B * nper).astype(np.int32).reshape(B, nper)).to(dev)
        q = torch.from_numpy(rng.standard_normal((B, 1, H, D)).astype(np.float32)).to(dev, torch.bfloat16)
        ref = fa.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                                         block_table=bt)
        # this rank's chunk, copied into its own dense pages (page-aligned local positions)
        starts, ends = M.plan_kv_split(torch.from_numpy(lens), world)
        s, e = starts[rank], ends[rank]
        loc = (e - s).to(torch.int32)
        lp = int((int(loc.max()) + page - 1) // page)
        kl = torch.zeros(B * lp, page, Hk, D, device=dev, dtype=torch.bfloat16)
        vl = torch.zeros_like(kl)
        for b in range(B):
            fk = kc[bt[b].long()].reshape(-1, Hk, D)[int(s[b]):int(e[b])]
            fv = vc[bt[b].long()].reshape(-1, Hk, D)[int(s[b]):int(e[b])]
            kl.view(B, lp * page, Hk, D)[b, :fk.shape[0]] = fk
            vl.view(B, lp * page, Hk, D)[b, :fv.shape[0]] = fv
        btl = torch.arange(B * lp, device=dev, dtype=torch.int32).view(B, lp)
        out = M.decode_kv_split(q, kl, vl, btl, loc.to(dev))
        err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        # the same step captured in a CUDA graph (all-gather as a graph node) replays bitwise
        graph = M.DecodeKVSplitGraph(q, kl, vl, btl, loc.to(dev))
        try:
            for _ in range(2):
                if not torch.equal(graph.replay(), out):
                    err = float("inf")
            torch.cuda.synchronize()
        finally:
            graph.close()
            del graph
        # the exchange over peer memory (one merge kernel reading every rank's buffer over NVLink),
        # eager and graph-replayed, gives the NCCL path's result
        ex = M.PeerDecodeExchange(B, 1, H, D, dev)
        loc = loc.to(dev)   # device tensors only: the step is captured below
        try:
            for _ in range(2):
                got = ex.step(q, kl, vl, btl, loc)
                err = max(err, ((got.float() - ref.float()).norm() / ref.float().norm()).item())
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                ex.step(q, kl, vl, btl, loc)
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):   # two steps: one per slot of the double buffer
                gouts = [ex.step(q, kl, vl, btl, loc) for _ in range(2)]
            for _ in range(3):
                g.replay()
                torch.cuda.synchronize()
                for gout in gouts:
                    err = max(err, ((gout.float() - ref.float()).norm() / ref.float().norm()).item())
            if int(ex.err.item()) != 0 or int(ex.step_count.item()) != 3 + 6:
                err = float("inf")
            del g
        finally:
            ex.close()
        ret[rank] = err
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_decode_kv_split_nccl_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    assert len(ret) == 2 and max(ret.values()) < 2.5e-3


def _chunked_case(dev, world):
    """A paged cache and, per emulated rank, its contiguous chunk of every sequence copied into its
    own pages (what each rank of decode_kv_split holds)."""
    from fable_attn import multigpu as M
    B, H, Hk, D, page = 4, 16, 4, 128, 64
    rng = np.random.default_rng(1)
    lens = np.array([3000, 640, 1999, 129])
    nper = int((lens.max() + page - 1) // page)
    kc = torch.from_numpy(rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)).to(dev, torch.bfloat16)
    vc = torch.from_numpy(rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)).to(dev, torch.bfloat16)
    bt = torch.from_numpy(rng.permutation(B * nper).astype(np.int32).reshape(B, nper)).to(dev)
    q = torch.from_numpy(rng.standard_normal((B, 1, H, D)).astype(np.float32)).to(dev, torch.bfloat16)
    starts, ends = M.plan_kv_split(torch.from_numpy(lens), world)
    chunks = []
    for r in range(world):
        s, e = starts[r], ends[r]
        loc = (e - s).to(torch.int32)
        lp = max(int((int(loc.max()) + page - 1) // page), 1)
        kl = torch.zeros(B * lp, page, Hk, D, device=dev, dtype=torch.bfloat16)
        vl = torch.zeros_like(kl)
        for b in range(B):
            kl.view(B, lp * page, Hk, D)[b, :int(e[b] - s[b])] = kc[bt[b].long()].reshape(-1, Hk, D)[int(s[b]):int(e[b])]
            vl.view(B, lp * page, Hk, D)[b, :int(e[b] - s[b])] = vc[bt[b].long()].reshape(-1, Hk, D)[int(s[b]):int(e[b])]
        chunks.append((kl, vl, torch.arange(B * lp, device=dev, dtype=torch.int32).view(B, lp), loc.to(dev)))
    return q, kc, vc, bt, lens, chunks


def test_decode_kv_split_one_process_equals_decode():
    """The N=1 form of decode_kv_split (no process group: the exchange is the local buffer)."""
    import fable_attn as fa
    from fable_attn import multigpu as M
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, lens, chunks = _chunked_case(dev, 1)
    ref = fa.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                                     block_table=bt)
    out = M.decode_kv_split(q, *chunks[0])
    assert (out.float() - ref.float()).norm() / ref.float().norm() < 2.5e-3


@pytest.mark.parametrize("world", [2, 3, 8])
def test_packed_partials_merge_in_place(world):
    """What every rank of decode_kv_split computes after its all-gather, with the ranks emulated as
    context chunks on one GPU: each chunk's decode writes its packed (out, lse) buffer, the buffers
    are concatenated in rank order (the all-gather's layout) and merged in place."""
    import fable_attn as fa
    from fable_attn import _C
    from fable_attn import multigpu as M
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, lens, chunks = _chunked_case(dev, world)
    ref = fa.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                                     block_table=bt)
    B, nq, H, D = q.shape
    sends = []
    for kl, vl, btl, loc in chunks:
        send = torch.empty(B * nq * H * (D + 1), device=dev, dtype=torch.float32)
        o_v, l_v = M.packed_partial_views(send, B, nq, H, D)
        _C.dec(q, kl, vl, btl, loc, None, None, None, None, False, D ** -0.5, -1, 0, None, True, out_fp32=True,
               out=o_v, lse_out=l_v)
        sends.append(send)
    recv = torch.cat(sends)
    out = _C.combine_packed(recv, world, B, nq, H, D, q.dtype)
    assert (out.float() - ref.float()).norm() / ref.float().norm() < 2.5e-3
    # the same merge through flash_attn_combine on the unpacked layout agrees bitwise
    o_all, l_all = M.unpack_partials(recv, world, B, nq, H, D)
    out2 = fa.flash_attn_combine(o_all.contiguous(), l_all.contiguous(), out_dtype=q.dtype)
    assert torch.equal(out, out2)


def test_decode_kv_split_graph_replays_the_step():
    """The captured decode step (N=1 form) equals the op-by-op step, replay after replay, and picks
    up new query values written into the captured q in place."""
    from fable_attn import multigpu as M
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, lens, chunks = _chunked_case(dev, 1)
    g = M.DecodeKVSplitGraph(q, *chunks[0])
    try:
        for it in range(3):
            if it == 2:
                q.copy_(torch.randn_like(q))
            want = M.decode_kv_split(q, *chunks[0])
            got = g.replay().clone()
            torch.cuda.synchronize()
            assert torch.equal(got, want)
    finally:
        g.close()


@pytest.mark.parametrize("slots", [1, 2])
def test_peer_exchange_one_process(slots):
    """PeerDecodeExchange with one rank (no process group): the merge kernel reads only its own
    buffer; eager and graph-replayed steps equal the decode, and the device step counter advances
    (a two-slot graph holds two steps)."""
    from fable_attn import multigpu as M
    dev = torch.device("cuda", 0)
    q, kc, vc, bt, lens, chunks = _chunked_case(dev, 1)
    import fable_attn as fa
    ref = fa.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                                     block_table=bt)
    ex = M.PeerDecodeExchange(q.shape[0], 1, q.shape[2], q.shape[3], dev, slots=slots)
    out = ex.step(q, *chunks[0])
    assert (out.float() - ref.float()).norm() / ref.float().norm() < 2.5e-3
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ex.step(q, *chunks[0])
    torch.cuda.current_stream().wait_stream(side)
    per_graph = 2 if slots == 2 else 1
    with torch.cuda.graph(g):
        gouts = [ex.step(q, *chunks[0]) for _ in range(per_graph)]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for gout in gouts:
        assert torch.equal(gout, out)
    assert int(ex.step_count.item()) == 2 + 3 * per_graph and int(ex.err.item()) == 0
    del g
    ex.close()
