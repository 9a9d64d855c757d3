"""Host-side multi-rank logic on CPU ranks (gloo, world_size 2 and 3): the KV-range plan, the
all-gather of partial (out, lse) pairs, and the LSE merge reproduce single-process decode.  The
per-rank partial attention is computed by the CPU oracle here (the GPU path runs the decode
kernel); the merge is checked with the oracle's combine."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fable_attn import multigpu as M


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from oracle import oracle as O
        rng = np.random.default_rng(0)            # same data on every rank
        B, H, Hk, D, page = 3, 8, 2, 32, 16
        lens = np.array([101, 64, 7], np.int32)
        nper = 8
        kc = rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)
        vc = rng.standard_normal((B * nper, page, Hk, D)).astype(np.float32)
        bt = rng.permutation(B * nper).astype(np.int32).reshape(B, nper)
        q = rng.standard_normal((B, 1, H, D)).astype(np.float32)
        starts, ends = M.plan_kv_split(lens, world)
        # this rank's data placement: its positions copied into a local dense-per-sequence cache
        s, e = starts[rank].numpy(), ends[rank].numpy()
        Lmax = max(int((e - s).max()), 1)
        kl = np.zeros((B, Lmax, Hk, D), np.float32)
        vl = np.zeros((B, Lmax, Hk, D), np.float32)
        for b in range(B):
            full_k = kc[bt[b]].reshape(-1, Hk, D)
            full_v = vc[bt[b]].reshape(-1, Hk, D)
            kl[b, : e[b] - s[b]] = full_k[s[b]:e[b]]
            vl[b, : e[b] - s[b]] = full_v[s[b]:e[b]]
        o_r, l_r = O.decode(q, kl, vl, np.arange(B, dtype=np.int32)[:, None], (e - s).astype(np.int32))
        # the exchange decode_kv_split makes: one packed (out rows, LSE) buffer per rank, one all-gather
        send = M.pack_partials(torch.from_numpy(o_r), torch.from_numpy(l_r))
        views = M.packed_partial_views(send, B, 1, H, D)
        assert np.array_equal(views[0].numpy(), o_r) and np.array_equal(views[1].numpy(), l_r)
        out_all, lse_all = M.unpack_partials(M.exchange(send), world, B, 1, H, D)
        merged, _ = O.combine(out_all.numpy(), lse_all.numpy())
        # and the two-collective form agrees with it
        out2, lse2 = M.gather_partials(torch.from_numpy(o_r), torch.from_numpy(l_r).transpose(1, 2).contiguous())
        assert torch.equal(out2, out_all) and torch.equal(lse2, lse_all)
        ref, _ = O.decode(q, kc, vc, bt, lens)
        ret[rank] = float(np.abs(merged - ref).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_decode_kv_split_gather_combine(world):
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert len(ret) == world and max(ret.values()) < 1e-5


def test_plan_and_shard_cover_everything():
    lens = torch.tensor([0, 1, 5, 16384, 32768])
    for world in (1, 2, 4, 8):
        s, e = M.plan_kv_split(lens, world)
        assert torch.equal(s[0], torch.zeros_like(lens)) and torch.equal(e[-1], lens)
        assert torch.equal(s[1:], e[:-1]) and bool((e >= s).all())
        spans = [M.shard_range(32, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 32
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
