"""Multi-GPU partitioning of the attention path (one process per GPU, torch.distributed).

Only two kinds of work are split, and only one of them communicates:

* independent units — heads (dense forward), (batch, head) pairs (forward+backward), kv-head
  groups (varlen prefill): `shard_range` gives each rank its contiguous slice; no collective.
* long-context decode — every sequence's KV range [0, L_b) is cut into `world` contiguous
  chunks; rank r holds the pages of its chunk locally and attends to them, producing a
  normalised partial output and its LSE, packed into one fp32 buffer.  One all-gather (NCCL over
  NVLink) brings every rank's packed buffer to every rank, and the merge kernel applies the LSE
  rule out = sum_r exp(lse_r - M) out_r / sum_r exp(lse_r - M), M = max_r lse_r, reading the
  gathered buffer in place.
  PeerDecodeExchange replaces the all-gather and the merge with one kernel that loads every
  rank's packed partial over NVLink (peer pointers of a symmetric allocation, plain loads, no
  multicast) after a bounded ready handshake.
  The reference has no multi-GPU layer; the merge rule is its flash_attn_combine
  (package/fable_attn/flash_attn_interface.py:567-580).
"""
import torch
import torch.distributed as dist


def shard_range(n, world, rank):
    """Contiguous share [lo, hi) of n units for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def plan_kv_split(lengths, world):
    """Per-rank position ranges of each sequence: (starts, ends) int64 tensors of shape
    (world, batch) with rank r owning [starts[r,b], ends[r,b]) = [floor(L*r/R), floor(L*(r+1)/R))."""
    L = torch.as_tensor(lengths, dtype=torch.int64).flatten()
    r = torch.arange(world + 1, dtype=torch.int64).view(-1, 1)
    cuts = (L.view(1, -1) * r) // world
    return cuts[:-1].contiguous(), cuts[1:].contiguous()


def local_block_table(block_table, start, end, page):
    """Block-table rows of one rank's chunk: the pages covering [start, end) of each sequence,
    re-based so local position 0 is global position start (start must be page-aligned for the
    pages to be reused as they are; callers that place data per rank build their own pages)."""
    nb = int(((end - start).max().item() + page - 1) // page) if end.numel() else 0
    rows = []
    for b in range(block_table.shape[0]):
        first = int(start[b]) // page
        row = block_table[b, first:first + max(nb, 1)]
        if row.numel() < max(nb, 1):
            row = torch.cat([row, row.new_zeros(max(nb, 1) - row.numel())])
        rows.append(row)
    return torch.stack(rows).contiguous()


def _world(group):
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def gather_partials(out_r, lse_r, group=None):
    """All-gather every rank's partial (out_r (B, nq, H, D), lse_r (B, H, nq) fp32) into
    (world, B, nq, H, D) and (world, B, H, nq).  Two collectives; decode_kv_split sends one packed
    buffer instead (pack_partials / unpack_partials)."""
    world = dist.get_world_size(group)
    # flat (world * dim0, ...) buffers: the layout both NCCL and gloo gather into
    out_all = out_r.new_empty((world * out_r.shape[0],) + tuple(out_r.shape[1:]))
    lse_all = lse_r.new_empty((world * lse_r.shape[0],) + tuple(lse_r.shape[1:]))
    dist.all_gather_into_tensor(out_all, out_r.contiguous(), group=group)
    dist.all_gather_into_tensor(lse_all, lse_r.contiguous(), group=group)
    return out_all.view((world,) + tuple(out_r.shape)), lse_all.view((world,) + tuple(lse_r.shape))


def packed_partial_views(buf, B, nq, H, D):
    """One rank's packed partial: B*nq*H output rows of D fp32 values, then the rows' fp32 LSE in
    the same (b, t, h) order.  Returns the (out (B, nq, H, D), lse (B, nq, H)) views of buf."""
    rows = B * nq * H
    return buf[:rows * D].view(B, nq, H, D), buf[rows * D:rows * (D + 1)].view(B, nq, H)


def pack_partials(out_r, lse_r):
    """(out (B, nq, H, D), lse (B, nq, H)) fp32 -> one flat fp32 buffer of B*nq*H*(D+1) floats."""
    return torch.cat([out_r.reshape(-1).float(), lse_r.reshape(-1).float()])


def unpack_partials(recv, world, B, nq, H, D):
    """Gathered packed buffers (world * B*nq*H*(D+1) floats) -> (out (world, B, nq, H, D),
    lse (world, B, H, nq)): the layout flash_attn_combine takes."""
    per = recv.view(world, -1)
    rows = B * nq * H
    out = per[:, :rows * D].reshape(world, B, nq, H, D)
    lse = per[:, rows * D:].reshape(world, B, nq, H).transpose(2, 3)
    return out, lse


def exchange(send, group=None):
    """One all-gather of every rank's packed partial into (world * len) floats (world = 1: send)."""
    world = _world(group)
    if world == 1:
        return send
    recv = send.new_empty(world * send.numel())
    dist.all_gather_into_tensor(recv, send, group=group)
    return recv


def decode_kv_split(q, k_cache_local, v_cache_local, block_table_local, local_lengths, softmax_scale=None,
                    group=None, num_splits=0, phase_events=None):
    """Decode against a context split across ranks (no rotary / alibi / window: those depend on
    the global query position and are served by the single-GPU flash_attn_with_kvcache).
    Each rank passes its local paged cache and local lengths; every rank returns the full
    output (B, nq, H, D) in q's dtype.
      1. the decode kernels write this rank's partial output (fp32: its 16-bit rounding would add
         to the final one) and LSE straight into one packed send buffer;
      2. one all-gather (NCCL over NVLink) of the packed buffers;
      3. the merge kernel reads the gathered buffer in place (no unpacking copies).
    phase_events: optional list of 4 CUDA events recorded at the phase boundaries (timing)."""
    from . import _C
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    B, nq, H, D = q.shape
    lens = local_lengths.to(device=q.device, dtype=torch.int32).contiguous()
    send = torch.empty(B * nq * H * (D + 1), device=q.device, dtype=torch.float32)
    out_v, lse_v = packed_partial_views(send, B, nq, H, D)
    ev = phase_events or [None] * 4
    if ev[0] is not None:
        ev[0].record()
    _C.dec(q.contiguous(), k_cache_local, v_cache_local, block_table_local.to(torch.int32).contiguous(), lens, None,
           None, None, None, False, float(scale), -1, int(num_splits), None, True, out_fp32=True, out=out_v,
           lse_out=lse_v)
    if ev[1] is not None:
        ev[1].record()
    recv = exchange(send, group)
    if ev[2] is not None:
        ev[2].record()
    out = _C.combine_packed(recv, recv.numel() // send.numel(), B, nq, H, D, q.dtype)
    if ev[3] is not None:
        ev[3].record()
    return out


class DecodeKVSplitGraph:
    """decode_kv_split captured once in a CUDA graph and replayed per decode step.

    A split decode step is three short launches (the decode partial, the all-gather, the merge);
    at 1/8 of a context each takes tens of microseconds, so launching them from Python every step
    costs as much as running them.  The graph is captured for fixed input tensors (q, the local
    cache, block table and lengths are read in place, so a caller updates them between steps) and
    one replay runs the whole step; `out` is the graph's output tensor.  NCCL collectives are
    captured as graph nodes; every rank must capture and replay in the same order.  Call close()
    (or drop the object) before destroying the process group."""

    def __init__(self, q, k_cache_local, v_cache_local, block_table_local, local_lengths, softmax_scale=None,
                 group=None, num_splits=0, warmup=3):
        args = (q, k_cache_local, v_cache_local, block_table_local, local_lengths)
        self._args, self._kw = args, dict(softmax_scale=softmax_scale, group=group, num_splits=num_splits)
        side = torch.cuda.Stream(device=q.device)
        side.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(side):   # warm-up off the capture (allocator pools, NCCL communicator)
            for _ in range(warmup):
                decode_kv_split(*args, **self._kw)
        torch.cuda.current_stream(q.device).wait_stream(side)
        torch.cuda.synchronize(q.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = decode_kv_split(*args, **self._kw)

    def replay(self):
        self.graph.replay()
        return self.out

    def close(self):
        self.graph = None
        self.out = None


class PeerDecodeExchange:
    """decode_kv_split with the all-gather and the merge replaced by one kernel over peer memory.

    Every rank's packed partial lives in one symmetric allocation (torch's symmetric memory: each
    rank can load every other rank's buffer through NVLink).  A step is: this rank's decode writes
    its partial into its own buffer; the merge kernel tells every peer this rank is ready, waits
    until every peer is, and merges each row straight from all ranks' buffers (P2P loads, no copy).

    slots=2 (default): the buffer holds two partials and steps alternate between them.  A slot is
    rewritten two steps later, and by then every peer has said "ready" for the step in between,
    which it only does after its previous merge finished reading, so a step is two launches (the
    decode and the merge, which also advances the device step counter).  slots=1: one partial and a
    third launch per step, the step end, which tells every peer this rank is done reading and waits
    for every peer's done before the buffer may be overwritten.

    The step number is a device counter, so steps can be captured in a CUDA graph; with slots=2 a
    captured graph must hold an even number of steps (the host picks the slot of each step).  Waits
    are bounded: a peer that does not arrive sets `err` (read it with int(err)) instead of hanging
    the GPU.  Every rank of `group` must construct the exchange and run the same steps; drop it
    before destroying the process group."""

    SIGNAL_WORDS_OFFSET = 256   # our words start past the part of the signal pad torch may use itself

    def __init__(self, B, nq, H, D, device, group=None, slots=2):
        import os
        # plain peer loads only: no NVLink multicast object is created for the buffers
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        if slots not in (1, 2):
            raise ValueError("PeerDecodeExchange: slots must be 1 or 2")
        self.world = _world(group)
        self.B, self.nq, self.H, self.D, self.slots = B, nq, H, D, slots
        if self.world > 8:
            raise ValueError("PeerDecodeExchange: at most 8 ranks")
        per = B * nq * H * (D + 1)
        self.per = per
        dev = torch.device(device)
        if self.world > 1:
            self.buf = symm_mem.empty(slots * per, dtype=torch.float32, device=dev)
            g = group if group is not None else dist.group.WORLD
            self.hdl = symm_mem.rendezvous(self.buf, g)
            self.rank = self.hdl.rank
            pad_words = self.hdl.signal_pad_size // 4
            if pad_words < self.SIGNAL_WORDS_OFFSET + 2 * self.world:
                raise RuntimeError("PeerDecodeExchange: signal pad too small")
            own = self.hdl.get_signal_pad(self.rank, (pad_words,), dtype=torch.int32)
            own.zero_()
            torch.cuda.synchronize(dev)
            dist.barrier(group=group)
            # the buffer sits at the same offset in every rank's block of the symmetric allocation
            off = self.buf.data_ptr() - self.hdl.buffer_ptrs[self.rank]
            if not 0 <= off <= self.hdl.buffer_size - 4 * slots * per:
                raise RuntimeError("PeerDecodeExchange: buffer outside its symmetric block")
            bufs = [a + off for a in self.hdl.buffer_ptrs]
            sigs = [a + 4 * self.SIGNAL_WORDS_OFFSET for a in self.hdl.signal_pad_ptrs]
        else:
            self.buf = torch.empty(slots * per, dtype=torch.float32, device=dev)
            self.hdl, self.rank = None, 0
            self._own_signal = torch.zeros(2, dtype=torch.int32, device=dev)
            bufs, sigs = [self.buf.data_ptr()], [self._own_signal.data_ptr()]
        self.peer_bufs = torch.tensor(bufs, dtype=torch.int64, device=dev)
        self.peer_signals = torch.tensor(sigs, dtype=torch.int64, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done_ctas = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.views = [packed_partial_views(self.buf[i * per:(i + 1) * per], B, nq, H, D) for i in range(slots)]
        self.out_view, self.lse_view = self.views[0]
        self._issued = 0   # steps enqueued by this host (the slot of the next one is _issued % slots)

    def step(self, q, k_cache_local, v_cache_local, block_table_local, local_lengths, softmax_scale=None,
             num_splits=0, phase_events=None):
        """One decode step over this rank's chunk of the context; returns the merged output
        (B, nq, H, D) in q's dtype.  phase_events: optional CUDA events (3, or 4 with slots=1)
        recorded around the partial, the peer merge and the step end."""
        from . import _C
        scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
        ev = list(phase_events or []) + [None] * 4
        lens = local_lengths.to(device=q.device, dtype=torch.int32)
        args = (self.peer_bufs, self.peer_signals, self.rank, self.world, self.B, self.nq, self.H, self.D,
                self.step_count, self.err)
        out_v, lse_v = self.views[self._issued % self.slots]
        self._issued += 1
        if ev[0] is not None:
            ev[0].record()
        _C.dec(q.contiguous(), k_cache_local, v_cache_local, block_table_local.to(torch.int32).contiguous(),
               lens.contiguous(), None, None, None, None, False, float(scale), -1, int(num_splits), None, True,
               out_fp32=True, out=out_v, lse_out=lse_v)
        if ev[1] is not None:
            ev[1].record()
        if self.slots == 2:
            out = _C.peer_merge(*args, q.dtype, slot_floats=self.per, done_ctas=self.done_ctas)
            if ev[2] is not None:
                ev[2].record()
            return out
        out = _C.peer_merge(*args, q.dtype)
        if ev[2] is not None:
            ev[2].record()
        _C.peer_step_end(*args)
        if ev[3] is not None:
            ev[3].record()
        return out

    def close(self):
        self.hdl = None
        self.buf = None
