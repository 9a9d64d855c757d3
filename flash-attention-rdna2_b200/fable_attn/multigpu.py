"""Multi-GPU partitioning of the attention path (one process per GPU, torch.distributed).

Only two kinds of work are split, and only one of them communicates:

* independent units — heads (dense forward), (batch, head) pairs (forward+backward), kv-head
  groups (varlen prefill): `shard_range` gives each rank its contiguous slice; no collective.
* long-context decode — every sequence's KV range [0, L_b) is cut into `world` contiguous
  chunks; rank r holds the pages of its chunk locally and attends to them, producing a
  normalised partial output and its LSE.  One all-gather (NCCL over NVLink) brings every rank's
  (out, lse) pair to every rank, and flash_attn_combine merges them with the LSE rule
  out = sum_r exp(lse_r - M) out_r / sum_r exp(lse_r - M), M = max_r lse_r.
  The reference has no multi-GPU layer; the merge rule is its flash_attn_combine
  (package/fable_attn/flash_attn_interface.py:567-580).
Remote partials always arrive through NCCL into local buffers: no kernel reads peer memory.
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


def gather_partials(out_r, lse_r, group=None):
    """All-gather every rank's partial (out_r (B, nq, H, D), lse_r (B, H, nq) fp32) into
    (world, B, nq, H, D) and (world, B, H, nq)."""
    world = dist.get_world_size(group)
    # flat (world * dim0, ...) buffers: the layout both NCCL and gloo gather into
    out_all = out_r.new_empty((world * out_r.shape[0],) + tuple(out_r.shape[1:]))
    lse_all = lse_r.new_empty((world * lse_r.shape[0],) + tuple(lse_r.shape[1:]))
    dist.all_gather_into_tensor(out_all, out_r.contiguous(), group=group)
    dist.all_gather_into_tensor(lse_all, lse_r.contiguous(), group=group)
    return out_all.view((world,) + tuple(out_r.shape)), lse_all.view((world,) + tuple(lse_r.shape))


def decode_kv_split(q, k_cache_local, v_cache_local, block_table_local, local_lengths, softmax_scale=None,
                    group=None, num_splits=0):
    """Decode against a context split across ranks (no rotary / alibi / window: those depend on
    the global query position and are served by the single-GPU flash_attn_with_kvcache).
    Each rank passes its local paged cache and local lengths; every rank returns the full
    output (B, nq, H, D) in q's dtype.  The rank's partial stays fp32 until the LSE merge (its
    16-bit rounding would otherwise add to the final one)."""
    from . import _C
    from .flash_attn_interface import flash_attn_combine
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    lens = local_lengths.to(device=q.device, dtype=torch.int32).contiguous()
    out_r, lse_r = _C.dec(q.contiguous(), k_cache_local, v_cache_local, block_table_local.to(torch.int32).contiguous(),
                          lens, None, None, None, None, False, float(scale), -1, int(num_splits), None, True,
                          out_fp32=True)
    out_all, lse_all = gather_partials(out_r, lse_r.transpose(1, 2).contiguous(), group)
    return flash_attn_combine(out_all, lse_all, out_dtype=q.dtype)
