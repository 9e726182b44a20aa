"""Row sharding across ranks: rows are independent (src/generation.js pickToken
is per row), so each rank samples a contiguous block with no collective."""
from __future__ import annotations


def row_shard(B: int, world: int, rank: int) -> tuple[int, int]:
    """[r0, r1) rows of rank `rank` when B rows are split over `world` ranks:
    contiguous blocks of ceil(B / world), the last ones possibly short or empty."""
    if world < 1 or not 0 <= rank < world or B < 0:
        raise ValueError("bad shard arguments")
    per = -(-B // world)
    r0 = min(B, rank * per)
    return r0, min(B, r0 + per)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of a per-rank value (step time) over the process group."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return float(t[0])


# ---------------------------------------------------------------- vocabulary sharding
def col_shard(V: int, world: int, rank: int) -> tuple[int, int]:
    """[c0, c1) columns of rank `rank` when V columns are split over `world`
    ranks (contiguous, ceil(V / world) wide, the last ones possibly short)."""
    return row_shard(V, world, rank)


def exchange_records(rec, group=None):
    """All-to-all of shard records so that each rank holds every shard's record
    of the rows it merges.  rec: this rank's [B, R] uint8 records (one per row).
    Returns ([Bb, world, R] records of rows [rank*Bb, rank*Bb + Bb) in shard
    order, Bb) with Bb = ceil(B / world); rows past B are zero padding."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    B, R = rec.shape
    Bb = -(-B // world)
    if world * Bb == B and rec.is_contiguous():
        send = rec  # no padding rows needed
    else:
        send = torch.zeros((world * Bb, R), dtype=rec.dtype, device=rec.device)
        send[:B] = rec
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)  # block s of recv: shard s's records of my rows
    return recv.view(world, Bb, R).permute(1, 0, 2).contiguous(), Bb


def gather_rows(shard_rows, group=None):
    """Whole rows from their column shards: [n, cols_g] on each rank (the same
    n rows everywhere) -> [n, V] on every rank, columns in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n = shard_rows.shape[0]
    widths = [None] * world
    dist.all_gather_object(widths, int(shard_rows.shape[1]), group=group)
    wmax = max(widths)
    buf = torch.zeros((n, wmax), dtype=shard_rows.dtype, device=shard_rows.device)
    buf[:, : shard_rows.shape[1]] = shard_rows
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[g][:, : widths[g]] for g in range(world)], dim=1)


def sample_vocab_sharded(sampler, logits_shard, col0: int, V: int, params, u, hist=None, hist_off=None,
                         group=None, resolve: bool = True):
    """Vocabulary-sharded sampling, one rank per column shard: the shard's
    records, an all-to-all so each rank merges a block of rows, an all-gather
    of the ids.  u: [B] fp64 CUDA uniforms (every rank the same).  Returns the
    [B] int32 ids on every rank.

    Rows the shard lists cannot settle (rare probability ties at a shard's
    cut) come back as -1.  With resolve=True they are then sampled from their
    gathered whole rows; that needs the ids on the host (one small copy, the
    same on every rank, so every rank takes the same collective steps).  With
    resolve=False nothing waits on the host: the caller gets the -1 rows and
    resolves them later with resolve_unsettled (bench loops keep the device
    busy this way)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B = logits_shard.shape[0]
    rec = sampler.shard_records(logits_shard, V, col0, params, hist, hist_off)
    recs, Bb = exchange_records(rec, group)
    r0, r1 = min(B, rank * Bb), min(B, rank * Bb + Bb)
    blk = torch.full((Bb,), -1, dtype=torch.int32, device=logits_shard.device)
    if r1 > r0:
        sampler.merge_records(recs[: r1 - r0], V, params, u=u[r0:r1], out=blk[: r1 - r0])
    allb = torch.empty((world * Bb,), dtype=torch.int32, device=logits_shard.device)
    dist.all_gather_into_tensor(allb, blk, group=group)
    ids = allb[:B]
    if resolve:
        ids = resolve_unsettled(sampler, ids, logits_shard, params, u, hist, hist_off, group)
    return ids


def resolve_unsettled(sampler, ids, logits_shard, params, u, hist=None, hist_off=None, group=None):
    """Samples the rows whose id is -1 from their whole rows (gathered from the
    column shards).  Every rank holds the same ids, so every rank finds the same
    rows and runs the same collectives."""
    import torch

    bad = torch.nonzero(ids.cpu() < 0).flatten().tolist()
    if not bad:
        return ids
    ids = ids.clone()
    bad_d = torch.tensor(bad, dtype=torch.int64, device=ids.device)
    rows = gather_rows(logits_shard[bad_d], group)
    sub_h = sub_o = None
    if hist_off is not None:
        offs = hist_off.cpu().numpy()
        hs = [hist[int(offs[i]):int(offs[i + 1])] for i in bad]
        sub_h = torch.cat(hs) if hs else hist[:0]
        sub_o = torch.tensor([0] + [int(x.numel()) for x in hs], dtype=torch.int64).cumsum(0).to(ids.device)
    ids[bad_d] = sampler.sample(rows.contiguous(), params, u=u[bad_d].contiguous(), hist=sub_h, hist_off=sub_o)
    return ids
