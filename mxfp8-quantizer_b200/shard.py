"""Row sharding of a quantization across ranks (one process per GPU).

Quantization is row-local and the packed scale storage is row-block major,
so a rank that owns whole 128-row chunks [r0, r1) owns Q rows [r0, r1) and
the contiguous scale bytes [r0/128 * CB * 512, ceil(r1/128) * CB * 512):
its outputs are slices of the global buffers and no exchange is needed.
"""

from __future__ import annotations

SCALE_ROWS_PER_PACK = 128


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def row_shard(m_total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank `rank`: whole 128-row chunks, as even as possible."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    chunks = ceil_div(m_total, SCALE_ROWS_PER_PACK)
    base, extra = divmod(chunks, world)
    c0 = rank * base + min(rank, extra)
    c1 = c0 + base + (1 if rank < extra else 0)
    return min(m_total, c0 * SCALE_ROWS_PER_PACK), min(m_total, c1 * SCALE_ROWS_PER_PACK)


def scale_byte_range(r0: int, r1: int, q_cols: int) -> tuple[int, int]:
    """Byte range of the packed scale storage owned by rows [r0, r1) (r0 % 128 == 0)."""
    if r0 % SCALE_ROWS_PER_PACK:
        raise ValueError("a shard must start on a 128-row chunk")
    chunk_row_bytes = ceil_div(ceil_div(q_cols, 32), 4) * 512
    return (r0 // SCALE_ROWS_PER_PACK) * chunk_row_bytes, ceil_div(r1, SCALE_ROWS_PER_PACK) * chunk_row_bytes


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(value: float, device=None) -> list[float]:
    """Every rank's value of a per-rank float, in rank order (a one-element
    list when torch.distributed is not initialised).  Every rank must call
    it, in the same order as its other collectives."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return [value]
    t = torch.tensor([value], dtype=torch.float64, device=device)
    parts = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return [float(p.item()) for p in parts]
