"""Multi-GPU partitioning and the verification gather.

Every kbt_* op is independent across output rows and flash across
(batch, head) pairs, so the multi-GPU layout needs no exchange step:
``row_range`` / ``unit_range`` give each rank a contiguous shard, the timed
loop runs the op on the local shard only, and afterwards ``gather_rows``
collects a few sampled rows from every rank (an all-gather over the process
group: NCCL on GPUs, gloo in the CPU tests) so rank 0 can check them.
"""
from __future__ import annotations


def unit_range(units: int, world: int, rank: int, quantum: int = 1) -> tuple[int, int]:
    """Contiguous [start, end) of `units` for `rank`, balanced in multiples of `quantum`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    blocks = (units + quantum - 1) // quantum
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(units, b0 * quantum), min(units, b1 * quantum)


def row_range(M: int, world: int, rank: int) -> tuple[int, int]:
    """GEMM rows of `rank` (multiples of 8, as the C ABI requires)."""
    return unit_range(M, world, rank, 8)


def sample_rows(n: int, k: int = 4) -> list[int]:
    """A few verification rows of a shard: first, second, middle, last."""
    if n <= 0:
        return []
    cand = [0, 1, n // 2, n - 1][:max(1, k)]
    return sorted({r for r in cand if 0 <= r < n})


def gather_rows(tensors, world: int):
    """All-gather each tensor of `tensors` (same shape on every rank).

    Returns, per input tensor, the list of per-rank tensors.  With world == 1
    no process group is needed."""
    if world == 1:
        return [[t] for t in tensors]
    import torch
    import torch.distributed as dist
    out = []
    for t in tensors:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        out.append(parts)
    return out


def check_gathered(outs, ins, reference, parity) -> dict:
    """Check every rank's sampled output rows against `reference(in_rows)`.

    `outs`/`ins` are the per-rank lists from gather_rows; `reference` maps the
    sampled input rows (numpy) to the expected output rows; `parity` is
    akili_bench_b200.parity.parity.  Returns the worst rank's result."""
    worst = None
    for r, (o, x) in enumerate(zip(outs, ins)):
        p = parity(o.float().cpu().numpy(), reference(x.float().cpu().numpy()))
        p["rank"] = r
        if worst is None or (not p["ok"] and worst["ok"]) or (p["ok"] == worst["ok"] and
                                                              p["min_cos"] < worst["min_cos"]):
            worst = p
    return worst or {"ok": True, "rank": None}
