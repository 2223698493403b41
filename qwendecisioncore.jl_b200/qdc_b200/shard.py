"""Sequence sharding across the GPUs of one box.

Every per-layer kernel is independent per token row; the only sequence
dependence is the RoPE position, the token's index inside its own sequence
(src/backbone_cpu.jl:95; the reference runs one sequence per call,
src/backbone.jl:424-432).  A batch of equal-length sequences is therefore
split into contiguous runs of WHOLE sequences, one run per rank, and every
rank runs the same kernels on its run with `seq_len` set so positions restart
at each sequence boundary.  Nothing crosses ranks on the data path: no
collective is issued by the kernels.  The only cross-rank traffic is the
timing reduction (max over ranks) and, outside any timed region, an optional
gather of results.
"""
import torch


def sequence_shard(num_sequences, world, rank):
    """[start, stop) of the sequences rank `rank` of `world` owns.

    Sequences are dealt in contiguous blocks; when `num_sequences` does not
    divide evenly the first ranks take one extra sequence."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if num_sequences < 0:
        raise ValueError("negative sequence count")
    base, extra = divmod(num_sequences, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def token_rows(num_sequences, seq_len, world, rank):
    """[start, stop) token rows of the rank's shard in the flattened
    (sequences * seq_len, hidden) batch."""
    s, e = sequence_shard(num_sequences, world, rank)
    return s * seq_len, e * seq_len


def positions(rows, seq_len, first_row=0):
    """RoPE positions of `rows` consecutive token rows starting at global
    row `first_row`: (first_row + t) mod seq_len.  A shard always starts on a
    sequence boundary, so this equals t mod seq_len there."""
    return [(first_row + t) % seq_len for t in range(rows)]


def max_over_ranks(value, group=None, device=None):
    """The slowest rank's time: the job is done when the last rank is."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
