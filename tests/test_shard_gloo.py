"""Sequence sharding over 2 ranks (gloo, CPU): each rank runs the per-layer
ops on its run of whole sequences; the concatenation equals the unsharded
result and the timing reduction returns the slowest rank's time."""
import os
import socket

import numpy as np
import pytest


def test_sequence_shard_partitions():
    from qdc_b200.shard import sequence_shard, token_rows
    for n in (0, 1, 5, 32):
        for world in (1, 2, 3, 4, 8):
            spans = [sequence_shard(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    assert token_rows(32, 2048, 8, 3) == (3 * 4 * 2048, 4 * 4 * 2048)
    with pytest.raises(ValueError):
        sequence_shard(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import sys
    import time
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                 "qwendecisioncore.jl_b200")]
    import torch.distributed as dist
    from oracle import oracle as O
    from qdc_b200.shard import max_over_ranks, token_rows
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    seqs, seq_len, heads, dim, rotary = 5, 37, 2, 64, 16
    rng = np.random.default_rng(0)  # same global batch on every rank
    x = rng.normal(0, 1, (seqs * seq_len, heads, dim)).astype(np.float32)
    m = rng.normal(0, 1, (seqs * seq_len, heads * dim)).astype(np.float32)
    w = rng.normal(0, 0.02, dim).astype(np.float32)
    wh = rng.normal(0, 0.02, heads * dim).astype(np.float32)
    cos, sin = O.rope_table(1e7, rotary, seq_len)
    a, b = token_rows(seqs, seq_len, world, rank)
    qk = O.qk_norm_rope(x[a:b], w, 1e-6, rotary, cos, sin, seq_len=seq_len)
    _, y = O.residual_rms(x[a:b].reshape(b - a, -1), m[a:b], wh, 1e-6)
    np.save(os.path.join(out_dir, f"qk{rank}.npy"), qk)
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    t = max_over_ranks(0.5 + rank)
    np.save(os.path.join(out_dir, f"t{rank}.npy"), np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_shards_match_unsharded(tmp_path, oracle):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    seqs, seq_len, heads, dim, rotary = 5, 37, 2, 64, 16
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (seqs * seq_len, heads, dim)).astype(np.float32)
    m = rng.normal(0, 1, (seqs * seq_len, heads * dim)).astype(np.float32)
    w = rng.normal(0, 0.02, dim).astype(np.float32)
    wh = rng.normal(0, 0.02, heads * dim).astype(np.float32)
    cos, sin = oracle.rope_table(1e7, rotary, seq_len)
    full_qk = oracle.qk_norm_rope(x, w, 1e-6, rotary, cos, sin, seq_len=seq_len)
    _, full_y = oracle.residual_rms(x.reshape(len(x), -1), m, wh, 1e-6)
    qk = np.concatenate([np.load(tmp_path / f"qk{r}.npy") for r in range(world)])
    y = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    assert np.array_equal(qk, full_qk) and np.array_equal(y, full_y)
    assert all(float(np.load(tmp_path / f"t{r}.npy")[0]) == 1.5 for r in range(world))
