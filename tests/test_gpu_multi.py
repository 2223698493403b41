"""Sequence sharding on real GPUs: two ranks (one per GPU, NCCL only to
compare results afterwards) each run the whole forward on their run of
whole sequences; the rows they produce equal the single-GPU forward of the
whole batch at the whole-forward bar.  Skipped where fewer than 2 GPUs are
visible."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-5
SEQS, SEQ_LEN = 6, 70


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch():
    rng = np.random.default_rng(11)
    ids = rng.integers(0, 4096, (SEQS, SEQ_LEN))
    mask = np.ones((SEQS, SEQ_LEN), np.int64)
    mask[1, 0:SEQ_LEN - 1:3] = 0
    mask[4, :9] = 0
    return ids, mask


def _config():
    from qdc_b200.model import Config
    return Config(hidden=256, head_dim=64, heads=4, kv_heads=2, key_heads=2, value_heads=4, key_dim=128,
                  value_dim=128, eps=float(np.float32(1e-6)), rope_theta=float(np.float32(1e7)),
                  rotary_dim=16, vocab=4096, intermediate=768,
                  layer_types=["linear_attention"] * 3 + ["full_attention"])


def _rank_main(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "qwendecisioncore.jl_b200")]
    import torch.distributed as dist
    import qdc_b200 as q
    from qdc_b200.shard import sequence_shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        model = q.QwenBackbone.random(_config(), seed=7, device=dev)
        ids, mask = _batch()
        s, e = sequence_shard(SEQS, world, rank)
        rows = model.batch_hidden(ids[s:e], mask[s:e]).view(e - s, SEQ_LEN, -1)  # this rank's run
        gathered = [torch.empty_like(rows) for _ in range(world)]
        dist.all_gather(gathered, rows)                                              # after the work
        if rank == 0:
            np.save(os.path.join(out_dir, "sharded.npy"), torch.cat(gathered).cpu().numpy())
            full = model.batch_hidden(ids, mask).view(SEQS, SEQ_LEN, -1)  # the whole batch, one GPU
            np.save(os.path.join(out_dir, "single.npy"), full.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sequence_shards_match_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    sharded = np.load(tmp_path / "sharded.npy").astype(np.float64)
    single = np.load(tmp_path / "single.npy").astype(np.float64)
    assert sharded.shape == (SEQS, SEQ_LEN, 256)
    assert np.all(np.abs(sharded - single) <= TOL + TOL * np.abs(single))
