"""Host-side multi-GPU logic on CPU: world_size-2 gloo ranks check the sequence partition and the counter reduction."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "lucebox-hub_b200"))


def _free_port():
    s = socket.socket(); s.bind(("127.0.0.1", 0)); p = s.getsockname()[1]; s.close(); return p


def _rank_main(rank, world, port, n_seq, out_dir):
    from qwen35_b200.sharding import reduce_counters, sequence_seed, sequences_of_rank
    os.environ["MASTER_ADDR"] = "127.0.0.1"; os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mine = sequences_of_rank(n_seq, world, rank)
    # every rank sees every rank's list: the lists partition range(n_seq)
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    flat = sorted(i for part in gathered for i in part)
    assert flat == list(range(n_seq))
    assert all(i % world == r for r, part in enumerate(gathered) for i in part)
    seeds = [sequence_seed(0, rank, j) for j in range(len(mine))]
    all_seeds = [None] * world
    dist.all_gather_object(all_seeds, seeds)
    assert len({s for part in all_seeds for s in part}) == n_seq           # no two sequences share a seed
    # rank r produced 10 tokens per sequence in (5 + r) ms: the job is the sum of tokens over the slowest rank's time
    job = reduce_counters(tokens=10 * len(mine), elapsed_ms=5.0 + rank, algorithmic_bytes=100 * len(mine), mismatches=rank)
    assert job.tokens == 10 * n_seq and job.elapsed_ms == 5.0 + (world - 1)
    assert job.algorithmic_bytes == 100 * n_seq and job.mismatches == sum(range(world))
    assert abs(job.tokens_per_s - job.tokens / (job.elapsed_ms * 1e-3)) < 1e-9
    dist.barrier()
    dist.destroy_process_group()
    open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")


@pytest.mark.parametrize("n_seq", [7, 64])
def test_two_gloo_ranks_partition_and_reduce(tmp_path, n_seq):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), n_seq, str(tmp_path)), nprocs=world, join=True)
    assert all((tmp_path / f"ok{r}").exists() for r in range(world))


def test_single_rank_needs_no_process_group():
    from qwen35_b200.sharding import reduce_counters, sequences_of_rank
    assert sequences_of_rank(5, 1, 0) == [0, 1, 2, 3, 4]
    j = reduce_counters(12, 3.0)
    assert j.tokens == 12 and j.elapsed_ms == 3.0 and j.tokens_per_s == 4000.0
    with pytest.raises(ValueError):
        sequences_of_rank(5, 2, 2)
