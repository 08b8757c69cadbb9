"""Request-level sharding across GPUs: the only way this path shards.  Sequences are independent (weights replicated,
state and KV cache live on the owning GPU), so sequence i goes to rank i mod world and no collective runs inside a
timed region.  After it, one all-reduce of the per-rank counters gives the whole-job figures: tokens are summed, the
time is the maximum over ranks (every rank starts after the same barrier, so the slowest one defines the job)."""
from dataclasses import dataclass

import torch
import torch.distributed as dist


def sequences_of_rank(n_sequences: int, world: int, rank: int):
    """Global indices of the sequences rank `rank` owns: i mod world == rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    return list(range(rank, n_sequences, world))


def sequence_seed(base: int, rank: int, local_index: int) -> int:
    """Seed of the token ids of a rank's local sequence (1000 * rank + local index, offset by `base`)."""
    return base + 1000 * rank + local_index


@dataclass
class JobCounters:
    tokens: int            # tokens produced inside the timed region, all ranks
    elapsed_ms: float      # slowest rank's device time
    algorithmic_bytes: int
    mismatches: int

    @property
    def tokens_per_s(self) -> float:
        return self.tokens / (self.elapsed_ms * 1e-3) if self.elapsed_ms > 0 else 0.0


def reduce_counters(tokens: int, elapsed_ms: float, algorithmic_bytes: int = 0, mismatches: int = 0, device="cpu") -> JobCounters:
    """Whole-job counters from this rank's.  Works without a process group (single rank)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return JobCounters(int(tokens), float(elapsed_ms), int(algorithmic_bytes), int(mismatches))
    sums = torch.tensor([tokens, algorithmic_bytes, mismatches], dtype=torch.int64, device=device)
    dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    tmax = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    return JobCounters(int(sums[0]), float(tmax[0]), int(sums[1]), int(sums[2]))
