"""KV-head sharding of the decode across GPUs (one process per GPU).

The op splits by KV head with no exchange step: rank r of N owns KV heads
[r*Hkv/N, (r+1)*Hkv/N), their K/V pool (its own allocation, [num_pages, P, Hkv/N, D]) and
query heads [r*Hq/N, (r+1)*Hq/N); block_table and seq_lens are replicated.  Each rank
runs the single-GPU decode on its shard.  Assembling the full [B, Hq, D] output is an
optional all-gather over the process group (NCCL on GPUs), timed separately from the
decode.
"""
import torch
import torch.distributed as dist


def kv_head_range(rank, world_size, num_heads_k):
    if num_heads_k % world_size != 0:
        raise ValueError(f"num_heads_k={num_heads_k} is not divisible by {world_size} ranks")
    per = num_heads_k // world_size
    return rank * per, (rank + 1) * per


def q_head_range(rank, world_size, num_heads, num_heads_k):
    lo, hi = kv_head_range(rank, world_size, num_heads_k)
    g = num_heads // num_heads_k
    return lo * g, hi * g


def shard_tensors(q, k_cache, v_cache, rank, world_size):
    """Slices a full problem into rank `rank`'s shard (copies; used by tests)."""
    Hkv = k_cache.shape[2]
    lo, hi = kv_head_range(rank, world_size, Hkv)
    qlo, qhi = q_head_range(rank, world_size, q.shape[-2], Hkv)
    return (q[..., qlo:qhi, :].contiguous(), k_cache[:, :, lo:hi].contiguous(),
            v_cache[:, :, lo:hi].contiguous())


def gather_heads(out_local, group=None):
    """All-gather every rank's [B, Hq/N, D] output into the full [B, Hq, D]."""
    world = dist.get_world_size(group)
    B, hq_local, D = out_local.shape
    buf = torch.empty((world * B, hq_local, D), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
    return buf.view(world, B, hq_local, D).permute(1, 0, 2, 3).reshape(B, world * hq_local, D)


class PeerFailure(RuntimeError):
    """A rank did not report for a step within the timeout."""

    def __init__(self, step, missing):
        self.step = step
        self.missing = list(missing)
        super().__init__(f"step {step}: no report from rank(s) {self.missing}")


class StepCheck:
    """Host-side liveness check between decode steps (no GPU involvement).

    Every rank calls `arrive(step)` before its next launch or collective; it records the
    rank's report in a key-value store (a torch.distributed TCPStore) and waits, at most
    `timeout_s`, for every other rank's report of the same step.  A rank that died or
    left between steps never reports, so the survivors raise PeerFailure naming it
    before they launch anything that would wait on it -- instead of blocking in the next
    collective until the process-group timeout.
    """

    def __init__(self, store, rank, world_size, timeout_s=10.0, prefix="pgqa"):
        self.store = store
        self.rank = rank
        self.world = world_size
        self.timeout_s = float(timeout_s)
        self.prefix = prefix

    def _key(self, step, rank):
        return f"{self.prefix}/step{step}/rank{rank}"

    def arrive(self, step):
        import datetime

        self.store.set(self._key(step, self.rank), "1")
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception:
            missing = [r for r in range(self.world) if not self.store.check([self._key(step, r)])]
            raise PeerFailure(step, missing) from None
