"""Worker for the KV-head sharding tests (launched with world_size >= 2).

Each rank builds its shard (KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads) of a
seeded problem, decodes it -- the CUDA library on GPUs (backend nccl), the CPU oracle
on CPU ranks (backend gloo, host-logic test only) -- gathers the head slices with
sharding.gather_heads and, on rank 0, compares with the unsharded oracle.
"""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def failing_peer():
    """Host-side failure detection, CPU only: a 3-step decode loop over gloo ranks in
    which the last rank exits after step 0.  The survivors must name it through
    sharding.StepCheck before their next collective (printed as PEER_FAILURE)."""
    import datetime

    import torch
    import torch.distributed as dist

    from mx_flash_attn_kernel_opt__b200 import inputs, sharding
    from oracle import paged_decode_ref

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    store = dist.TCPStore("127.0.0.1", int(os.environ["MASTER_PORT"]) + 1, world,
                          is_master=(rank == 0), timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    check = sharding.StepCheck(store, rank, world, timeout_s=3.0)
    full = inputs.baseline_config("c1")
    q, k, v = sharding.shard_tensors(full.q, full.k, full.v, rank, world)
    for step in range(3):
        if rank == world - 1 and step == 1:
            print(f"rank{rank} leaving after step 0", flush=True)
            os._exit(5)  # between steps: nothing of this rank is in flight
        try:
            check.arrive(step)
        except sharding.PeerFailure as e:
            print(f"rank{rank} PEER_FAILURE step={e.step} missing={e.missing}", flush=True)
            os._exit(0)
        out = paged_decode_ref(q, k, v, full.block_table, full.seq_lens).to(torch.bfloat16)
        sharding.gather_heads(out)
        print(f"rank{rank} step {step} done", flush=True)
    os._exit(4)  # the failure was not detected


def main():
    import datetime

    import torch
    import torch.distributed as dist

    from mx_flash_attn_kernel_opt__b200 import inputs, sharding
    from oracle import match_stats, paged_decode_ref

    backend = sys.argv[1]
    if backend == "gloo-fail":
        failing_peer()
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    if backend == "nccl":
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    else:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    full = inputs.baseline_config("c1")
    lo, hi = sharding.kv_head_range(rank, world, full.num_heads_k)
    q, k, v = sharding.shard_tensors(full.q, full.k, full.v, rank, world)
    if backend == "nccl":
        import mx_flash_attn_kernel_opt__b200 as pgqa
        out = pgqa.decode(q.to(dev), k.to(dev), v.to(dev), full.block_table.to(dev),
                          full.seq_lens.to(dev), scale=full.scale)
    else:
        out = paged_decode_ref(q, k, v, full.block_table, full.seq_lens).to(torch.bfloat16)
    gathered = sharding.gather_heads(out)
    ok = torch.tensor([1], dtype=torch.int32, device=dev)
    if rank == 0:
        ref = paged_decode_ref(full.q, full.k, full.v, full.block_table, full.seq_lens)
        frac, outlier, maxd = match_stats(gathered.cpu(), ref)
        good = (not outlier) and frac >= 0.99 and torch.allclose(
            gathered.cpu().float(), ref, atol=1e-2, rtol=1e-2)
        print(f"rank0 gathered {tuple(gathered.shape)} match={frac:.4f} max={maxd:.3e}")
        ok[0] = int(good)
    dist.broadcast(ok, 0)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if int(ok[0]) == 1 else 3)


if __name__ == "__main__":
    main()
