"""KV-head sharding: head ranges, shard slicing and the output all-gather.

world_size-2 runs use `gloo` on CPU ranks (host logic; each rank decodes its shard with
the oracle); the NCCL variant runs the CUDA library on 2 GPUs when they are present.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

from mx_flash_attn_kernel_opt__b200 import inputs, sharding

HERE = os.path.dirname(os.path.abspath(__file__))


def test_head_ranges_partition_heads():
    for world in (1, 2, 4, 8):
        got = [sharding.kv_head_range(r, world, 8) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
        q = [sharding.q_head_range(r, world, 64, 8) for r in range(world)]
        assert q[-1][1] == 64 and all(h - l == 64 // world for l, h in q)
    with pytest.raises(ValueError):
        sharding.kv_head_range(0, 3, 8)


def test_shard_tensors_match_generator_shards():
    full = inputs.baseline_config("c1")
    q, k, v = sharding.shard_tensors(full.q, full.k, full.v, 1, 4)
    assert tuple(q.shape) == (4, 8, 128) and k.shape[2] == 2
    assert torch.equal(k, full.k[:, :, 2:4])
    assert torch.equal(q, full.q[:, 8:16])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _torchrun(nproc, backend, timeout):
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(HERE, "shard_worker.py"), backend]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="2")
    return subprocess.run(cmd, capture_output=True, text=True, env=env)


def test_gloo_two_ranks_gather_matches_unsharded_oracle():
    r = _torchrun(2, "gloo", 240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "match=1.0000" in r.stdout


@pytest.mark.gpu
def test_nccl_two_gpus_gather_matches_unsharded_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    r = _torchrun(2, "nccl", 300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


def test_step_check_names_a_rank_that_left():
    """Failure detection on the host (gloo, CPU): rank 1 exits between steps; rank 0's
    StepCheck raises PeerFailure naming it within the 3 s limit, instead of waiting in
    the next all-gather.  Processes are started directly (not through torchrun, whose
    agent would stop the survivor when one worker exits)."""
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), OMP_NUM_THREADS="2")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "shard_worker.py"),
                                       "gloo-fail"], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for pr in procs:
        try:
            out, _ = pr.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            pr.kill()
            out, _ = pr.communicate()
        outs.append((pr.returncode, out))
    (rc0, out0), (rc1, out1) = outs
    assert rc1 == 5, out1[-2000:]
    assert rc0 == 0, out0[-2000:]
    assert "rank0 step 0 done" in out0
    assert "rank0 PEER_FAILURE step=1 missing=[1]" in out0, out0[-2000:]
