"""The decode captured in a CUDA graph (caller-owned workspace, programmatic dependent
launch edges) replays with the same results as eager calls.

A graph bakes in the pointers, shapes and the tensor maps of the captured call; new
inputs are copied into the same buffers before each replay.  The fused combine's arrival
counters must return to zero at the end of every replay, or the next replay would merge
early, so several replays are compared bit for bit with eager calls.
"""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import inputs, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["c1", "c3"])
def test_graph_replay_matches_eager(name, cuda_device):
    inp = inputs.baseline_config(name).to(cuda_device)
    B, Hq, _ = inp.q.shape
    ws = torch.zeros(ops.lib().pgqa_workspace_size(B, Hq, inp.num_heads_k, 128, inp.page_size),
                     dtype=torch.uint8, device=cuda_device)
    q = inp.q.clone()
    out = torch.empty_like(q)

    def call():
        pgqa.decode(q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale,
                    out=out, workspace=ws)

    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        call()                                    # warm-up: device info, smem attribute
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    torch.cuda.synchronize(cuda_device)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
        call()                                    # two launches: the PDL edge inside the graph

    g = torch.Generator(device=cuda_device).manual_seed(3)
    for step in range(4):
        q.copy_(torch.randn(q.shape, generator=g, device=cuda_device).to(q.dtype))
        graph.replay()
        torch.cuda.synchronize(cuda_device)
        got = out.clone()
        expect = pgqa.decode(q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale,
                             workspace=ws)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(got, expect), f"{name}: replay {step} differs from eager"
    del graph
