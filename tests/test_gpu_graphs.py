"""The engine inside CUDA graphs (gpu).

A layer step — a decode-shaped fused linear (split-K, its counters reset by
the kernel itself), the gated dual GEMM and a tensor-core fused linear with
residual — is captured once into a CUDA graph and replayed with new inputs
copied into the captured buffers; every replay must equal the eager result
bit for bit.  No host work happens at replay, so the launches cost only their
device time.
"""
import pytest
import torch

from deepx_op_gpukernelcompiler_b200 import _native as nat
from deepx_op_gpukernelcompiler_b200 import fused_gated_linear, fused_linear

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_graph_replay_matches_eager():
    torch.manual_seed(0)
    # H = 5120: 20 tiles of 256 columns, so the first launch is the decode
    # kernel with each tile's K range split over a cluster of 4 CTAs.
    M, K, H, N = 16, 1024, 5120, 768
    bf = torch.float16
    plans = []
    W1 = (torch.randn(K, H, device=DEV) / K ** 0.5).to(bf)
    b1 = (torch.rand(H, device=DEV) * 0.2 - 0.1).to(bf)
    Wg = (torch.randn(H, N, device=DEV) / H ** 0.5).to(bf)
    Wu = (torch.randn(H, N, device=DEV) / H ** 0.5).to(bf)
    bg = (torch.rand(N, device=DEV) * 0.2 - 0.1).to(bf)
    bu = (torch.rand(N, device=DEV) * 0.2 - 0.1).to(bf)
    W2 = (torch.randn(512, 640, device=DEV) / 512 ** 0.5).to(bf)
    b2 = (torch.rand(640, device=DEV) * 0.2 - 0.1).to(bf)
    x_static = torch.randn(M, K, device=DEV).to(bf)
    r_static = torch.randn(384, 512, device=DEV).to(bf)
    res_static = torch.randn(384, 640, device=DEV).to(bf)

    def step():
        h = fused_linear(x_static, W1, b1, "gelu_erf")
        plans.append(nat.last_launch_plan())
        g = fused_gated_linear(h, Wg, Wu, bg, bu, "silu")
        plans.append(nat.last_launch_plan())
        y = fused_linear(r_static, W2, b2, "silu", residual=res_static)
        plans.append(nat.last_launch_plan())
        return h, g, y

    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up outside capture: workspaces, tensor maps
            step()
    torch.cuda.current_stream(DEV).wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        h_out, g_out, y_out = step()
    assert plans[-3].startswith("decode ") and "max_seg=1 " not in plans[-3], plans[-3]
    assert plans[-2].startswith("decode_gated"), plans[-2]
    assert plans[-1].startswith("umma"), plans[-1]

    for rep in range(3):
        x_new = torch.randn(M, K, device=DEV).to(bf)
        r_new = torch.randn(384, 512, device=DEV).to(bf)
        res_new = torch.randn(384, 640, device=DEV).to(bf)
        x_static.copy_(x_new)
        r_static.copy_(r_new)
        res_static.copy_(res_new)
        graph.replay()
        torch.cuda.synchronize()
        h_ref = fused_linear(x_new, W1, b1, "gelu_erf")
        g_ref = fused_gated_linear(h_ref, Wg, Wu, bg, bu, "silu")
        y_ref = fused_linear(r_new, W2, b2, "silu", residual=res_new)
        torch.cuda.synchronize()
        assert torch.equal(h_out, h_ref), f"replay {rep}: decode linear differs"
        assert torch.equal(g_out, g_ref), f"replay {rep}: gated differs"
        assert torch.equal(y_out, y_ref), f"replay {rep}: tensor-core linear differs"
    assert nat.device_status(torch.cuda.current_stream(DEV).cuda_stream) == 0
