"""GPU: the gated activation's first call is captured into a CUDA graph.

The table kernel reads a per-device activation table that the library
builds on first use.  A build recorded into a graph would run only at the
graph's replay, so an eager call between capture and replay must not find
the table marked built.  The check needs a process whose library has never
built the table, hence the child process."""

import subprocess
import sys

import pytest

from conftest import PKG_DIR, REPO

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import torch
import fast_moss_b200 as moss

def chain(x, bias, act):
    h = x + bias
    w = x.shape[-1] // 2
    gate, up = h[..., :w], h[..., w:]
    if act == "silu":
        a = torch.nn.functional.silu(gate)
    elif act == "gelu":
        a = torch.nn.functional.gelu(gate)
    else:
        a = torch.nn.functional.gelu(gate, approximate="tanh")
    return a * up

dev = torch.device("cuda:0")
g = torch.Generator().manual_seed(5)
# 2048 x 2048 outputs: large enough for the table kernel
x = torch.randn(2048, 4096, generator=g).to(dev, torch.bfloat16)
bias = (0.02 * torch.randn(4096, generator=g)).to(dev, torch.bfloat16)
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph):
    y_graph = moss.gated_activation(x, bias, "silu", gated=True)
# eager, before the graph has ever run
y_eager = moss.gated_activation(x, bias, "gelu", gated=True)
graph.replay()
# a graph captured after the table exists
graph2 = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph2):
    y_graph2 = moss.gated_activation(x, bias, "gelu_tanh", gated=True)
graph2.replay()
torch.cuda.synchronize()
for y, act in ((y_graph, "silu"), (y_eager, "gelu"), (y_graph2, "gelu_tanh")):
    ref = chain(x, bias, act)
    bad = int((y.view(torch.int16) != ref.view(torch.int16)).sum())
    assert bad == 0, (act, bad)
print("ok")
"""


def test_first_gate_call_inside_a_graph_capture(cuda_device):
    r = subprocess.run([sys.executable, "-c", CHILD, REPO, PKG_DIR], capture_output=True, text=True,
                       timeout=600, cwd=REPO)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
