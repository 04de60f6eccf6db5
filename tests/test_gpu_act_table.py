"""The GELU / SiLU lookup tables are filled on the first large call per device. A call made
while its stream is being captured into a CUDA graph before that cannot fill them (the fill
synchronises), so it must take the table-free kernel -- with the same results. This needs a
process whose tables are still empty, hence the child process.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1] + "/anima.cu_b200", sys.argv[1] + "/oracle"]
import torch, anima_b200, refkernels
R = refkernels.load_reference()
torch.cuda.set_device(0)
n = 1 << 21
x = (torch.randn(n, device="cuda") * 3).to(torch.bfloat16).view(torch.int16)
for op in ("gelu_tanh", "silu"):
    want = torch.empty_like(x)
    getattr(R, op + "_bf16")(x.data_ptr(), want.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    got_graph, got_eager = torch.empty_like(x), torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):  # first call of the process: captured, table empty
            getattr(anima_b200, op)(x, got_graph, n, s)
        g.replay()
    s.synchronize()
    getattr(anima_b200, op)(x, got_eager, n)  # fills the table, then looks up
    g.replay()  # the captured table-free launch again, now beside a filled table
    torch.cuda.synchronize()
    assert torch.equal(got_graph, want), op + ": captured first call differs from the reference"
    assert torch.equal(got_eager, want), op + ": table path differs from the reference"
    del g
print("ok")
"""


def test_first_call_inside_graph_capture():
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
