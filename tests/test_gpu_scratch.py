"""Library scratch memory and CUDA graphs.

The library grows its scratch buffers (split-K partials, stream-K pieces, attention
partials) on demand, outside stream capture.  A graph captured earlier keeps the address
of the buffer that was current at capture, so an outgrown buffer must stay allocated:
these tests capture a GEMM, make a later call outgrow the scratch slot, and replay the
graph.  They run in a fresh process, where the slot starts empty, so the growth happens
whatever other tests ran before.
"""
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys
sys.path.insert(0, {repo!r})
import torch
from pilm_b200 import bindings, ckernel as ck

bindings.init()
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(3)


def w4(n, k):
    return (torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g),
            torch.rand((n, k // 128), device=dev, generator=g) * 0.01 + 1e-4)


# split schedule (4 tiles, 16 splits): fp32 partials in the split-K slot, its first use (16 MiB)
x1 = torch.randn((24, 4096), device=dev, generator=g).to(torch.bfloat16)
w1, s1 = w4(512, 4096)
y1 = torch.empty((24, 512), dtype=torch.bfloat16, device=dev)
ck.linear_w4a16g128_bf16(x1, w1, s1, out=y1)
torch.cuda.synchronize()
want = y1.clone()
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph):
    ck.linear_w4a16g128_bf16(x1, w1, s1, out=y1)
torch.cuda.synchronize()

# stream-K schedule (149 tiles): its cut-tile pieces (19.4 MB) outgrow the slot
x2 = torch.randn((24, 512), device=dev, generator=g).to(torch.bfloat16)
w2, s2 = w4(19000, 512)
y2 = ck.linear_w4a16g128_bf16(x2, w2, s2)
torch.cuda.synchronize()

# memory released to the driver now could be handed out again: take some and mark it
fill = [torch.full((1 << 22,), 7, dtype=torch.int32, device=dev) for _ in range(8)]
torch.cuda.synchronize()
for _ in range(2):
    y1.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y1, want), "graph replay after scratch growth changed the result"
assert all(bool((f == 7).all()) for f in fill), "graph replay wrote outside its buffers"
y2b = ck.linear_w4a16g128_bf16(x2, w2, s2)
torch.cuda.synchronize()
assert torch.equal(y2, y2b)
del graph
print("scratch ok")
"""


def test_graph_replays_after_scratch_growth():
    out = subprocess.run([sys.executable, "-c", SCRIPT.format(repo=str(REPO))], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    assert "scratch ok" in out.stdout
