"""CUDA-graph capture of the library's calls: one step is captured after an eager warm-up (so
workspaces are at size), then replayed on new inputs written into the captured buffers. Replays
must equal eager calls bit for bit, for every kernel family and composed block."""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from gpu_pipes_b200 import workloads as W

pytestmark = pytest.mark.gpu

CASES = [("mgn_node", 4096), ("mgn_edge", 3000), ("gc_edge", 2000), ("nerf", 2000),
         ("bert_ffn", 1024), ("dlrm_top", 2048), ("bert_addln", 1500), ("dlrm_interact", 1000),
         ("nerf_full", 1000), ("mgn_mp", 4096)]


@pytest.mark.parametrize("wname,m", CASES)
def test_capture_and_replay(cuda_dev, wname, m):
    w = W.WORKLOADS[wname].with_m(m)
    layers, ln = W.make_weights(w)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = None if ln is None else tuple(t.to(cuda_dev) for t in ln)
    xs = [W.make_input(w, r0, m).to(cuda_dev) for r0 in (0, 7 * m)]
    refs = []
    for x in xs:
        o = torch.empty(m, w.n_out, dtype=w.dtype, device=cuda_dev)
        cuda_ext.run_workload_out(w, x, wd, lnd, o)
        refs.append(o)
    torch.cuda.synchronize()
    x_cap = xs[0].clone()
    out_cap = torch.empty(m, w.n_out, dtype=w.dtype, device=cuda_dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cuda_ext.run_workload_out(w, x_cap, wd, lnd, out_cap)
    for x, ref in zip(xs[::-1], refs[::-1]):
        x_cap.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_cap, ref), wname
