"""gp_fused_mlp_host: host buffers streamed in chunks through double-buffered device staging on
three streams. Results must be bit-identical to the device-buffer entry point."""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from gpu_pipes_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _device_result(w, x, wd, lnd, dev):
    out = torch.empty(x.shape[0], w.n_out, dtype=w.dtype, device=dev)
    cuda_ext.run_workload_out(w, x.to(dev), wd, lnd, out)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("wname,m,chunk", [("mgn_node", 300_000, 65536), ("mgn_node", 1000, 0),
                                           ("nerf", 70_001, 16384), ("gc_edge", 20_000, 4096),
                                           ("bert_ffn", 5000, 2048), ("dlrm_top", 9000, 0)])
def test_host_pipeline_matches_device_path(cuda_dev, wname, m, chunk):
    w = W.WORKLOADS[wname].with_m(m)
    x = W.make_input(w, 0, m)
    layers, ln = W.make_weights(w)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = None if ln is None else tuple(t.to(cuda_dev) for t in ln)
    ref = _device_result(w, x, wd, lnd, cuda_dev)
    x_host = x.pin_memory()
    out_host = torch.full((m, w.n_out), float("nan"), dtype=w.dtype).pin_memory()
    gamma, beta = lnd if lnd is not None else (None, None)
    cuda_ext.fused_mlp_host_out(x_host, [p[0] for p in wd], [p[1] for p in wd], out_host, acts=w.acts,
                                tail=w.tail, gamma=gamma, beta=beta, ln_eps=w.ln_eps,
                                skip_layer=w.skip_layer, chunk_rows=chunk)
    torch.cuda.current_stream(cuda_dev).synchronize()
    assert torch.equal(out_host, ref)


def test_host_pipeline_back_to_back_calls(cuda_dev):
    """Two calls in a row with different inputs reuse the staging; each result is its own."""
    w = W.WORKLOADS["mgn_node"].with_m(200_000)
    layers, ln = W.make_weights(w)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = tuple(t.to(cuda_dev) for t in ln)
    xs = [W.make_input(w, r0, w.m) for r0 in (0, 300_000)]
    refs = [_device_result(w, x, wd, lnd, cuda_dev) for x in xs]
    outs = [torch.empty(w.m, w.n_out, dtype=w.dtype).pin_memory() for _ in xs]
    pinned = [x.pin_memory() for x in xs]  # alive until the stream is synchronised
    for x, o in zip(pinned, outs):
        cuda_ext.run_workload_host(w, x, wd, lnd, o)
    torch.cuda.current_stream(cuda_dev).synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
