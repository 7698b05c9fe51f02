"""GPU parity of the MeshGraphNet message-passing kernels (graphmodel/mgn_dp.py:28-54): the edge
update with the node gather fused into the resident kernel's producer and the segment sum fused
into its epilogue, and the node update on [nf | aggregates], through the C ABI."""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O
from tests._util import load_golden, u16_to
from tests.golden.make_golden import layer_params

pytestmark = pytest.mark.gpu


def _ln(seed):
    g = torch.Generator().manual_seed(seed)
    return (1 + 0.1 * torch.randn(128, generator=g)).half(), (0.1 * torch.randn(128, generator=g)).half()


def _graph(n_nodes, n_edges, seed):
    g = torch.Generator().manual_seed(seed)
    nf = torch.randn(n_nodes, 128, generator=g).half()
    ef = torch.randn(n_edges, 128, generator=g).half()
    srcs = torch.randint(0, n_nodes, (n_edges,), generator=g)
    dsts = torch.randint(0, n_nodes, (n_edges,), generator=g)
    return nf, ef, srcs, dsts


def _dev(ts, dev):
    return [None if t is None else t.to(dev) for t in ts]


def _edge(nf, ef, srcs, dsts, layers, ln, dev, agg=None):
    (w1, b1), (w2, b2), (w3, b3) = [(w.to(dev), b.to(dev)) for w, b in layers]
    out = torch.full((ef.shape[0], 128), float("nan"), dtype=torch.float16, device=dev)
    cuda_ext.mgn_edge_update_out(nf.to(dev), ef.to(dev), srcs.to(dev), dsts.to(dev), w1, b1, w2, b2,
                                 w3, b3, *_dev(ln, dev), out, agg=agg)
    torch.cuda.synchronize()
    return out


def _node(nf, aggs, layers, ln, dev):
    (w1, b1), (w2, b2), (w3, b3) = [(w.to(dev), b.to(dev)) for w, b in layers]
    out = cuda_ext.mgn_node_update(nf.to(dev), [a.to(dev) for a in aggs], w1, b1, w2, b2, w3, b3,
                                   *_dev(ln, dev))
    torch.cuda.synchronize()
    return out.float().cpu()


def _check(out, ref):
    r = O.compare(out, ref)
    assert r["ok"], r


def test_golden_message_passing_step(cuda_dev):
    g = load_golden("mgn_graph_step")
    seed = int(g["seed"])
    le = layer_params(seed + 1, [384, 128, 128, 128])
    lnode = layer_params(seed + 2, [256, 128, 128, 128])
    nf, ef = u16_to(g["nf"], torch.float16), u16_to(g["ef"], torch.float16)
    srcs, dsts = torch.from_numpy(g["srcs"]), torch.from_numpy(g["dsts"])
    lne = (u16_to(g["edge_gamma"], torch.float16), u16_to(g["edge_beta"], torch.float16))
    lnn = (u16_to(g["node_gamma"], torch.float16), u16_to(g["node_beta"], torch.float16))
    agg = torch.zeros(nf.shape[0], 128, device=cuda_dev)
    y_edge = _edge(nf, ef, srcs, dsts, le, lne, cuda_dev, agg=agg)
    _check(y_edge.float().cpu(), torch.from_numpy(g["y_edge"]))
    torch.testing.assert_close(agg.cpu(), torch.from_numpy(g["agg"]), atol=4e-3, rtol=2e-3)
    _check(_node(nf, [agg], lnode, lnn, cuda_dev), torch.from_numpy(g["y_node"]))


@pytest.mark.parametrize("n_nodes,n_edges", [(1, 1), (7, 129), (300, 5000), (4096, 65536 + 300)])
def test_edge_update_vs_oracle(cuda_dev, n_nodes, n_edges):
    nf, ef, srcs, dsts = _graph(n_nodes, n_edges, n_nodes + n_edges)
    layers = layer_params(5 + n_nodes % 13, [384, 128, 128, 128])
    ln = _ln(n_edges)
    agg = torch.zeros(n_nodes, 128, device=cuda_dev)
    out = _edge(nf, ef, srcs, dsts, layers, ln, cuda_dev, agg=agg)
    outc = out.float().cpu()
    n = min(n_edges, 4096)
    for sl in ([slice(0, n)] + ([slice(n_edges - n, n_edges)] if n_edges > n else [])):
        _check(outc[sl], O.mgn_edge_update(nf, ef[sl], srcs[sl], dsts[sl], layers, ln))
    # the fused segment sum equals the sum of the stored rows (fp32, any order)
    ref_agg = O.mgn_aggregate(out.cpu(), dsts, n_nodes)
    torch.testing.assert_close(agg.cpu(), ref_agg, atol=1e-3, rtol=1e-4)


def test_edge_update_without_aggregate_and_accumulation(cuda_dev):
    nf, ef, srcs, dsts = _graph(50, 1000, 3)
    layers = layer_params(9, [384, 128, 128, 128])
    ln = (None, None)
    out = _edge(nf, ef, srcs, dsts, layers, ln, cuda_dev)
    # NULL gamma / beta: LayerNorm with gamma = 1, beta = 0
    ident = (torch.ones(128), torch.zeros(128))
    _check(out.float().cpu(), O.mgn_edge_update(nf, ef, srcs, dsts, layers, ident))
    # accumulation onto existing contents: two calls add up
    agg = torch.ones(50, 128, device=cuda_dev)
    _edge(nf, ef, srcs, dsts, layers, ln, cuda_dev, agg=agg)
    _edge(nf, ef, srcs, dsts, layers, ln, cuda_dev, agg=agg)
    ref = 1 + 2 * O.mgn_aggregate(out.cpu(), dsts, 50)
    torch.testing.assert_close(agg.cpu(), ref, atol=2e-3, rtol=1e-4)


def test_bad_index_reads_zero_and_reports(cuda_dev):
    """An index outside [0, n_nodes) reads a zero node row, stays out of the aggregate and sets
    device status 0x600; nothing faults."""
    nf, ef, srcs, dsts = _graph(20, 300, 4)
    layers = layer_params(10, [384, 128, 128, 128])
    ln = _ln(1)
    dev_index = cuda_dev.index if cuda_dev.index is not None else 0
    L.device_status(dev_index, clear=True)
    bad_src, bad_dst = srcs.clone(), dsts.clone()
    bad_src[7] = 20 + 5
    bad_dst[11] = -3
    agg = torch.zeros(20, 128, device=cuda_dev)
    out = _edge(nf, ef, bad_src, bad_dst, layers, ln, cuda_dev, agg=agg).float().cpu()
    assert L.device_status(dev_index, clear=True) == 0x600
    nf_z = torch.cat([nf, torch.zeros(1, 128, dtype=nf.dtype)])  # row 20: the zero row
    s2, d2 = bad_src.clone(), bad_dst.clone()
    s2[7], d2[11] = 20, 20
    _check(out, O.mgn_edge_update(nf_z, ef, s2, d2, layers, ln))
    keep = torch.ones(300, dtype=torch.bool)
    keep[11] = False
    ref_agg = O.mgn_aggregate(out.half()[keep], bad_dst[keep], 20)
    torch.testing.assert_close(agg.cpu(), ref_agg, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("n_sets,n", [(1, 1), (1, 300), (1, 70000), (2, 129), (2, 20000)])
def test_node_update_vs_oracle(cuda_dev, n_sets, n):
    g = torch.Generator().manual_seed(n * 3 + n_sets)
    nf = torch.randn(n, 128, generator=g).half()
    aggs = [torch.randn(n, 128, generator=g) * 3 for _ in range(n_sets)]
    layers = layer_params(20 + n_sets, [128 * (1 + n_sets), 128, 128, 128])
    ln = _ln(n_sets)
    out = _node(nf, aggs, layers, ln, cuda_dev)
    k = min(n, 4096)
    _check(out[:k], O.mgn_node_update(nf[:k], [a[:k] for a in aggs], layers, ln))
    if n > k:
        _check(out[-k:], O.mgn_node_update(nf[-k:], [a[-k:] for a in aggs], layers, ln))


def test_shape_errors(cuda_dev):
    nf, ef, srcs, dsts = _graph(10, 64, 2)
    layers = layer_params(3, [384, 128, 128, 128])
    (w1, b1), (w2, b2), (w3, b3) = [(w.to(cuda_dev), b.to(cuda_dev)) for w, b in layers]
    nf, ef, srcs, dsts = _dev((nf, ef, srcs, dsts), cuda_dev)
    with pytest.raises(RuntimeError):
        cuda_ext.mgn_edge_update(nf, ef, srcs.int(), dsts, w1, b1, w2, b2, w3, b3, None, None)
    with pytest.raises(RuntimeError):
        cuda_ext.mgn_edge_update(nf, ef, srcs[:10], dsts, w1, b1, w2, b2, w3, b3, None, None)
    with pytest.raises(RuntimeError):
        cuda_ext.mgn_edge_update(nf, ef, srcs, dsts, w2, b1, w2, b2, w3, b3, None, None)
    with pytest.raises(RuntimeError):
        cuda_ext.mgn_node_update(nf, [], w1, b1, w2, b2, w3, b3, None, None)
    e = cuda_ext.mgn_edge_update(nf, ef[:0], srcs[:0], dsts[:0], w1, b1, w2, b2, w3, b3, None, None)
    assert e.shape == (0, 128)


def test_bench_workload_step(cuda_dev):
    """The bench's mgn_mp step (edge update with gather and segment sum, then node update) through
    cuda_ext.run_workload_out, against the oracle on the same packed input."""
    from gpu_pipes_b200 import workloads as W

    w = W.WORKLOADS["mgn_mp"].with_m(65536)
    x = W.make_input(w, 0, w.m)
    layers, ln = W.make_weights(w)
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=cuda_dev)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = tuple(t.to(cuda_dev) for t in ln)
    for _ in range(2):  # the aggregate is re-zeroed on every step
        cuda_ext.run_workload_out(w, x.to(cuda_dev), wd, lnd, out)
    torch.cuda.synchronize()
    ref = O.workload_forward(w, x, layers, ln).reshape(-1)
    got = out.float().cpu().reshape(-1)
    m, n = w.m, w.m // 16
    _check(got[:m * 128].view(m, 128), ref[:m * 128].view(m, 128))
    _check(got[m * 128:].view(n, 128), ref[m * 128:].view(n, 128))
