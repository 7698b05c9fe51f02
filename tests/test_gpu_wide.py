"""GPU parity of the wide chains (BERT-large FFN with residual + LayerNorm, DLRM top MLP with the
sigmoid head) against the CPU oracle, through the C ABI. Row counts cross the chunk boundaries the
host uses (4,096 rows for BERT, 16,384 for DLRM top) and, on the single-kernel form, wrap its
rings of row blocks; full-size runs are checked on row samples."""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=[0, 1], ids=["default", "other"])
def variant(request):
    """Every case on both forms: layer by layer through the workspace, and the single-kernel
    chain with its intermediates in L2-sized rings (tile sequence with completion counters)."""
    L.set_kernel_variant(request.param)
    yield request.param
    L.set_kernel_variant(0)


def _run(w, dev):
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=dev)
    cuda_ext.run_workload_out(w, x.to(dev), [(a.to(dev), b.to(dev)) for a, b in layers],
                              None if ln is None else tuple(t.to(dev) for t in ln), out)
    torch.cuda.synchronize()
    return x, layers, ln, out


def _check(w, x, layers, ln, out, spans):
    for r0, n in spans:
        ref = O.workload_forward(w, x[r0:r0 + n], layers, ln)
        r = O.compare(out[r0:r0 + n].float().cpu(), ref)
        assert r["ok"], f"{w.name} rows {r0}+{n}: {r}"


@pytest.mark.parametrize("m", [1, 129, 4096 + 77, 9000])
def test_bert_ffn_ragged(cuda_dev, m):
    w = W.BERT_FFN.with_m(m)
    x, layers, ln, out = _run(w, cuda_dev)
    _check(w, x, layers, ln, out, [(0, m)])


def test_bert_ffn_full_size(cuda_dev):
    w = W.BERT_FFN
    x, layers, ln, out = _run(w, cuda_dev)
    _check(w, x, layers, ln, out, [(0, 2048), (8192 - 1024, 2048), (w.m - 2048, 2048)])


@pytest.mark.parametrize("m", [1, 255, 16384 + 5, 40000])
def test_dlrm_top_ragged(cuda_dev, m):
    w = W.DLRM_TOP.with_m(m)
    x, layers, ln, out = _run(w, cuda_dev)
    _check(w, x, layers, ln, out, [(0, m)])


def test_dlrm_top_full_size(cuda_dev):
    w = W.DLRM_TOP
    x, layers, ln, out = _run(w, cuda_dev)
    _check(w, x, layers, ln, out, [(0, 8192), (131072 - 4096, 8192), (w.m - 8192, 8192)])


def test_named_entry_points(cuda_dev):
    """cuda_ext.bert_ffn / cuda_ext.dlrm_topmlp (the reference's names) give the same rows."""
    w = W.BERT_FFN.with_m(300)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    d = [t.to(cuda_dev) for p in layers for t in p]
    out = cuda_ext.bert_ffn(x.to(cuda_dev), *d, *[t.to(cuda_dev) for t in ln], eps=1e-12)
    torch.cuda.synchronize()
    assert O.compare(out.float().cpu(), O.workload_forward(w, x, layers, ln))["ok"]
    w = W.DLRM_TOP.with_m(300)
    x = W.make_input(w)
    layers, _ = W.make_weights(w)
    d = [t.to(cuda_dev) for p in layers for t in p]
    out = cuda_ext.dlrm_topmlp(x.to(cuda_dev), *d)
    torch.cuda.synchronize()
    assert O.compare(out.float().cpu(), O.workload_forward(w, x, layers, None))["ok"]


def test_bert_ffn_gamma_beta_4_byte_aligned(cuda_dev):
    """gamma/beta need only 4-byte alignment: a copy at a 4-byte (not 8-byte) offset takes the
    LayerNorm kernel's scalar path and must give the same bits as the aligned one."""
    w = W.BERT_FFN.with_m(513)
    x, layers, ln, out = _run(w, cuda_dev)
    g, b = (t.to(cuda_dev) for t in ln)
    buf = torch.zeros(2 * (w.n_out + 4), dtype=g.dtype, device=cuda_dev)
    g_off = buf[2:2 + w.n_out]  # 4-byte offset from a 256-byte aligned base
    b_off = buf[w.n_out + 6:w.n_out + 6 + w.n_out]
    assert g_off.data_ptr() % 8 == 4 and b_off.data_ptr() % 8 == 4
    g_off.copy_(g)
    b_off.copy_(b)
    out2 = torch.empty_like(out)
    cuda_ext.run_workload_out(w, x.to(cuda_dev), [(a.to(cuda_dev), bb.to(cuda_dev)) for a, bb in layers],
                              (g_off, b_off), out2)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_chain_dependency_timeout_is_reported(cuda_dev, variant):
    """Single-kernel form only. Host-side fault injection drops every completion signal, so the
    later layers' dependency waits run out after 5 ms. The kernel exits cleanly, the status word
    reports it, and the next call on the same context is correct."""
    if variant != 1:
        pytest.skip("the single-kernel form only")
    w = W.DLRM_TOP.with_m(3000)
    x, layers, ln, _ = _run(w, cuda_dev)
    xd = x.to(cuda_dev)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=cuda_dev)
    assert L.device_status(0, clear=True) == 0
    try:
        L.set_timeout_ns(5_000_000)
        L.set_fault_injection(1)
        cuda_ext.run_workload_out(w, xd, wd, None, out)
        torch.cuda.synchronize()
    finally:
        L.set_fault_injection(0)
        L.set_timeout_ns(0)
    st = L.device_status(0, clear=True)
    assert st in (0x700, 0x100, 0x200, 0x300), hex(st)
    assert L.device_status(0) == 0
    out.zero_()
    cuda_ext.run_workload_out(w, xd, wd, None, out)
    torch.cuda.synchronize()
    _check(w, x, layers, ln, out, [(0, w.m)])
