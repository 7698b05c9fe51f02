"""Back-to-back dependent calls on one stream, the case programmatic dependent launch must keep
correct: the chain kernels may start while the previous kernel of the stream drains, and must not
read its output or overwrite its input before it has completed.

Each case runs a ping-pong sequence (A -> B, B -> A, ...): call i reads what call i-1 wrote
(read after write) and overwrites what call i-1 read (write after read). The sequence is enqueued
without host synchronisation and compared bit for bit with the same sequence run with a device
synchronisation after every call; the first output is also checked against the CPU oracle.
"""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O

pytestmark = pytest.mark.gpu

STEPS = 6


@pytest.fixture(params=[0, 1], ids=["default", "other"])
def variant(request):
    L.set_kernel_variant(request.param)
    yield request.param
    L.set_kernel_variant(0)


def _params(widths, dtype, dev, seed, scale=None):
    g = torch.Generator().manual_seed(seed)
    ws, bs = [], []
    for k, n in zip(widths[:-1], widths[1:]):
        s = scale if scale is not None else (2.0 / k) ** 0.5
        ws.append((torch.randn(k, n, generator=g) * s).to(dtype))
        bs.append((torch.randn(n, generator=g) * 0.05).to(dtype))
    ga = (1.0 + 0.1 * torch.randn(widths[-1], generator=g)).to(dtype)
    be = (0.1 * torch.randn(widths[-1], generator=g)).to(dtype)
    return ws, bs, ga, be, [w.to(dev) for w in ws], [b.to(dev) for b in bs], ga.to(dev), be.to(dev)


def _ping_pong(call, x0, sync_each):
    a, b = x0.clone(), torch.empty_like(x0)
    first = None
    for i in range(STEPS):
        call(a, b)
        if sync_each:
            torch.cuda.synchronize()
        if i == 0:
            first = b.clone()
        a, b = b, a
    torch.cuda.synchronize()
    return first, a


def _run(call, x0):
    first_s, last_s = _ping_pong(call, x0, sync_each=True)
    first_p, last_p = _ping_pong(call, x0, sync_each=False)
    assert torch.equal(first_p, first_s)
    assert torch.equal(last_p, last_s)
    return first_p


def test_resident_chain_ping_pong(cuda_dev, variant):
    """MGN-shaped 128 -> 128 -> 128 -> 128 + LayerNorm (weight-resident kernel)."""
    m = 20000
    ws, bs, ga, be, wd, bd, gad, bed = _params([128, 128, 128, 128], torch.float16, cuda_dev, 11)
    x0 = torch.randn(m, 128, generator=torch.Generator().manual_seed(12)).to(torch.float16)
    acts = [L.ACT_RELU, L.ACT_RELU, L.ACT_NONE]

    def call(x, out):
        cuda_ext.fused_mlp_out(x, wd, bd, out, acts=acts, tail=L.TAIL_LAYERNORM, gamma=gad, beta=bed)

    first = _run(call, x0.to(cuda_dev))
    ref = O.chain_forward(x0.float(), [(w.float(), b.float()) for w, b in zip(ws, bs)], acts,
                          O.TAIL_LAYERNORM, ln=(ga.float(), be.float()))
    r = O.compare(first.float().cpu(), ref)
    assert r["ok"], r


def test_ffn_residual_ln_ping_pong(cuda_dev, variant):
    """The reference's BERT FFN, 128 -> 512 ReLU -> 128, + x, LayerNorm (TMEM-activation kernel,
    and the weight-streaming kernel as the other variant)."""
    m = 9000
    ws, bs, ga, be, wd, bd, gad, bed = _params([128, 512, 128], torch.float16, cuda_dev, 21, scale=0.05)
    x0 = torch.randn(m, 128, generator=torch.Generator().manual_seed(22)).to(torch.float16)

    def call(x, out):
        cuda_ext.bert_ffn_out(x, wd[0], bd[0], wd[1], bd[1], gad, bed, out)

    first = _run(call, x0.to(cuda_dev))
    ref = O.bert_ffn(x0.float(), [(w.float(), b.float()) for w, b in zip(ws, bs)], (ga.float(), be.float()),
                     act_id=L.ACT_RELU, ln_eps=1e-5)
    r = O.compare(first.float().cpu(), ref)
    assert r["ok"], r


def test_wide_gemm_chain_ping_pong(cuda_dev, variant):
    """BERT-large FFN, 1024 -> 4096 GELU -> 1024, + x, LayerNorm (GEMM launches through the
    workspace and the row LayerNorm; or the single-kernel chain)."""
    m = 1024
    ws, bs, ga, be, wd, bd, gad, bed = _params([1024, 4096, 1024], torch.bfloat16, cuda_dev, 31, scale=0.02)
    x0 = torch.randn(m, 1024, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)

    def call(x, out):
        cuda_ext.bert_ffn_out(x, wd[0], bd[0], wd[1], bd[1], gad, bed, out)

    first = _run(call, x0.to(cuda_dev))
    ref = O.bert_ffn(x0.float(), [(w.float(), b.float()) for w, b in zip(ws, bs)], (ga.float(), be.float()))
    r = O.compare(first.float().cpu(), ref)
    assert r["ok"], r


def test_weights_written_by_previous_call(cuda_dev, variant):
    """Call 1 writes the buffer that call 2 takes as its weight matrix (and call 3 its bias): the
    second call must not read its weights before the first has completed."""
    g = torch.Generator().manual_seed(41)
    a = (torch.randn(128, 128, generator=g) * 0.1).to(torch.float16).to(cuda_dev)
    wa = (torch.randn(128, 128, generator=g) * 0.1).to(torch.float16).to(cuda_dev)
    x2 = (torch.randn(4096, 128, generator=g) * 0.1).to(torch.float16).to(cuda_dev)
    ones = torch.ones(1, 128, dtype=torch.float16, device=cuda_dev)
    none = [L.ACT_NONE]

    def seq(sync_each):
        w = torch.zeros(128, 128, dtype=torch.float16, device=cuda_dev)
        bias = torch.zeros(1, 128, dtype=torch.float16, device=cuda_dev)
        out2 = torch.empty(4096, 128, dtype=torch.float16, device=cuda_dev)
        out3 = torch.empty(4096, 128, dtype=torch.float16, device=cuda_dev)
        cuda_ext.fused_mlp_out(a, [wa], [None], w, acts=none)
        if sync_each:
            torch.cuda.synchronize()
        cuda_ext.fused_mlp_out(x2, [w], [None], out2, acts=none)
        if sync_each:
            torch.cuda.synchronize()
        cuda_ext.fused_mlp_out(ones, [wa], [None], bias, acts=none)
        if sync_each:
            torch.cuda.synchronize()
        cuda_ext.fused_mlp_out(x2, [wa], [bias.view(128)], out3, acts=none)
        torch.cuda.synchronize()
        return w, out2, out3

    ref = seq(True)
    got = seq(False)
    for r, t in zip(ref, got):
        assert torch.equal(r, t)
    assert float(ref[1].float().abs().max()) > 0.0
