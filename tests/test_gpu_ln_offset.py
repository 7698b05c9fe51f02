"""LayerNorm statistics with a large per-row mean against a small spread.

A one-pass E[y^2] - mean^2 variance cancels catastrophically when |mean| is large next to the
row's standard deviation; the reference's LayerNorm is two-pass (common/layer_norm_v2.cuh:34-62)
and so is torch.nn.LayerNorm. These cases put the pre-LayerNorm rows at mean 64 +- 32 (different
per row) with a spread of about 0.3, and use gamma != 1, beta != 0, so any cancellation in the
fused kernels' statistics shows up against the fp32 oracle.

Covered tails:
  * the weight-resident kernel's LayerNorm (MeshGraphNet edge and node MLPs, both kernel forms),
  * the weight-streaming kernel's LayerNorm (GraphCast, CTA pair, bf16),
  * the residual LayerNorm tails: the reference's BERT FFN 128 -> 512 -> 128 (offset from the
    FFN output) and the BERT attention-output block (offset from the residual x),
  * the BERT-large GEMM chain's row LayerNorm.
Tolerance: the north-star max |err| <= 2e-2 and relative L2 <= 5e-3 against the fp32 oracle.
"""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O

pytestmark = pytest.mark.gpu


def _lin(g, k, n, scale, dtype):
    w = (torch.randn(k, n, generator=g) * scale).to(dtype)
    b = (torch.randn(n, generator=g) * 0.01).to(dtype)
    return w, b


def offset_last_layer(g, k, n, dtype, spread=0.02, per_row=0.5, base=64.0):
    """Last layer [K, N] whose output rows have mean ~ base + per_row * sum(h) and a small
    spread: W = spread * N(0,1) + per_row (a common column added to every output), b = base."""
    w = (torch.randn(k, n, generator=g) * spread + per_row).to(dtype)
    b = (torch.full((n,), base) + torch.randn(n, generator=g) * 0.01).to(dtype)
    return w, b


def ln_params(g, n, dtype):
    """gamma != 1, beta != 0. For bf16 outputs they stay small enough that |out| < 8: from 8 up,
    the bf16 rounding of the stored result alone (half a unit in the last place, 2^-5) exceeds
    the 2e-2 bound."""
    sg, sb = (0.5, 0.3) if dtype == torch.float16 else (0.1, 0.05)
    return ((1.0 + sg * torch.randn(n, generator=g)).to(dtype),
            (sb * torch.randn(n, generator=g)).to(dtype))


def mgn_offset_case(m, k0, seed=11):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k0, generator=g).half()
    l1 = _lin(g, k0, 128, k0 ** -0.5, torch.float16)
    l2 = _lin(g, 128, 128, 128 ** -0.5, torch.float16)
    # h2 >= 0 (ReLU) with sum ~ 50 per row: per_row = 0.6 / 128 * ... gives offsets of tens
    l3 = offset_last_layer(g, 128, 128, torch.float16, spread=0.02, per_row=0.6)
    return x, [l1, l2, l3], ln_params(g, 128, torch.float16)


def gc_offset_case(m, seed=12):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, 1536, generator=g).bfloat16()
    l1 = _lin(g, 1536, 512, 1536 ** -0.5, torch.bfloat16)
    l2 = offset_last_layer(g, 512, 512, torch.bfloat16, spread=0.01, per_row=0.15)
    return x, [l1, l2], ln_params(g, 512, torch.bfloat16)


def resid_offset_x(g, m, h, dtype):
    """x rows with mean 64 +- 32 (per row) and spread 0.3."""
    off = 64.0 + 32.0 * (2 * torch.rand(m, 1, generator=g) - 1)
    return (off + 0.3 * torch.randn(m, h, generator=g)).to(dtype)


def _pre_ln(x, layers, acts, resid=False):
    h = x.float()
    for i, (w, b) in enumerate(layers):
        h = O.linear(h, w.float(), b.float())
        if i < len(layers) - 1:
            h = O.act(acts[i], h)
    return h + x.float() if resid else h


def _check_ratio(pre, lo=50.0):
    """The case is only meaningful if |mean| / std is large for every row."""
    mean = pre.mean(-1)
    std = pre.std(-1, unbiased=False)
    assert float((mean.abs() / std).min()) > lo, float((mean.abs() / std).min())
    assert float(mean.std()) > 1.0  # the offset differs between rows


def _close(out, ref, what):
    r = O.compare(out.float().cpu(), ref)
    assert r["ok"], f"{what}: {r}"


@pytest.fixture(params=[0, 1], ids=["default", "other"])
def variant(request):
    L.set_kernel_variant(request.param)
    yield request.param
    L.set_kernel_variant(0)


@pytest.mark.parametrize("k0,m", [(384, 65_536 + 77), (256, 40_000)])
def test_resident_layernorm_offset_rows(cuda_dev, variant, k0, m):
    x, layers, (ga, be) = mgn_offset_case(m, k0)
    _check_ratio(_pre_ln(x[:4096], layers, [O.ACT_RELU] * 2))
    d = [t.to(cuda_dev) for t in [x] + [t for p in layers for t in p] + [ga, be]]
    out = cuda_ext.mgn_fullmlp(*d)
    torch.cuda.synchronize()
    _close(out, O.mgn_mlp(x, layers, (ga, be), 1e-5), f"mgn k0={k0}")


def test_stream_layernorm_offset_rows(cuda_dev):
    x, layers, (ga, be) = gc_offset_case(20_000)
    _check_ratio(_pre_ln(x[:2048], layers, [O.ACT_SILU]))
    (w0, b0), (w1, b1) = layers
    d = [t.to(cuda_dev) for t in (x, w0, b0, w1, b1, ga, be)]
    out = cuda_ext.gc_edges(*d, act=L.ACT_SILU)
    torch.cuda.synchronize()
    _close(out, O.gc_edges(x, layers, (ga, be), O.ACT_SILU, 1e-5), "gc_edges")


def ffn_offset_case(g, m, h, f, dtype, w1_scale, per_row):
    """Residual-tail FFN case whose pre-LayerNorm rows x + FFN(x) sit at a large, per-row mean.
    The mean comes from the second layer: W2 = per_row + 0.002 N(0,1) adds per_row * sum(h) (h >=
    0 after ReLU/GELU, different for every row) to every column, so the rows keep the spread of x
    (0.3) while bf16 inputs stay finely resolved (a large offset in x itself would quantise a
    bf16 row to a few distinct values)."""
    x = (0.3 * torch.randn(m, h, generator=g)).to(dtype)
    w1 = (torch.randn(h, f, generator=g) * w1_scale).to(dtype)
    b1 = (torch.randn(f, generator=g) * 0.01).to(dtype)
    w2 = (torch.randn(f, h, generator=g) * 0.002 + per_row).to(dtype)
    b2 = torch.zeros(h).to(dtype)
    return x, [(w1, b1), (w2, b2)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_residual_layernorm_offset_rows_bert128(cuda_dev, dtype):
    g = torch.Generator().manual_seed(13)
    x, layers = ffn_offset_case(g, 30_000, 128, 512, dtype, 0.09, 1.5)
    ga, be = ln_params(g, 128, dtype)
    _check_ratio(_pre_ln(x[:4096], layers, [O.ACT_RELU], resid=True))
    (w1, b1), (w2, b2) = layers
    out = cuda_ext.bert_ffn(*[t.to(cuda_dev) for t in (x, w1, b1, w2, b2, ga, be)])
    torch.cuda.synchronize()
    _close(out, O.bert_ffn(x, layers, (ga, be), O.ACT_RELU, 1e-5), "bert_ffn 128")


def test_residual_layernorm_offset_rows_addln(cuda_dev):
    g = torch.Generator().manual_seed(14)
    m = 20_000
    x = resid_offset_x(g, m, 128, torch.float16)
    attn = (0.3 * torch.randn(m, 128, generator=g)).half()
    layers = [_lin(g, 128, 128, 0.01, torch.float16), _lin(g, 128, 512, 0.09, torch.float16),
              _lin(g, 512, 128, 0.05, torch.float16)]
    (w0, b0), _, _ = layers
    _check_ratio((attn.float() @ w0.float() + b0.float() + x.float())[:4096])
    ln0, ln2 = ln_params(g, 128, torch.float16), ln_params(g, 128, torch.float16)
    # the offset rows meet the first LayerNorm (h = LN0(attn W0 + b0 + x)); h is kept in 16 bits
    # between the two launches, so the second LayerNorm runs on ordinary unit-scale rows
    (w0, b0), (w1, b1), (w2, b2) = layers
    d = [t.to(cuda_dev) for t in (attn, x, w0, b0, w1, b1, w2, b2, ln0[0], ln0[1], ln2[0], ln2[1])]
    out = cuda_ext.bert_addln_ffn(*d)
    torch.cuda.synchronize()
    _close(out, O.bert_addln_ffn(attn, x, layers, ln0, ln2), "bert_addln_ffn")


def test_gemm_chain_layernorm_offset_rows_bert_large(cuda_dev):
    g = torch.Generator().manual_seed(15)
    x, layers = ffn_offset_case(g, 2_048, 1024, 4096, torch.bfloat16, 0.03, 0.6)
    ga, be = ln_params(g, 1024, torch.bfloat16)
    _check_ratio(_pre_ln(x[:1024], layers, [O.ACT_GELU_TANH], resid=True))
    (w1, b1), (w2, b2) = layers
    out = cuda_ext.bert_ffn(*[t.to(cuda_dev) for t in (x, w1, b1, w2, b2, ga, be)])
    torch.cuda.synchronize()
    _close(out, O.bert_ffn(x, layers, (ga, be), O.ACT_GELU_TANH, 1e-12), "bert-large ffn")
