"""GPU parity of the BERT attention-output block (apps/bert_addln_ffn, H = 128, ff = 512, fp16)
against the CPU oracle and the reference model's golden output, through the C ABI."""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O
from tests._util import load_golden, u16_to
from tests.golden.make_golden import layer_params

pytestmark = pytest.mark.gpu


def _params(seed, dev):
    layers = layer_params(seed, [128, 128]) + layer_params(seed + 1, [128, 512, 128])
    g = torch.Generator().manual_seed(seed + 7)
    lns = [((1 + 0.1 * torch.randn(128, generator=g)).half(), (0.1 * torch.randn(128, generator=g)).half())
           for _ in range(2)]
    return layers, lns


def _run(attn, x, layers, lns, dev):
    (w0, b0), (w1, b1), (w2, b2) = [(w.to(dev), b.to(dev)) for w, b in layers]
    (ga0, be0), (ga2, be2) = [(g.to(dev), b.to(dev)) for g, b in lns]
    out = torch.empty(x.shape[0], 128, dtype=torch.float16, device=dev)
    cuda_ext.bert_addln_ffn_out(attn.to(dev), x.to(dev), w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2, out)
    torch.cuda.synchronize()
    return out.float().cpu()


def test_golden_reference_model(cuda_dev):
    g = load_golden("bert_addln_ffn_128")
    seed = int(g["seed"])
    layers = layer_params(seed, [128, 128]) + layer_params(seed + 1, [128, 512, 128])
    attn, x = u16_to(g["attn"], torch.float16), u16_to(g["x"], torch.float16)
    lns = [(u16_to(g["ln0_gamma"], torch.float16), u16_to(g["ln0_beta"], torch.float16)),
           (u16_to(g["ln2_gamma"], torch.float16), u16_to(g["ln2_beta"], torch.float16))]
    out = _run(attn, x, layers, lns, cuda_dev)
    r = O.compare(out, torch.from_numpy(g["y"]))
    assert r["ok"], r


@pytest.mark.parametrize("m", [1, 129, 300, 64 * 512])
def test_ragged_vs_oracle(cuda_dev, m):
    layers, lns = _params(70 + m % 7, cuda_dev)
    g = torch.Generator().manual_seed(m)
    attn = torch.randn(m, 128, generator=g).half()
    x = torch.randn(m, 128, generator=g).half()
    out = _run(attn, x, layers, lns, cuda_dev)
    n = min(m, 4096)
    ref = O.bert_addln_ffn(attn[:n], x[:n], layers, lns[0], lns[1])
    r = O.compare(out[:n], ref)
    assert r["ok"], r
    if m > n:
        ref = O.bert_addln_ffn(attn[-n:], x[-n:], layers, lns[0], lns[1])
        r = O.compare(out[-n:], ref)
        assert r["ok"], r


def test_allocating_form_and_shape_errors(cuda_dev):
    layers, lns = _params(5, cuda_dev)
    m = 257
    g = torch.Generator().manual_seed(3)
    attn = torch.randn(m, 128, generator=g).half()
    x = torch.randn(m, 128, generator=g).half()
    ref = _run(attn, x, layers, lns, cuda_dev)
    (w0, b0), (w1, b1), (w2, b2) = [(w.to(cuda_dev), b.to(cuda_dev)) for w, b in layers]
    (ga0, be0), (ga2, be2) = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in lns]
    y = cuda_ext.bert_addln_ffn(attn.to(cuda_dev), x.to(cuda_dev), w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2)
    torch.cuda.synchronize()
    assert torch.equal(y.float().cpu(), ref)
    with pytest.raises(RuntimeError):
        cuda_ext.bert_addln_ffn(attn.to(cuda_dev), x.to(cuda_dev), w0[:64], b0, w1, b1, w2, b2,
                                ga0, be0, ga2, be2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_reference_bert_ffn_128(cuda_dev, dtype):
    """The reference's own small BERT FFN (apps/bert_ffn: 128 -> 512 ReLU -> 128, + x, LN eps
    1e-5) through cuda_ext.bert_ffn; the bf16 case against the reference model's golden output."""
    if dtype == torch.bfloat16:
        g = load_golden("bert_ffn_128")
        layers = layer_params(int(g["seed"]), [128, 512, 128], dtype=torch.bfloat16, init="normal002")
        x = u16_to(g["x"], torch.bfloat16)
        expected = torch.from_numpy(g["y"])
        ln = (torch.ones(128, dtype=dtype), torch.zeros(128, dtype=dtype))
    else:
        layers = layer_params(91, [128, 512, 128], dtype=dtype)
        gx = torch.Generator().manual_seed(92)
        x = torch.randn(5000, 128, generator=gx).to(dtype)
        ln = ((1 + 0.1 * torch.randn(128, generator=gx)).to(dtype), (0.1 * torch.randn(128, generator=gx)).to(dtype))
        expected = O.bert_ffn(x, layers, ln, act_id=O.ACT_RELU, ln_eps=1e-5)
    d = [t.to(cuda_dev) for wb in layers for t in wb]
    out = cuda_ext.bert_ffn(x.to(cuda_dev), *d, *[t.to(cuda_dev) for t in ln])
    torch.cuda.synchronize()
    r = O.compare(out.float().cpu(), expected)
    assert r["ok"], r
