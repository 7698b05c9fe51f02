"""GPU parity of NeRF with view directions (apps/nerf_full, use_viewdirs=True, the reference's
pipelined shapes: x [M, 64], d [M, 32], out_r and out_rgb [M, 64], fp16) against the CPU oracle
and the reference model's golden output, through the C ABI."""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O
from tests._util import load_golden, u16_to
from tests.golden.make_golden import layer_params

pytestmark = pytest.mark.gpu

DIMS = [(64, 256), (256, 256), (256, 256), (256, 256), (256, 256), (320, 256), (256, 256),
        (256, 256), (256, 64), (256, 256), (288, 128), (128, 64)]


def _layers(seed):
    return [layer_params(seed + i, [k, n])[0] for i, (k, n) in enumerate(DIMS)]


def _golden_layers(g):
    gen = torch.Generator().manual_seed(int(g["seed"]))
    layers = []
    for k, n in zip(g["dims_in"], g["dims_out"]):
        s = int(torch.randint(0, 2**31 - 1, (1,), generator=gen))
        layers.append(layer_params(s, [int(k), int(n)])[0])
    return layers


def _run(x, d, layers, dev, drop_bias=()):
    ws = [w.to(dev) for w, _ in layers]
    bs = [None if i in drop_bias else b.to(dev) for i, (_, b) in enumerate(layers)]
    out_r = torch.full((x.shape[0], 64), float("nan"), dtype=torch.float16, device=dev)
    out_rgb = torch.full_like(out_r, float("nan"))
    cuda_ext.nerf_full_out(x.to(dev), d.to(dev), ws, bs, out_r, out_rgb)
    torch.cuda.synchronize()
    return out_r.float().cpu(), out_rgb.float().cpu()


def _check(out, ref):
    r = O.compare(out, ref)
    assert r["ok"], r


def test_golden_reference_model(cuda_dev):
    g = load_golden("nerf_full_viewdirs")
    layers = _golden_layers(g)
    x, d = u16_to(g["x"], torch.float16), u16_to(g["d"], torch.float16)
    out_r, out_rgb = _run(x, d, layers, cuda_dev)
    _check(out_r, torch.from_numpy(g["alpha"]))
    _check(out_rgb, torch.from_numpy(g["rgb"]))


@pytest.mark.parametrize("m", [1, 127, 300, 4101, 65536 + 77])
def test_ragged_vs_oracle(cuda_dev, m):
    layers = _layers(300 + m % 11)
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, 64, generator=g).half()
    d = torch.randn(m, 32, generator=g).half()
    out_r, out_rgb = _run(x, d, layers, cuda_dev)
    n = min(m, 2048)
    for sl in ([slice(0, n)] + ([slice(m - n, m)] if m > n else [])):
        a, rgb = O.nerf_full(x[sl], d[sl], layers)
        _check(out_r[sl], a)
        _check(out_rgb[sl], rgb)


def test_null_biases(cuda_dev):
    """NULL bias entries mean no bias: the bottleneck, w11 and w12 biases as well as a trunk one."""
    layers = _layers(17)
    drop = (2, 9, 10, 11)
    zeroed = [(w, torch.zeros_like(b) if i in drop else b) for i, (w, b) in enumerate(layers)]
    g = torch.Generator().manual_seed(5)
    m = 1000
    x = torch.randn(m, 64, generator=g).half()
    d = torch.randn(m, 32, generator=g).half()
    out_r, out_rgb = _run(x, d, layers, cuda_dev, drop_bias=drop)
    a, rgb = O.nerf_full(x, d, zeroed)
    _check(out_r, a)
    _check(out_rgb, rgb)


def test_view_dirs_reach_rgb_only(cuda_dev):
    """Changing d changes out_rgb and leaves out_r bit-identical."""
    layers = _layers(23)
    g = torch.Generator().manual_seed(9)
    m = 513
    x = torch.randn(m, 64, generator=g).half()
    d0 = torch.randn(m, 32, generator=g).half()
    d1 = torch.randn(m, 32, generator=g).half()
    r0, rgb0 = _run(x, d0, layers, cuda_dev)
    r1, rgb1 = _run(x, d1, layers, cuda_dev)
    assert torch.equal(r0, r1)
    assert not torch.equal(rgb0, rgb1)
    _check(rgb1, O.nerf_full(x, d1, layers)[1])


def test_allocating_form_and_errors(cuda_dev):
    layers = _layers(41)
    m = 257
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, 64, generator=g).half()
    d = torch.randn(m, 32, generator=g).half()
    ref_r, ref_rgb = _run(x, d, layers, cuda_dev)
    wb = []
    for w, b in layers:
        wb += [w.to(cuda_dev), b.to(cuda_dev)]
    out_r, out_rgb = cuda_ext.nerf_full(x.to(cuda_dev), d.to(cuda_dev), *wb)
    torch.cuda.synchronize()
    assert torch.equal(out_r.float().cpu(), ref_r)
    assert torch.equal(out_rgb.float().cpu(), ref_rgb)
    bad = list(wb)
    bad[20] = bad[20][:256]  # w11 with 256 rows instead of 288
    with pytest.raises(RuntimeError):
        cuda_ext.nerf_full(x.to(cuda_dev), d.to(cuda_dev), *bad)
    with pytest.raises(RuntimeError):
        cuda_ext.nerf_full(x.to(cuda_dev), d[:, :24].contiguous().to(cuda_dev), *wb)
    e_r = torch.empty(0, 64, dtype=torch.float16, device=cuda_dev)
    cuda_ext.nerf_full_out(x[:0].to(cuda_dev), d[:0].to(cuda_dev), wb[0::2], wb[1::2], e_r, e_r.clone())
