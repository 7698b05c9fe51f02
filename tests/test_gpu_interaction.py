"""GPU parity of the DLRM feature interaction (graphmodel/dlrm.py:28-42) against the CPU oracle,
through the C ABI. The outputs are dot products stored in fp16 (the top MLP's input layout), so
the bound is element-wise relative: |gpu - oracle| <= 2e-3 |oracle| + 1e-3 (about 4 fp16 ulps)."""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(m, seed):
    g = torch.Generator().manual_seed(seed)
    bot = torch.relu(torch.randn(m, 128, generator=g)).mul(0.3).half()
    sparse = (torch.randn(m, 26, 128, generator=g) * 0.1).half()
    return bot, sparse


def _check(out, ref):
    d = (out.float().cpu() - ref).abs()
    bound = 2e-3 * ref.abs() + 1e-3
    assert bool((d <= bound).all()), f"max excess {(d - bound).max().item()}"


@pytest.mark.parametrize("m", [1, 3, 4, 5, 1000, 65536 + 3])
def test_interaction_vs_oracle(cuda_dev, m):
    bot, sparse = _inputs(m, m)
    out = cuda_ext.dlrm_interaction(bot.to(cuda_dev), sparse.to(cuda_dev))
    torch.cuda.synchronize()
    n = min(m, 4096)
    _check(out[:n], O.dlrm_interaction(bot[:n], sparse[:n]))
    if m > n:
        _check(out[-n:], O.dlrm_interaction(bot[-n:], sparse[-n:]))
    assert bool((out[:, 479] == 0).all())


def test_interaction_feeds_top_mlp(cuda_dev):
    """bottom output + embeddings -> interaction -> the DLRM top MLP, end to end on the GPU,
    against the oracle chain."""
    from gpu_pipes_b200 import workloads as W
    m = 700
    bot, sparse = _inputs(m, 11)
    z = cuda_ext.dlrm_interaction(bot.to(cuda_dev), sparse.to(cuda_dev))
    w = W.DLRM_TOP.with_m(m)
    layers, _ = W.make_weights(w)
    out = torch.empty(m, 1, dtype=torch.float16, device=cuda_dev)
    cuda_ext.run_workload_out(w, z, [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers], None, out)
    torch.cuda.synchronize()
    ref = O.workload_forward(w, z.cpu(), layers, None)
    r = O.compare(out.float().cpu(), ref)
    assert r["ok"], r


def test_shape_errors(cuda_dev):
    bot, sparse = _inputs(8, 1)
    with pytest.raises(RuntimeError):
        cuda_ext.dlrm_interaction(bot.to(cuda_dev), sparse[:, :25].contiguous().to(cuda_dev))
