"""GPU parity of the weight-streaming fused chain (DLRM bottom, GraphCast, NeRF) against the CPU
oracle and the reference models' golden outputs. All calls go through the C ABI.

Tolerance (north star): max |err| <= 2e-2 and relative L2 <= 5e-3 against the fp32 oracle.
Full-size configs whose CPU oracle would take minutes are checked on a deterministic row sample:
the first and last 65,536-row chunks and one from the middle."""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O
from tests._util import load_golden, u16_to
from tests.golden.make_golden import layer_params

pytestmark = pytest.mark.gpu


def _close(out, ref, what):
    r = O.compare(out.float().cpu(), ref)
    assert r["ok"], f"{what}: {r}"
    return r


def _run(w, dev, x=None):
    x = W.make_input(w) if x is None else x
    layers, ln = W.make_weights(w)
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=dev)
    cuda_ext.run_workload_out(w, x.to(dev), [(a.to(dev), b.to(dev)) for a, b in layers],
                              None if ln is None else tuple(t.to(dev) for t in ln), out)
    torch.cuda.synchronize()
    return x, layers, ln, out


def _sample_rows(m):
    c = W.CHUNK_ROWS
    spans = [(0, min(c, m))]
    if m > 2 * c:
        mid = (m // 2) // c * c
        spans.append((mid, c))
    if m > c:
        spans.append((m - min(c, m - c), min(c, m - c)))
    return spans


# ------------------------------------------------------------------ golden (reference models)
def test_golden_dlrm_bot(cuda_dev):
    g = load_golden("dlrm_bot")
    layers = layer_params(int(g["seed"]), list(g["dims"]), init="xavier")
    x = u16_to(g["x"], torch.float16).to(cuda_dev)
    d = [t.to(cuda_dev) for p in layers for t in p]
    out = cuda_ext.dlrm_botmlp(x, *d)
    torch.cuda.synchronize()
    _close(out, torch.from_numpy(g["y"]), "dlrm_bot golden")


def test_golden_gc_edges_relu_bf16(cuda_dev):
    g = load_golden("gc_edges_relu")
    layers = layer_params(int(g["seed"]), list(g["dims"]), dtype=torch.bfloat16)
    x = u16_to(g["x"], torch.bfloat16).to(cuda_dev)
    ga = torch.ones(512, dtype=torch.bfloat16, device=cuda_dev)
    be = torch.zeros(512, dtype=torch.bfloat16, device=cuda_dev)
    d = [t.to(cuda_dev) for p in layers for t in p]
    out = cuda_ext.gc_edges(x, *d, ga, be, act=L.ACT_RELU)
    torch.cuda.synchronize()
    _close(out, torch.from_numpy(g["y"]), "gc_edges golden")


def test_golden_nerf(cuda_dev):
    """Reference Nerf(in_x_ch=63, use_viewdirs=False, out_ch=4): 63 -> 64 and 319 -> 320 padding."""
    g = load_golden("nerf_63")
    gen = torch.Generator().manual_seed(int(g["seed"]))
    ws, bs = [], []
    for i, (k, n) in enumerate(zip(g["dims_in"], g["dims_out"])):
        s = int(torch.randint(0, 2**31 - 1, (1,), generator=gen))
        w, b = layer_params(s, [int(k), int(n)])[0]
        kp = {63: 64, 319: 320}.get(int(k), int(k))
        wp = torch.zeros(kp, int(n), dtype=torch.float16)
        if i == 5:   # [h (256) || x (63)] -> rows 0..255 = h, 256..318 = x, 319 = padding
            wp[:319] = w
        else:
            wp[:int(k)] = w
        ws.append(wp.to(cuda_dev))
        bs.append(b.to(cuda_dev))
    x = torch.zeros(g["x"].shape[0], 64, dtype=torch.float16)
    x[:, :63] = u16_to(g["x"], torch.float16)
    out = torch.zeros(x.shape[0], 4, dtype=torch.float16, device=cuda_dev)
    cuda_ext.nerf_out(x.to(cuda_dev), ws, bs, out)
    torch.cuda.synchronize()
    _close(out, torch.from_numpy(g["y"]), "nerf golden")


# ------------------------------------------------------------------ benchmark configs
def test_dlrm_bot_full_size(cuda_dev):
    w = W.DLRM_BOT
    x, layers, ln, out = _run(w, cuda_dev)
    print("dlrm_bot", _close(out, O.workload_forward(w, x, layers, ln), "dlrm_bot"))


@pytest.mark.parametrize("wname", ["gc_edge", "nerf"])
def test_full_size_sampled(cuda_dev, wname):
    w = W.WORKLOADS[wname]
    x, layers, ln, out = _run(w, cuda_dev)
    for r0, n in _sample_rows(w.m):
        ref = O.workload_forward(w, x[r0:r0 + n], layers, ln)
        print(wname, r0, _close(out[r0:r0 + n], ref, f"{wname} rows {r0}+{n}"))


@pytest.mark.parametrize("wname", ["dlrm_bot", "gc_edge", "nerf"])
@pytest.mark.parametrize("m", [1, 127, 129, 1000, 20000])
def test_ragged_rows(cuda_dev, wname, m):
    w = W.WORKLOADS[wname].with_m(m)
    x, layers, ln, out = _run(w, cuda_dev)
    _close(out, O.workload_forward(w, x, layers, ln), f"{wname} m={m}")


def test_nerf_trunk_matches_oracle(cuda_dev):
    """apps/nerf_a: the trunk alone, out [M, 256]."""
    w = W.NERF.with_m(3000)
    x = W.make_input(w)
    layers, _ = W.make_weights(w)
    trunk = layers[:8]
    d = [t.to(cuda_dev) for p in trunk for t in p]
    out = cuda_ext.nerf_a(x.to(cuda_dev), *d)
    torch.cuda.synchronize()
    ref = O.chain_forward(x, trunk, [O.ACT_RELU] * 8, skip_layer=5)
    _close(out, ref, "nerf trunk")


def test_gc_nodes_fp16_relu(cuda_dev):
    g = torch.Generator().manual_seed(9)
    x = torch.randn(3000, 1024, generator=g).half()
    layers = layer_params(9, [1024, 512, 512])
    ga = (1 + 0.1 * torch.randn(512, generator=g)).half()
    be = (0.1 * torch.randn(512, generator=g)).half()
    d = [t.to(cuda_dev) for p in layers for t in p]
    out = cuda_ext.gc_nodes(x.to(cuda_dev), *d, ga.to(cuda_dev), be.to(cuda_dev))
    torch.cuda.synchronize()
    ref = O.chain_forward(x, layers, [O.ACT_RELU, O.ACT_NONE], O.TAIL_LAYERNORM, (ga, be), 1e-5)
    _close(out, ref, "gc_nodes")


def test_stream_timeout_is_reported(cuda_dev):
    w = W.DLRM_BOT.with_m(2048)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
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
    assert L.device_status(0, clear=True) in (0x100, 0x200, 0x300)
    cuda_ext.run_workload_out(w, xd, wd, None, out)
    torch.cuda.synchronize()
    _close(out, O.workload_forward(w, x, layers, ln), "after timeout")
