"""The reference's own app checks (apps/<app>/pipelined/val.py), replayed through the drop-in
`cuda_ext` with the same model parameters, argument lists, shapes and row counts.

Every app's call goes through the C ABI. The first rows of each input are the fixture rows on
which tests/golden/val_replay.npz holds the reference model's own fp32 output; all rows are
compared with the fp32 oracle. The yardstick is the fp32 model, not the reference's
fp16-accumulating kernels. Tolerance: max |err| <= 2e-2 and relative L2 <= 5e-3.

nerf_full: the reference extension returns (out_r, out_rgb) (nerf_full_pl_ext.cu:133), which its
val.py unpacks under the names (rgb_act, alpha_act); the drop-in returns the extension's order.
"""
import pytest
import torch

from gpu_pipes_b200 import cuda_ext
from oracle import mlp_oracle as O
from tests import _val_apps as V
from tests._util import load_golden, u16_to

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden():
    return load_golden("val_replay")


def _close(out, ref, what):
    r = O.compare(out.float().cpu(), ref)
    assert r["ok"], f"{what}: {r}"


@pytest.mark.parametrize("app", sorted(V.APPS))
def test_reference_val_call(cuda_dev, golden, app):
    ws, bs, ln = V.build(app)
    assert V.checksum(ws, bs) == pytest.approx(float(golden[f"{app}_wsum"]), abs=1e-9)
    xs = V.inputs(app)
    n0 = golden[f"{app}_x0"].shape[0]
    for i, x in enumerate(xs):
        x[:n0] = u16_to(golden[f"{app}_x{i}"], torch.float16)
    dev = lambda ts: [t.to(cuda_dev) for t in ts]  # noqa: E731
    lnd = [tuple(dev(p)) for p in ln]
    out = V.call(cuda_ext, app, dev(xs), dev(ws), dev(bs), lnd)
    torch.cuda.synchronize()
    ref = V.oracle(O, app, xs, ws, bs, ln)
    if app == "nerf_full":
        out_r, out_rgb = out
        _close(out_r, ref[0], "nerf_full alpha")
        _close(out_rgb, ref[1], "nerf_full rgb")
        _close(out_r[:n0], torch.from_numpy(golden["nerf_full_alpha"]), "nerf_full alpha (reference model)")
        _close(out_rgb[:n0], torch.from_numpy(golden["nerf_full_rgb"]), "nerf_full rgb (reference model)")
    else:
        assert tuple(out.shape) == tuple(ref.shape)
        _close(out, ref, app)
        _close(out[:n0], torch.from_numpy(golden[f"{app}_y"]), f"{app} (reference model)")
