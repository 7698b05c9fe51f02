"""CPU checks of the restated reference app checks (tests/_val_apps.py): the parameters equal
those of the reference's own models built as each apps/<app>/pipelined/val.py builds them
(checksums from the reference classes), and the oracle reproduces those models' outputs."""
import pytest
import torch

from oracle import mlp_oracle as O
from tests import _val_apps as V
from tests._util import load_golden, u16_to


@pytest.fixture(scope="module")
def golden():
    return load_golden("val_replay")


@pytest.mark.parametrize("app", sorted(V.APPS))
def test_val_app_params_and_oracle(golden, app):
    ws, bs, ln = V.build(app)
    assert V.checksum(ws, bs) == pytest.approx(float(golden[f"{app}_wsum"]), abs=1e-9)
    n_in = len(V.APPS[app][2])
    xs = [u16_to(golden[f"{app}_x{i}"], torch.float16) for i in range(n_in)]
    assert all(torch.equal(a, b) for a, b in zip(xs, V.inputs(app, xs[0].shape[0])))
    y = V.oracle(O, app, xs, ws, bs, ln)
    if app == "nerf_full":
        alpha, rgb = y
        assert torch.allclose(alpha, torch.from_numpy(golden["nerf_full_alpha"]), atol=1e-5, rtol=1e-5)
        assert torch.allclose(rgb, torch.from_numpy(golden["nerf_full_rgb"]), atol=1e-5, rtol=1e-5)
    else:
        assert torch.allclose(y, torch.from_numpy(golden[f"{app}_y"]), atol=1e-5, rtol=1e-5)
