"""The MSE loss folded into the engines (cqt_synthesis_sqerr /
cqt_adj_synthesis_sqerr, TrainableCQT.mse_loss) against the reference's
train step ``((bwd(*fwd(x)) - target) ** 2).mean().backward()``.

* the loss equals the float64 mean of (y - target)^2 of the engine's own y
  (relative error < 1e-5) and y is bit-identical to the plain synthesis;
* dL/dx matches the oracle's chain rule at >= 120 dB (the north star's
  gradient tolerance) and the eager-loss path at >= 120 dB;
* the loss gradient scales the result (dL/dloss is read on the device),
  the target gradient is -2 (y - target) / n, results are deterministic, and
  the ctypes path equals the C++ fast path bit for bit.
"""
import numpy as np
import pytest
import torch

from fixtures import gy_seed, oracle, x_noise
from oracle.cqt_oracle import snr_db

pytestmark = pytest.mark.gpu

GRAD_DB = 120.0
N = 65536


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _trainable(dev, ctypes_only=False):
    from flash_cqt_b200 import OctCQT, TrainableCQT
    t = TrainableCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev), dev)
    if ctypes_only:
        t.eng._ops = None
    return t


def _np(t):
    return t.detach().cpu().numpy()


def test_loss_value_and_output(dev):
    t = _trainable(dev)
    x = torch.from_numpy(x_noise()).to(dev)
    tgt = torch.from_numpy(gy_seed()).to(dev)
    blocks, side = t.fwd(x)
    loss, y = t.mse_loss(blocks, side, tgt, return_output=True)
    y_plain = t.bwd(blocks, side)
    assert torch.equal(y, y_plain)
    want = float(((y.double() - tgt.double()) ** 2).mean())
    assert abs(float(loss) - want) <= 1e-5 * want
    loss2 = t.mse_loss(blocks, side, tgt)
    assert torch.equal(loss, loss2)


def test_gradient_matches_oracle_and_eager_loss(dev):
    t = _trainable(dev)
    x0, tgt0 = x_noise(), gy_seed()
    tgt = torch.from_numpy(tgt0).to(dev)
    xf = torch.from_numpy(x0).to(dev).requires_grad_(True)
    t.mse_loss(*t.fwd(xf), tgt).backward()
    xe = torch.from_numpy(x0).to(dev).requires_grad_(True)
    ((t.bwd(*t.fwd(xe)) - tgt) ** 2).mean().backward()
    o = oracle()
    yo = o.bwd(o.fwd(x0.astype(np.float64)))
    want = o.adj_fwd(o.adj_bwd(2.0 * (yo - tgt0) / yo.size))
    got = _np(xf.grad).astype(np.float64)
    assert snr_db(want, got) >= GRAD_DB
    assert snr_db(_np(xe.grad).astype(np.float64), got) >= GRAD_DB


def test_loss_gradient_scale_and_target_gradient(dev):
    t = _trainable(dev)
    x = torch.from_numpy(x_noise()).to(dev)
    tgt = torch.from_numpy(gy_seed()).to(dev)
    x1 = x.clone().requires_grad_(True)
    t.mse_loss(*t.fwd(x1), tgt).backward()
    x3 = x.clone().requires_grad_(True)
    tg = tgt.clone().requires_grad_(True)
    loss, y = t.mse_loss(*t.fwd(x3), tg, return_output=True)
    (3.0 * loss).backward()
    assert snr_db(3.0 * _np(x1.grad).astype(np.float64), _np(x3.grad)) >= GRAD_DB
    gt_want = -2.0 * 3.0 * (y.double() - tgt.double()) / y.numel()
    assert snr_db(_np(gt_want), _np(tg.grad).astype(np.float64)) >= GRAD_DB


def test_deterministic_and_ctypes_path_bitwise(dev):
    x = torch.from_numpy(x_noise()).to(dev)
    tgt = torch.from_numpy(gy_seed()).to(dev)
    res = []
    for ctypes_only in (False, False, True):
        t = _trainable(dev, ctypes_only)
        xg = x.clone().requires_grad_(True)
        loss = t.mse_loss(*t.fwd(xg), tgt)
        loss.backward()
        res.append((loss.detach().clone(), xg.grad.clone()))
    for loss, g in res[1:]:
        assert torch.equal(loss, res[0][0])
        assert torch.equal(g, res[0][1])


def test_batched_lead_dims_and_empty(dev):
    t = _trainable(dev)
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(2, 3, N, generator=g).to(dev)
    tgt = torch.randn(2, 3, N, generator=g).to(dev)
    loss, y = t.mse_loss(*t.fwd(x), tgt, return_output=True)
    assert y.shape == (2, 3, N)
    want = float(((y.double() - tgt.double()) ** 2).mean())
    assert abs(float(loss) - want) <= 1e-5 * want
    e = torch.empty(0, N, device=dev)
    le = t.mse_loss(*t.fwd(e), e)
    assert float(le) == 0.0
    with pytest.raises(ValueError):
        t.mse_loss(*t.fwd(x), tgt[:1])
