"""Training-path ops (ReLU / log-softmax / NLL backward, Adam's update) against
stock PyTorch CPU fp32, op by op and through a few Adam steps of an MLP.

Tolerances: threshold_backward, addcmul, addcdiv, lerp and the NLL gradient
are bit-exact (the operation order and FMA contraction of ATen's CPU loops);
sqrt is within 1 ulp (torch's CPU sqrt is not correctly rounded, ours is);
log-softmax backward and the NLL totals are within rtol 1e-5 / atol 1e-6
(sums in another order); parameters after three Adam steps of the MLP are
within rtol 1e-4 / atol 1e-5 (the GEMMs are 3xTF32, about fp32 accuracy)."""

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from oracle.tolerance import bit_exact, max_ulp

pytestmark = pytest.mark.gpu

aten = torch.ops.aten


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def randn(*shape, seed=0):
    return torch.randn(*shape, generator=gen(seed))


def test_threshold_backward_and_sqrt(mm):
    g, x = randn(37, 65, seed=1), randn(37, 65, seed=2)
    x[0, :5] = 0.0
    got = aten.threshold_backward(mm.to_device(g), mm.to_device(x), 0.0).cpu()
    assert bit_exact(got, aten.threshold_backward(g, x, 0.0))
    v = randn(1000, seed=3).abs()
    assert max_ulp(mm.to_device(v).sqrt().cpu(), v.sqrt()) <= 1
    d = mm.to_device(v)
    d.sqrt_()
    assert max_ulp(d.cpu(), v.sqrt()) <= 1


@pytest.mark.parametrize("value", [1.0, -0.37])
def test_addcmul_addcdiv_lerp(mm, value):
    s, a, b = randn(33, 70, seed=4), randn(33, 70, seed=5), randn(33, 70, seed=6).abs() + 0.1
    ds, da, db = mm.to_device(s), mm.to_device(a), mm.to_device(b)
    assert bit_exact(torch.addcmul(ds, da, db, value=value).cpu(), torch.addcmul(s, a, b, value=value))
    assert bit_exact(torch.addcdiv(ds, da, db, value=value).cpu(), torch.addcdiv(s, a, b, value=value))
    for w in (0.1, 0.9):
        assert bit_exact(torch.lerp(ds, da, w).cpu(), torch.lerp(s, a, w))
    # in place, with a broadcast operand
    row = randn(70, seed=7)
    ds.addcmul_(da, mm.to_device(row), value=value)
    assert bit_exact(ds.cpu(), s.clone().addcmul_(a, row, value=value))
    da.lerp_(db, 0.25)
    assert bit_exact(da.cpu(), a.clone().lerp_(b, 0.25))


@pytest.mark.parametrize("shape,dim", [((64, 10), 1), ((5, 7, 9), 0), ((3, 130), -1)])
def test_log_softmax_backward(mm, shape, dim):
    x = randn(*shape, seed=8)
    out = torch.log_softmax(x, dim)
    g = randn(*shape, seed=9)
    got = aten._log_softmax_backward_data(mm.to_device(g), mm.to_device(out), dim, torch.float32).cpu()
    want = aten._log_softmax_backward_data(g, out, dim, torch.float32)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("reduction", [0, 1, 2])
@pytest.mark.parametrize("weighted", [False, True])
def test_nll_loss_forward_backward(mm, reduction, weighted):
    n, c = 50, 11
    x = torch.log_softmax(randn(n, c, seed=10), 1)
    t = torch.randint(0, c, (n,), generator=gen(11))
    t[[3, 17]] = -100                                       # ignored rows
    w = randn(c, seed=12).abs() + 0.5 if weighted else None
    dx, dt = mm.to_device(x), mm.to_device(t)
    dw = mm.to_device(w) if weighted else None
    out, total = aten.nll_loss_forward(dx, dt, dw, reduction, -100)
    want_out, want_total = aten.nll_loss_forward(x, t, w, reduction, -100)
    if reduction == 0:
        assert bit_exact(out.cpu(), want_out)
    else:
        torch.testing.assert_close(out.cpu(), want_out, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(total.cpu(), want_total, rtol=1e-6, atol=0.0)
    go = randn(n, seed=13) if reduction == 0 else torch.tensor(0.7)
    got = aten.nll_loss_backward(mm.to_device(go), dx, dt, dw, reduction, -100, total).cpu()
    want = aten.nll_loss_backward(go, x, t, w, reduction, -100, want_total)
    if reduction == 1:
        # the mean divides by total_weight, summed in another order
        torch.testing.assert_close(got, want, rtol=1e-6, atol=0.0)
    else:
        assert bit_exact(got, want)


def test_nll_loss_rejects_out_of_range_targets(mm):
    x = mm.to_device(torch.log_softmax(randn(4, 3, seed=14), 1))
    with pytest.raises(RuntimeError, match="out-of-range"):
        aten.nll_loss_forward(x, mm.to_device(torch.tensor([0, 1, 3, 2])), None, 1, -100)


def _mlp(seed):
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(32, 64), nn.ReLU(), nn.Linear(64, 10))


def test_mlp_adam_steps_match_cpu(mm):
    cpu_net, dev_net = _mlp(0), _mlp(0)
    for m in dev_net:
        if isinstance(m, nn.Linear):
            m.weight = nn.Parameter(mm.to_device(m.weight.detach()))
            m.bias = nn.Parameter(mm.to_device(m.bias.detach()))
    cpu_opt = torch.optim.Adam(cpu_net.parameters(), lr=1e-2, foreach=False)
    dev_opt = torch.optim.Adam(dev_net.parameters(), lr=1e-2, foreach=False)
    for step in range(3):
        x = randn(16, 32, seed=20 + step)
        t = torch.randint(0, 10, (16,), generator=gen(30 + step))
        losses = []
        for net, opt, xi, ti in ((cpu_net, cpu_opt, x, t),
                                 (dev_net, dev_opt, mm.to_device(x), mm.to_device(t))):
            opt.zero_grad()
            loss = F.nll_loss(torch.log_softmax(net(xi), 1), ti)
            loss.backward()
            opt.step()
            losses.append(loss.detach())
        torch.testing.assert_close(losses[1].cpu(), losses[0], rtol=1e-4, atol=1e-5)
    for p_cpu, p_dev in zip(cpu_net.parameters(), dev_net.parameters()):
        torch.testing.assert_close(p_dev.detach().cpu(), p_cpu.detach(), rtol=1e-4, atol=1e-5)
