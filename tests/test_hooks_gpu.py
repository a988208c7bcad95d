"""EntropyRowResampler on CUDA layers: the fused device monitor (one kernel per layer, one sync per step)
makes exactly the decisions of the reference's op-by-op torch formulation (compactlogic.py:1113-1150)."""
import copy

import numpy as np
import pytest
import torch

import compactlogic_b200 as cl

pytestmark = pytest.mark.gpu


def _run(model, use_device, steps=40):
    opt = torch.optim.Adam(model.parameters(), lr=0.05)
    rs = cl.EntropyRowResampler(model, ema_decay=0.8, eps=2e-3, patience=3, threshold_low=0.3, threshold_high=0.6)
    rs.use_device_monitor = use_device
    rs.use_device_resample = False  # same RNG consumption on both sides: only the monitor differs
    torch.cuda.manual_seed(123)
    gen = torch.Generator(device="cuda").manual_seed(5)
    for it in range(steps):
        x = (torch.rand(64, 40, device="cuda", generator=gen) < 0.5).float()
        y = torch.randint(0, 4, (64,), device="cuda", generator=gen)
        opt.zero_grad()
        torch.nn.functional.cross_entropy(model(x), y).backward()
        if it % 3 == 0:  # freeze some rows' logits so they converge and get resampled
            opt.step()
        rs.step(it, opt)
    return model, rs


def test_device_monitor_matches_torch_ops():
    torch.manual_seed(0)
    base = torch.nn.Sequential(cl.LogicLayer(40, 64, num_gates=8), cl.LogicLayer(64, 48, num_gates=8),
                               cl.GroupSum(4, 2.0)).cuda()
    with torch.no_grad():
        base[0].weights[:10] = 0.0
        base[0].weights[10:20, 2] = 6.0
    m_ref, rs_ref = _run(copy.deepcopy(base), use_device=False)
    m_dev, rs_dev = _run(copy.deepcopy(base), use_device=True)
    resampled = 0
    for (k, a), (_, b) in zip(m_ref.state_dict().items(), m_dev.state_dict().items()):
        torch.testing.assert_close(a, b, rtol=0, atol=1e-6, msg=k)
    for idx in rs_ref.ema:
        torch.testing.assert_close(rs_ref.ema[idx], rs_dev.ema[idx], rtol=1e-5, atol=1e-6)
        assert torch.equal(rs_ref.counter[idx], rs_dev.counter[idx])
    # the scenario really resampled rows
    assert not torch.equal(base[0].indices.cpu(), m_dev[0].indices.cpu())
