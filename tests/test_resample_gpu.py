"""Device resampling (LogicLayer.resample_rows_device: clb_resample_rows + the sort-based inverse-index
rebuild) against the host formulation of resample_connections (compactlogic.py:282-368) fed the same
pre-drawn random tensors: identical gates, connections, start offsets and per-input index entries; logits
identical except the strong rows' winner logit (one fp32 log, 1e-6 relative)."""
import copy

import numpy as np
import pytest
import torch

import compactlogic_b200 as cl

pytestmark = pytest.mark.gpu


def _canonical_csr(layer):
    starts = layer.given_x_indices_of_y_start
    counts = starts[1:] - starts[:-1]
    bucket = torch.repeat_interleave(torch.arange(counts.numel(), device=starts.device), counts)
    key = (bucket << 40) | (layer.given_x_indices_of_y << 8) | (layer.given_x_indices_of_gate.to(torch.int64) + 128)
    return starts.cpu(), torch.sort(key).values.cpu()


def _layer(seed, in_dim=300, out=500, K=16):
    torch.manual_seed(seed)
    layer = cl.LogicLayer(in_dim, out, num_gates=K).cuda()
    with torch.no_grad():
        layer.weights[:100] = 0.0            # uniform: max prob 1/K, weak
        layer.weights[100:200, 3] = 8.0      # one dominant gate: strong
    return layer


@pytest.mark.parametrize("update_gate,keep_strong", [(True, True), (False, False)])
def test_device_resample_matches_host(update_gate, keep_strong):
    host = _layer(1)
    dev = copy.deepcopy(host)
    gen = torch.Generator(device="cuda").manual_seed(7)
    picked = (torch.rand(500, device="cuda", generator=gen) < 0.5)
    picked[:5] = True
    picked[100:105] = True
    draws = host.resample_draws(gen)
    kw = dict(threshold_high=0.6, threshold_low=0.1, update_gate=update_gate, keep_strong_weights=keep_strong)
    weak, strong = host.resample_connections(picked.nonzero().flatten(), draws=draws, **kw)
    m1 = torch.rand(500, 16, device="cuda")
    m2 = torch.rand(500, 16, device="cuda")
    counter = torch.full((500,), 9, dtype=torch.int32, device="cuda")
    changed = dev.resample_rows_device(picked.to(torch.uint8), draws, adam_state={"exp_avg": m1, "exp_avg_sq": m2},
                                       counter=counter, **kw)
    assert int(weak.sum()) > 0 and int(strong.sum()) > 0
    assert torch.equal(changed.bool(), weak | strong)
    assert torch.equal(dev.gate_sequence, host.gate_sequence)
    assert torch.equal(dev.indices, host.indices)
    winners = strong.nonzero().flatten()
    wk = host.weights.detach().argmax(-1)[winners]
    mask = torch.ones_like(host.weights, dtype=torch.bool)
    mask[winners, wk] = False
    assert torch.equal(dev.weights.detach()[mask], host.weights.detach()[mask])
    torch.testing.assert_close(dev.weights.detach()[winners, wk], host.weights.detach()[winners, wk], rtol=1e-6, atol=0)
    cs_h, ce_h = _canonical_csr(host)
    cs_d, ce_d = _canonical_csr(dev)
    assert torch.equal(cs_h, cs_d) and torch.equal(ce_h, ce_d)
    ch = changed.bool()
    assert float(m1[ch].abs().sum()) == 0 and float(m2[ch].abs().sum()) == 0
    assert bool((m1[~ch] > 0).all())
    assert bool((counter[picked] == 0).all()) and bool((counter[~picked] == 9).all())
    # the rebuilt slot table follows the new connections: forward equals a fresh layer with the same buffers
    fresh = copy.deepcopy(dev)
    fresh._spec_key = None
    x = torch.rand(8, 300, device="cuda")
    torch.testing.assert_close(dev(x), fresh(x), rtol=0, atol=0)


def test_full_device_rebuild_matches_host():
    layer = _layer(3, in_dim=784, out=12000)
    ref = copy.deepcopy(layer)
    layer.refresh_backward_index_device(None)
    ref.refresh_backward_index()
    assert all(torch.equal(a, b) for a, b in zip(_canonical_csr(layer), _canonical_csr(ref)))


def test_resampler_device_path_runs_without_host_reads():
    """EntropyRowResampler with the device monitor and device resampling rewrites rows and keeps the inverse
    index consistent with the connections."""
    torch.manual_seed(4)
    model = torch.nn.Sequential(cl.LogicLayer(40, 64, num_gates=8), cl.LogicLayer(64, 48, num_gates=8),
                                cl.GroupSum(4, 2.0)).cuda()
    before = model[0].indices.clone()
    opt = torch.optim.Adam(model.parameters(), lr=0.05)
    rs = cl.EntropyRowResampler(model, ema_decay=0.8, eps=1.0, patience=2, threshold_low=0.3, threshold_high=0.6)
    for it in range(6):
        x = (torch.rand(64, 40, device="cuda") < 0.5).float()
        opt.zero_grad()
        torch.nn.functional.cross_entropy(model(x), torch.randint(0, 4, (64,), device="cuda")).backward()
        opt.step()
        rs.step(it, opt)
    assert not torch.equal(before, model[0].indices)
    for m in model[:2]:
        ref = copy.deepcopy(m)
        ref.refresh_backward_index()
        assert all(torch.equal(a, b) for a, b in zip(_canonical_csr(m), _canonical_csr(ref)))
