"""The sync-free inverse-index rebuild (LogicLayer.refresh_backward_index_device, plain torch ops) against the
host rebuild that mirrors the reference (compactlogic.py:184-274), on CPU: full rebuilds and incremental
refreshes after connection changes give the same start offsets and the same entries per input."""
import copy

import torch

import compactlogic_b200 as cl


def _canonical(layer):
    starts = layer.given_x_indices_of_y_start
    counts = starts[1:] - starts[:-1]
    bucket = torch.repeat_interleave(torch.arange(counts.numel()), counts)
    key = (bucket << 40) | (layer.given_x_indices_of_y << 8) | (layer.given_x_indices_of_gate.to(torch.int64) + 128)
    return starts, torch.sort(key).values


def test_full_rebuild_matches_host():
    torch.manual_seed(0)
    layer = cl.LogicLayer(300, 700, num_gates=16)
    ref = copy.deepcopy(layer)
    layer.refresh_backward_index_device(None)
    ref.refresh_backward_index()
    for a, b in zip(_canonical(layer), _canonical(ref)):
        assert torch.equal(a, b)
    # the full rebuild keeps the entry-list order inside every input (stable)
    st = layer.given_x_indices_of_y_start
    ys = layer.given_x_indices_of_y
    codes = layer.given_x_indices_of_gate.to(torch.int64)
    eid = (codes < 0).to(torch.int64) * 700 * 16 + ys * 16 + torch.where(codes < 0, -codes - 1, codes)
    for i in range(0, 300, 37):
        seg = eid[st[i]:st[i + 1]]
        assert bool((seg[1:] > seg[:-1]).all())


def test_incremental_refresh_matches_host():
    torch.manual_seed(1)
    layer = cl.LogicLayer(200, 500, num_gates=8)
    ref = copy.deepcopy(layer)
    rows = torch.tensor([3, 17, 18, 250, 499])
    g = torch.Generator().manual_seed(5)
    new = torch.randint(0, 200, (2, rows.numel(), 8), generator=g)
    for m in (layer, ref):
        m.indices[:, rows] = new
    ref.refresh_backward_index(rows)
    changed = torch.zeros(500, dtype=torch.uint8)
    changed[rows] = 1
    layer.refresh_backward_index_device(changed)
    for a, b in zip(_canonical(layer), _canonical(ref)):
        assert torch.equal(a, b)
    # entries of unchanged neurons keep their relative order; the changed rows' entries follow them
    assert torch.equal(layer.given_x_indices_of_y_start, ref.given_x_indices_of_y_start)
