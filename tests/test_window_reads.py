"""The window path's ring reads (local sliding window with novelty, salient
carried + earlier admitted) against slot-by-slot loops of the reference's
definitions (memory.py:332-383, 405-429), on CPU tensors."""
from __future__ import annotations

import math

import pytest
import torch

from koemi_5hom_b200.model.network import _local_read, _ring_tail, _salient_read


def _loop_local(ck, cv, cvalid, k, v, valid, q, window):
    keys, values, ok = torch.cat((ck, k), 1), torch.cat((cv, v), 1), torch.cat((cvalid, valid), 1)
    batch, length, d = q.shape
    carried = ck.shape[1]
    out, novelty = torch.zeros_like(q), torch.ones(batch, length, dtype=q.dtype)
    for b in range(batch):
        for t in range(length):
            own = carried + t
            slots = [s for s in range(max(0, own - window), own) if ok[b, s]]
            if not slots:
                continue
            w = torch.softmax(keys[b, slots] @ q[b, t] / math.sqrt(d), dim=0)
            out[b, t] = w @ values[b, slots]
            cos = (keys[b, slots] / keys[b, slots].norm(dim=-1, keepdim=True)) @ (q[b, t] / q[b, t].norm())
            novelty[b, t] = (1.0 - cos.max()).clamp(0.0, 1.0)
    return out, novelty


def _loop_salient(ck, cv, cvalid, k, v, admission, q):
    batch, length, d = q.shape
    out = torch.zeros_like(q)
    for b in range(batch):
        for t in range(length):
            rows = [ck[b, s] for s in range(ck.shape[1]) if cvalid[b, s]] + [k[b, s] for s in range(t) if admission[b, s]]
            vals = [cv[b, s] for s in range(ck.shape[1]) if cvalid[b, s]] + [v[b, s] for s in range(t) if admission[b, s]]
            if rows:
                w = torch.softmax(torch.stack(rows) @ q[b, t] / math.sqrt(d), dim=0)
                out[b, t] = w @ torch.stack(vals)
    return out


@pytest.mark.parametrize("carried,length,window", [(6, 5, 4), (4, 9, 4), (0, 7, 3), (5, 3, 8)])
def test_window_reads_match_slot_loops(carried, length, window):
    g = torch.Generator().manual_seed(carried * 10 + length)
    batch, d = 3, 16
    t = lambda *shape: torch.randn(*shape, generator=g, dtype=torch.float64)  # noqa: E731
    ck, cv, k, v, q = t(batch, carried, d), t(batch, carried, d), t(batch, length, d), t(batch, length, d), t(batch, length, d)
    cvalid = torch.rand(batch, carried, generator=g) > 0.3
    valid = torch.rand(batch, length, generator=g) > 0.2
    admission = torch.rand(batch, length, generator=g) > 0.5
    value, novelty = _local_read(ck, cv, cvalid, k, v, valid, q, window)
    want_value, want_novelty = _loop_local(ck, cv, cvalid, k, v, valid, q, window)
    torch.testing.assert_close(value, want_value)
    torch.testing.assert_close(novelty, want_novelty)
    torch.testing.assert_close(_salient_read(ck, cv, cvalid, k, v, admission, q),
                               _loop_salient(ck, cv, cvalid, k, v, admission, q))


@pytest.mark.parametrize("carried,length,keep", [(4, 6, 4), (4, 2, 5), (0, 3, 3), (7, 7, 7)])
def test_ring_tail_keeps_the_latest_entries(carried, length, keep):
    c = torch.arange(carried).view(1, carried, 1).float()
    w = 100 + torch.arange(length).view(1, length, 1).float()
    assert torch.equal(_ring_tail(c, w, keep), torch.cat((c, w), 1)[:, carried + length - keep:])
