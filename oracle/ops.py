"""Per-operator CPU restatements (test infrastructure; see oracle/__init__.py).

Integer work (hash routing, pair order) is numpy uint64/int64 arithmetic and
must match the CUDA kernels bit for bit. Floating-point work runs in float64
by default so that it can serve as the reference for fp32 and bf16 kernels.
"""
from __future__ import annotations

import math

import numpy as np
import torch

PAD_TOKEN_ID = 256
MASK32 = np.uint64(0xFFFFFFFF)


# ------------------------------------------------------------------- dense

def affine_scan(retention: torch.Tensor, increment: torch.Tensor, initial: torch.Tensor | None = None,
                dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """h_t = a_t h_{t-1} + b_t, one position at a time (the recurrence that
    model/scan.py:17-30 evaluates by log-step doubling and
    dense/affine_scan.cu:18-56 evaluates per lane). ``retention`` may broadcast
    over trailing dims."""
    a = retention.to(dtype).expand_as(increment) if retention.shape != increment.shape else retention.to(dtype)
    b = increment.to(dtype)
    h = torch.zeros_like(b[:, 0]) if initial is None else initial.to(dtype).clone()
    out = torch.empty_like(b)
    for t in range(b.shape[1]):
        h = a[:, t] * h + b[:, t]
        out[:, t] = h
    return out


def affine_scan_grads(retention, increment, initial, grad_states, dtype=torch.float64):
    """Gradients of the scan by reverse-time adjoint (dense/affine_scan.cu:59-106)."""
    a = retention.to(dtype).expand_as(increment)
    states = affine_scan(retention, increment, initial, dtype)
    g = grad_states.to(dtype)
    adjoint = torch.zeros_like(g[:, 0])
    grad_a = torch.empty_like(g)
    grad_b = torch.empty_like(g)
    h0 = torch.zeros_like(g[:, 0]) if initial is None else initial.to(dtype)
    for t in range(g.shape[1] - 1, -1, -1):
        adjoint = adjoint + g[:, t]
        grad_b[:, t] = adjoint
        grad_a[:, t] = adjoint * (states[:, t - 1] if t > 0 else h0)
        adjoint = adjoint * a[:, t]
    return grad_a, grad_b, adjoint


# -------------------------------------------------------------------- core

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, dtype=torch.float64) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w (model/layers.py:14-16)."""
    v = x.to(dtype)
    return v / torch.sqrt(v.pow(2).mean(dim=-1, keepdim=True) + eps) * weight.to(dtype)


def silu(v: torch.Tensor) -> torch.Tensor:
    return v / (1.0 + torch.exp(-v))


def rmsnorm_silu(x, weight, eps=1e-6, dtype=torch.float64):
    """silu(rmsnorm(x) * w) and inv_rms (core/rmsnorm_silu.cu:63-91)."""
    v = x.to(dtype)
    inv = 1.0 / torch.sqrt(v.pow(2).mean(dim=-1) + eps)
    return silu(v * inv.unsqueeze(-1) * weight.to(dtype)), inv


def gated_rmsnorm_silu(x, gate, weight, eps=1e-6, dtype=torch.float64):
    """silu(gate) * rmsnorm(x) * w (config-3 form)."""
    return silu(gate.to(dtype)) * rms_norm(x, weight, eps, dtype)


def rmsnorm_silu_grads(x, weight, grad_y, eps=1e-6, dtype=torch.float64):
    v = x.to(dtype).clone().requires_grad_(True)
    w = weight.to(dtype).clone().requires_grad_(True)
    y, _ = rmsnorm_silu(v, w, eps, dtype)
    y.backward(grad_y.to(dtype))
    return v.grad, w.grad


# ------------------------------------------------------------------- think

def causal_surprise(prior, weight, bias, targets, valid, dtype=torch.float64):
    """1 - exp(-NLL / ln C) of ``targets`` under softmax(prior W^T + b), zero
    where invalid (network.py:677-688; think/surprise_kernel.cu:85-134)."""
    logits = prior.to(dtype) @ weight.to(dtype).T + bias.to(dtype)
    log_z = torch.logsumexp(logits, dim=-1)
    safe = torch.where(valid, targets, torch.zeros_like(targets))
    nll = log_z - logits.gather(-1, safe.unsqueeze(-1)).squeeze(-1)
    surprise = 1.0 - torch.exp(-nll / math.log(weight.shape[0]))
    return torch.where(valid, surprise, torch.zeros_like(surprise))


def salient_tail(carried_keys, carried_values, carried_valid, keys, values, admission, capacity):
    """Latest ``capacity`` admitted entries of [carried ; window] in temporal
    order (memory.py:431-455). The reference leaves the placement of empty
    slots to topk's tie order; this restatement packs the admitted entries at
    the end behind zeroed invalid slots, the layout the CUDA kernel writes.
    Short path (total <= capacity): plain concatenation, as the reference."""
    all_keys = torch.cat((carried_keys, keys), dim=1)
    all_values = torch.cat((carried_values, values), dim=1)
    all_valid = torch.cat((carried_valid, admission), dim=1)
    total = all_keys.shape[1]
    if total <= capacity:
        return all_keys, all_values, all_valid
    batch, _, width = all_keys.shape
    out_k = all_keys.new_zeros(batch, capacity, width)
    out_v = all_values.new_zeros(batch, capacity, width)
    out_valid = torch.zeros(batch, capacity, dtype=torch.bool)
    for b in range(batch):
        kept = torch.nonzero(all_valid[b], as_tuple=False).squeeze(-1)[-capacity:]
        start = capacity - kept.numel()
        out_k[b, start:] = all_keys[b, kept]
        out_v[b, start:] = all_values[b, kept]
        out_valid[b, start:] = True
    return out_k, out_v, out_valid


def admitted_sequence(keys, values, valid):
    """Per row, the (keys, values) of valid ring slots in slot order: the
    layout-independent content of a salient ring."""
    return [(keys[b][valid[b]], values[b][valid[b]]) for b in range(keys.shape[0])]


# --------------------------------------------------------------------- moe

def content_hash(tokens: np.ndarray, previous: np.ndarray) -> np.ndarray:
    """32-bit bigram hash in 64-bit arithmetic (experts.py:93-101)."""
    t = tokens.astype(np.int64).astype(np.uint64)
    p = previous.astype(np.int64).astype(np.uint64)
    with np.errstate(over="ignore"):
        v = (t * np.uint64(1000003) + p * np.uint64(97409)) & MASK32
        v ^= v >> np.uint64(16)
        v = (v * np.uint64(0x45D9F3B)) & MASK32
        v ^= v >> np.uint64(16)
        v = (v * np.uint64(0x45D9F3B)) & MASK32
        return v ^ (v >> np.uint64(16))


def route_topk(tokens, previous, valid, expert_count: int, top_k: int) -> np.ndarray:
    """Slot s -> (hash + s * 0x9E3779B9) mod E in int64, -1 where invalid
    (experts.py:346-352)."""
    h = content_hash(np.asarray(tokens), np.asarray(previous))
    slots = np.arange(top_k, dtype=np.uint64) * np.uint64(0x9E3779B9)
    out = ((h[..., None] + slots) % np.uint64(expert_count)).astype(np.int64)
    out[~np.asarray(valid, dtype=bool)] = -1
    return out


def pair_keys(assignments: np.ndarray, valid: np.ndarray, expert_count: int) -> np.ndarray:
    """Expert of each pair, or E when invalid / a repeat of an earlier slot
    (experts.py:245-257,324-330)."""
    tokens, top_k = assignments.shape
    keys = np.full((tokens, top_k), expert_count, dtype=np.int64)
    for slot in range(top_k):
        e = assignments[:, slot]
        ok = valid & (e >= 0) & (e < expert_count)
        for earlier in range(slot):
            ok &= assignments[:, earlier] != e
        keys[ok, slot] = e[ok]
    return keys.reshape(-1)


def permute_topk(assignments: np.ndarray, valid: np.ndarray, expert_count: int):
    """Stable pair order (experts.py:194): (order, sorted_rows, sorted_experts,
    segment_offsets, pair_positions)."""
    keys = pair_keys(np.asarray(assignments), np.asarray(valid, dtype=bool), expert_count)
    order = np.argsort(keys, kind="stable")
    counts = np.bincount(keys, minlength=expert_count + 1)
    offsets = np.concatenate(([0], np.cumsum(counts[:expert_count]))).astype(np.int64)
    positions = np.empty_like(order)
    positions[order] = np.arange(order.size)
    top_k = assignments.shape[1]
    return order, order // top_k, keys[order], offsets, positions


def learned_topk(logits: torch.Tensor, valid: torch.Tensor, top_k: int, renormalize: bool = False):
    """softmax_fp32 then top-k (router.py:43-59); ties broken by lower id."""
    probs = torch.softmax(logits.double(), dim=-1)
    order = np.lexsort((np.arange(logits.shape[-1])[None, :].repeat(logits.shape[0], 0),
                        -logits.double().numpy()), axis=-1)[:, :top_k]
    idx = torch.from_numpy(order)
    weights = probs.gather(-1, idx)
    if renormalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    idx = idx.masked_fill(~valid.unsqueeze(-1), -1)
    weights = weights.masked_fill(~valid.unsqueeze(-1), 0.0)
    return idx, weights, probs * valid.unsqueeze(-1)


def gated_ffn(x, gate_w, gate_b, value_w, value_b, out_w, out_b, dtype=torch.float64):
    """W_o (silu(W_g x + b_g) * (W_v x + b_v)) + b_o (layers.py:19-29)."""
    x = x.to(dtype)
    hidden = silu(x @ gate_w.to(dtype).T + gate_b.to(dtype)) * (x @ value_w.to(dtype).T + value_b.to(dtype))
    return hidden @ out_w.to(dtype).T + out_b.to(dtype)


def grouped_mlp(sorted_context, sorted_experts, offsets, gw, gb, vw, vb, ow, ob, dtype=torch.float64,
                round_hidden_to=None):
    """Per-pair gated FFN of the pair's expert; zero past offsets[-1]."""
    out = torch.zeros(sorted_context.shape, dtype=dtype)
    valid = int(offsets[-1])
    for e in range(gw.shape[0]):
        begin, end = int(offsets[e]), int(offsets[e + 1])
        if end <= begin:
            continue
        x = sorted_context[begin:end].to(dtype)
        hidden = silu(x @ gw[e].to(dtype).T + gb[e].to(dtype)) * (x @ vw[e].to(dtype).T + vb[e].to(dtype))
        if round_hidden_to is not None:
            hidden = hidden.to(round_hidden_to).to(dtype)
        out[begin:end] = hidden @ ow[e].to(dtype).T + ob[e].to(dtype)
    del valid
    return out


def combine_topk(expert_outputs, sorted_rows, offsets, token_count, top_k, dtype=torch.float64):
    """out[row] = sum of the row's valid pair outputs / k (moe_kernels.cu:201-229)."""
    out = torch.zeros(token_count, expert_outputs.shape[1], dtype=dtype)
    for i in range(int(offsets[-1])):
        out[int(sorted_rows[i])] += expert_outputs[i].to(dtype) / top_k
    return out


# ---------------------------------------------------------------- expert parallelism
# The reference has no expert parallelism; these restate the slab layout of the
# dispatch (koemi_moe_ep_pack / koemi_moe_ep_unpack) so the exchange can be
# checked against the single-rank grouped MLP above.

def ep_pack(sorted_rows, sorted_experts, offsets, ranks: int, local_experts: int, capacity: int):
    """Slab [ranks * capacity, width]: owner g's sorted rows at g * capacity,
    owner-local expert ids beside them, -1 (and zero rows) for padding."""
    width = sorted_rows.shape[1]
    slab = torch.zeros(ranks * capacity, width, dtype=sorted_rows.dtype)
    ids = torch.full((ranks * capacity,), -1, dtype=torch.int32)
    for g in range(ranks):
        begin, end = int(offsets[g * local_experts]), int(offsets[(g + 1) * local_experts])
        slab[g * capacity:g * capacity + end - begin] = sorted_rows[begin:end]
        ids[g * capacity:g * capacity + end - begin] = (sorted_experts[begin:end] - g * local_experts).to(torch.int32)
    return slab, ids


def ep_unpack(slab, sorted_experts, offsets, ranks: int, local_experts: int, capacity: int):
    """Rows back in sorted order from the returned slab; zero past the valid pairs."""
    out = torch.zeros(sorted_experts.shape[0], slab.shape[1], dtype=slab.dtype)
    for g in range(ranks):
        begin, end = int(offsets[g * local_experts]), int(offsets[(g + 1) * local_experts])
        out[begin:end] = slab[g * capacity:g * capacity + end - begin]
    return out


def permute_rows(rows, assignments, valid, expert_count: int, gather: bool = True):
    """The 5-tuple of the permute front (sorted rows, sorted token rows, sorted
    experts, segment offsets, pair positions) from `permute_topk` above."""
    a = assignments.cpu().numpy()
    order, sorted_tokens, keys, offsets, positions = permute_topk(a, valid.cpu().numpy(), expert_count)
    n_valid = int(offsets[-1])
    sorted_rows = torch.zeros(order.size, rows.shape[1], dtype=rows.dtype)
    sorted_rows[:n_valid] = rows[torch.from_numpy(sorted_tokens[:n_valid])]
    return (sorted_rows, torch.from_numpy(sorted_tokens), torch.from_numpy(keys), torch.from_numpy(offsets),
            torch.from_numpy(positions))


_GOLDEN_GAMMA = np.uint64(0x9E3779B97F4A7C15)


def _splitmix64(z):
    """SplitMix64 finaliser (Steele, Lea and Flood, OOPSLA 2014) on uint64
    arrays, wrapping modulo 2^64 like the kernel's unsigned arithmetic."""
    with np.errstate(over="ignore"):
        z = np.asarray(z, dtype=np.uint64) + _GOLDEN_GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def gumbel_sample(logits, temperature, seed, stream_offset, step, pad, thresholds=None):
    """Counter-based Gumbel-max sampling from softmax(logits / T) with PAD,
    NaN and below-threshold columns excluded (the kernel of
    koemi_sampler_temperature; the reference samples the same distribution
    with torch.multinomial, runtime/fast_decode.py:72-80). Returns
    (ids [rows], scores [rows, vocab] in float64)."""
    x = np.asarray(logits, dtype=np.float64)
    rows, vocab = x.shape
    with np.errstate(over="ignore"):
        streams = np.arange(rows, dtype=np.uint64) + np.uint64(stream_offset)
        key = _splitmix64(np.uint64(seed) ^ _splitmix64(streams ^ _splitmix64(np.uint64(step))))
        columns = np.arange(vocab, dtype=np.uint64) * _GOLDEN_GAMMA
        bits = _splitmix64(key[:, None] + columns[None, :])
    u = ((bits >> np.uint64(41)).astype(np.float64) + 0.5) / 8388608.0
    scores = x / temperature - np.log(-np.log(u))
    dropped = np.isnan(x)
    if 0 <= pad < vocab:
        dropped[:, pad] = True
    if thresholds is not None:
        dropped |= x < np.asarray(thresholds, dtype=np.float64)[:, None]
    scores = np.where(dropped, -np.inf, scores)
    ids = np.where(np.isneginf(scores).all(axis=1), 0, scores.argmax(axis=1))
    return ids, scores
