"""The in-place decode path (circular rings, fused step kernels) against the
oracle and against the window path of the same model."""
from __future__ import annotations

import math

import pytest
import torch

from conftest import load_golden
from herm_weights import HermShape, herm_parameters
from koemi_5hom_b200 import _native
from koemi_5hom_b200.model import KoemiModel, ModelSettings
from koemi_5hom_b200.model.decode import from_koemi_state, to_koemi_state
from koemi_5hom_b200.runtime import BatchDecoder, SamplingPolicy, TokenSampler
from oracle import ops

pytestmark = pytest.mark.gpu


def _ring_case(batch, width, local_slots, salient_slots, seed, fill=0.6):
    g = torch.Generator().manual_seed(seed)
    t = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    lk, lv = t(batch, local_slots, width), t(batch, local_slots, width)
    lvalid = torch.rand(batch, local_slots, generator=g) > 0.2
    counts = [int(c) for c in torch.randint(0, salient_slots + 1, (batch,), generator=g)]
    counts[0] = salient_slots  # one full ring, one empty ring
    counts[-1] = 0
    heads = [int(h) for h in torch.randint(0, salient_slots, (batch,), generator=g)]
    sk, sv = t(batch, salient_slots, width), t(batch, salient_slots, width)
    svalid = torch.zeros(batch, salient_slots, dtype=torch.bool)
    for b in range(batch):
        for i in range(counts[b]):
            svalid[b, (heads[b] + i) % salient_slots] = True
    query = t(batch, width)
    entries = t(batch, 2 * width)
    valid = torch.rand(batch, generator=g) > 0.15
    surprise = torch.rand(batch, generator=g)
    return dict(lk=lk, lv=lv, lvalid=lvalid, sk=sk, sv=sv, svalid=svalid, heads=heads, counts=counts, q=query,
                entries=entries, valid=valid, surprise=surprise)


def _logical_salient(sk, sv, head, count, slots):
    idx = [(head + i) % slots for i in range(count)]
    return sk[idx], sv[idx]


@pytest.mark.parametrize("ring_dtype", [torch.float32, torch.bfloat16])
# >= 148 streams take the one-CTA-per-(stream, ring) kernel, fewer the
# cluster-split kernel
@pytest.mark.parametrize("batch,width,local_slots,salient_slots", [(7, 64, 16, 12), (256, 2048, 128, 128),
                                                                   (3, 128, 5, 9), (16, 256, 128, 128),
                                                                   (37, 512, 64, 128), (32, 2048, 128, 128),
                                                                   (160, 4096, 16, 8), (200, 1000, 24, 40)])
def test_ring_decode_step_matches_oracle(batch, width, local_slots, salient_slots, ring_dtype, cuda):
    c = _ring_case(batch, width, local_slots, salient_slots, seed=width)
    # the kernel reads stored (possibly bf16) rows and computes in fp32, so the
    # expectation is built from the stored values
    for key in ("lk", "lv", "sk", "sv"):
        c[key] = c[key].to(ring_dtype).float()
    head = 3 % local_slots
    threshold = 0.5
    dev = lambda x: x.to(cuda).contiguous()  # noqa: E731
    ring = lambda x: x.to(device=cuda, dtype=ring_dtype).contiguous()  # noqa: E731
    lk, lv, lvalid = ring(c["lk"]), ring(c["lv"]), dev(c["lvalid"])
    sk, sv, svalid = ring(c["sk"]), ring(c["sv"]), dev(c["svalid"])
    s_head = torch.tensor(c["heads"], dtype=torch.int32, device=cuda)
    s_count = torch.tensor(c["counts"], dtype=torch.int32, device=cuda)
    local_head = torch.tensor([head], dtype=torch.int64, device=cuda)
    out = torch.zeros(batch, 4 * width, device=cuda)
    novelty = torch.empty(batch, device=cuda)
    admission = torch.empty(batch, dtype=torch.bool, device=cuda)
    q_rows = torch.zeros(batch, 4 * width)
    q_rows[:, :width] = c["q"]
    q_rows = dev(q_rows)
    entries, valid, surprise = dev(c["entries"]), dev(c["valid"]), dev(c["surprise"])
    p = _native.ptr
    _native.call("koemi_think_ring_decode_step", p(q_rows), 4 * width, p(entries), 2 * width, p(valid), p(surprise),
                 threshold, p(lk), p(lv), p(lvalid), p(local_head), p(sk), p(sv), p(svalid), p(s_head), p(s_count),
                 p(out[:, 2 * width:]), p(out[:, 3 * width:]), 4 * width, p(novelty), p(admission), batch, width,
                 local_slots, salient_slots, _native.dtype_code(ring_dtype), _native.F32,
                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    scale = 1.0 / math.sqrt(width)
    for b in range(batch):
        q = c["q"][b].double()
        # local read over every valid slot (all slots are inside the window at T=1)
        slots = [s for s in range(local_slots) if c["lvalid"][b, s]]
        if slots:
            k = c["lk"][b, slots].double()
            w = torch.softmax(k @ q * scale, dim=0)
            expected = w @ c["lv"][b, slots].double()
            cos = (k / k.norm(dim=-1, keepdim=True).clamp_min(1e-12)) @ (q / q.norm().clamp_min(1e-12))
            expected_novelty = float((1 - cos.max()).clamp(0, 1))
        else:
            expected, expected_novelty = torch.zeros(width, dtype=torch.float64), 1.0
        torch.testing.assert_close(out[b, 2 * width:3 * width].cpu().double(), expected, rtol=1e-4, atol=1e-5)
        assert abs(novelty[b].item() - expected_novelty) < 1e-4
        # salient read over the admitted entries carried in
        ks, vs = _logical_salient(c["sk"][b], c["sv"][b], c["heads"][b], c["counts"][b], salient_slots)
        if ks.shape[0]:
            w = torch.softmax(ks.double() @ q * scale, dim=0)
            expected = w @ vs.double()
        else:
            expected = torch.zeros(width, dtype=torch.float64)
        torch.testing.assert_close(out[b, 3 * width:].cpu().double(), expected, rtol=1e-4, atol=1e-5)
        # writes: the oldest local slot takes the (masked) new entry
        entry_k = c["entries"][b, :width] if c["valid"][b] else torch.zeros(width)
        entry_v = c["entries"][b, width:] if c["valid"][b] else torch.zeros(width)
        entry_k, entry_v = entry_k.to(ring_dtype).float(), entry_v.to(ring_dtype).float()
        assert torch.equal(lk[b, head].cpu().float(), entry_k) and torch.equal(lv[b, head].cpu().float(), entry_v)
        assert bool(lvalid[b, head]) == bool(c["valid"][b])
        # salient: the admitted sequence is the latest `salient_slots` of old + new
        admitted = bool(c["valid"][b]) and float(c["surprise"][b]) > threshold
        assert bool(admission[b]) == admitted
        old_k, old_v = _logical_salient(c["sk"][b], c["sv"][b], c["heads"][b], c["counts"][b], salient_slots)
        if admitted:
            old_k = torch.cat((old_k, entry_k.unsqueeze(0)))[-salient_slots:]
            old_v = torch.cat((old_v, entry_v.unsqueeze(0)))[-salient_slots:]
        new_k, new_v = _logical_salient(sk[b].cpu().float(), sv[b].cpu().float(), int(s_head[b]), int(s_count[b]),
                                        salient_slots)
        assert torch.equal(new_k, old_k) and torch.equal(new_v, old_v)


@pytest.mark.parametrize("batch,d", [(9, 256), (5, 2048), (300, 2048)])
@pytest.mark.parametrize("feature_source", ["logits", "f32_weight", "bf16_weight"])
def test_assoc_decode_step_matches_oracle(feature_source, batch, d, cuda):
    """Rows split over a cluster of CTAs (few streams) or one CTA per stream
    walking the rows in several passes (many streams)."""
    g = torch.Generator().manual_seed(3)
    m = 16
    proj = torch.randn(batch, 3 * d + 2, generator=g)
    feats = torch.randn(2, batch, m, generator=g)
    feature_weight = torch.randn(m, d, generator=g) * 0.1
    feature_bias = torch.randn(m, generator=g) * 0.1
    if feature_source != "logits":
        # logits of the in-kernel projection: key / query rounded to the weight type, fp32 accumulation
        wd = torch.float32 if feature_source == "f32_weight" else torch.bfloat16
        feature_weight, feature_bias = feature_weight.to(wd), feature_bias.to(wd)
        rows = torch.stack((proj[:, :d], proj[:, d:2 * d])).to(wd).double()
        feats = (rows @ feature_weight.double().T + feature_bias.double()).float()
    surprise = torch.rand(batch, generator=g)
    valid = torch.rand(batch, generator=g) > 0.2
    basis = torch.randn(batch, d, m, generator=g) * 0.1
    normalizer = torch.rand(batch, m, generator=g)
    b_dev, n_dev = basis.to(cuda), normalizer.to(cuda)
    out = torch.zeros(batch, 4 * d, device=cuda)
    # keep every device input alive until the kernel has run: a temporary's
    # memory can be handed to the next argument's copy as soon as it is freed
    proj_dev, feats_dev, surprise_dev, valid_dev = proj.to(cuda), feats.to(cuda), surprise.to(cuda), valid.to(cuda)
    w_dev, wb_dev = feature_weight.to(cuda), feature_bias.to(cuda)
    p = _native.ptr
    logits_ptr = p(feats_dev) if feature_source == "logits" else None
    _native.call("koemi_assoc_decode_step", p(proj_dev), 3 * d + 2, logits_ptr, p(w_dev), p(wb_dev),
                 _native.dtype_code(w_dev.dtype), p(surprise_dev), p(valid_dev), p(b_dev), p(n_dev), p(out[:, d:]),
                 4 * d, batch, d, m, _native.F32, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    f, qf = torch.softmax(feats[0].double(), -1), torch.softmax(feats[1].double(), -1)
    decay = 2.0 ** -12 + (1 - 2.0 ** -11) * torch.sigmoid(proj[:, 3 * d].double())
    write = torch.sigmoid(proj[:, 3 * d + 1].double()) * (0.25 + 0.75 * surprise.double().clamp(0, 1))
    decay = torch.where(valid, decay, 1.0)
    write = torch.where(valid, write, 0.0)
    value = torch.tanh(proj[:, 2 * d:3 * d].double())
    read, new_basis, new_norm = _oracle_scan_read(basis.double(), normalizer.double(), decay, value, f, write, qf)
    torch.testing.assert_close(out[:, d:2 * d].cpu().double(), read, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(b_dev.cpu().double(), new_basis, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(n_dev.cpu().double(), new_norm, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("weight_dtype", [torch.float32, torch.bfloat16])
def test_assoc_decode_stream_does_not_depend_on_its_batch(weight_dtype, cuda):
    """A stream's read, basis and normalizer are bit-identical whether it is
    stepped in a batch of 256 streams, 100 or 5: the batch size sets how many
    CTAs share a stream's rows (on 148 SMs one at 256 streams, 2 at 100, 8 at
    5), and every CTA computes the stream's feature logits in full and only
    its own rows, so the split leaves the arithmetic unchanged."""
    g = torch.Generator().manual_seed(11)
    batch, d, m = 256, 2048, 16
    proj = torch.randn(batch, 3 * d + 2, generator=g).to(cuda)
    weight = (torch.randn(m, d, generator=g) * 0.1).to(weight_dtype).to(cuda)
    bias = (torch.randn(m, generator=g) * 0.1).to(weight_dtype).to(cuda)
    surprise = torch.rand(batch, generator=g).to(cuda)
    valid = (torch.rand(batch, generator=g) > 0.2).to(cuda)
    basis = (torch.randn(batch, d, m, generator=g) * 0.1).to(cuda)
    normalizer = torch.rand(batch, m, generator=g).to(cuda)
    results = {}
    for rows in (256, 100, 5):
        b_dev, n_dev = basis[:rows].clone(), normalizer[:rows].clone()
        out = torch.zeros(rows, d, device=cuda)
        p = _native.ptr
        _native.call("koemi_assoc_decode_step", p(proj), 3 * d + 2, None, p(weight), p(bias),
                     _native.dtype_code(weight_dtype), p(surprise), p(valid), p(b_dev), p(n_dev), p(out), d, rows,
                     d, m, _native.F32, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        results[rows] = (out, b_dev, n_dev)
    for rows in (100, 5):
        for got, full in zip(results[rows], results[256]):
            assert torch.equal(got, full[:rows]), rows
    _native.raise_for_device_status(cuda)


def _oracle_scan_read(basis, normalizer, decay, value, features, write, qf):
    from oracle.herm import HermOracle
    reads, b, n = HermOracle._scan_read(None, basis, normalizer, decay.unsqueeze(1), value.unsqueeze(1),
                                        features.unsqueeze(1), write.unsqueeze(1), qf.unsqueeze(1))
    return reads[:, 0], b, n


def _build(name, compute_dtype):
    fx = load_golden(name)
    case = fx["case"]
    settings = ModelSettings(**case["settings"], compute_dtype=compute_dtype)
    params = herm_parameters(HermShape(settings.vocabulary_size, settings.embedding_size, settings.memory_features,
                                       settings.expert_count, settings.expert_routing, settings.ablation),
                             case["seed"], case["init"], dtype=torch.bfloat16 if case.get("bf16") else torch.float32)
    model = KoemiModel(settings, device="cuda")
    model.load_reference_parameters({k: v.cuda() for k, v in params.items()})
    return fx, model


@pytest.mark.parametrize("name,dtype,steps", [("c1_t065", "float32", 64), ("c5_small", "bfloat16", 40)])
@pytest.mark.parametrize("capture_graph", [False, True])
def test_in_place_decoder_matches_window_decoder(name, dtype, steps, capture_graph):
    fx, model = _build(name, dtype)
    ids = fx["ids"].cuda()
    sampler = TokenSampler(SamplingPolicy(greedy=True), model.device)
    runs = []
    for in_place in (False, True):
        decoder = BatchDecoder(model, capture_graph=capture_graph and in_place, in_place=in_place)
        assert (decoder._dstate is None) or in_place
        logits = decoder.prefill(ids)
        tokens, all_logits = [], []
        for _ in range(steps):
            token = sampler(logits)
            tokens.append(token)
            all_logits.append(logits.clone())
            logits = decoder.step(token)
        runs.append((torch.cat(tokens, 1), torch.stack(all_logits, 1), decoder.state))
    (t0, l0, s0), (t1, l1, s1) = runs
    assert torch.equal(t0, t1)
    tol = 1e-4 if dtype == "float32" else 2e-2
    torch.testing.assert_close(l1, l0, rtol=tol, atol=tol)
    stored = min(steps, fx["decode_tokens"].shape[1])  # the golden holds this many reference steps
    assert torch.equal(t1[:, :stored].cpu(), fx["decode_tokens"][:, :stored])
    for field in ("working_state", "memory_basis", "memory_normalizer", "local_keys", "local_values"):
        torch.testing.assert_close(getattr(s1, field), getattr(s0, field), rtol=1e-3, atol=1e-4)
    assert torch.equal(s1.local_valid, s0.local_valid)
    assert torch.equal(s1.last_token_ids, s0.last_token_ids)
    mine = ops.admitted_sequence(s1.salient_keys.cpu(), s1.salient_values.cpu(), s1.salient_valid.cpu())
    theirs = ops.admitted_sequence(s0.salient_keys.cpu(), s0.salient_values.cpu(), s0.salient_valid.cpu())
    for (mk, mv), (rk, rv) in zip(mine, theirs):
        assert mk.shape == rk.shape
        torch.testing.assert_close(mk, rk, rtol=1e-3, atol=1e-4)


def test_bf16_rings_keep_greedy_tokens():
    """bf16 ring storage (fp32 arithmetic) against the fp32 rings of the same
    bf16 model: same greedy tokens as the reference golden (64 steps), logits
    within 2e-2. The config-5-width case runs both ring types in
    test_gpu_model.test_bf16_model_within_logit_gate."""
    fx, model = _build("c5_small", "bfloat16")
    ids = fx["ids"].cuda()
    sampler = TokenSampler(SamplingPolicy(greedy=True), model.device)
    stored = fx["decode_tokens"].shape[1]
    runs = []
    for ring_dtype in (torch.float32, torch.bfloat16):
        decoder = BatchDecoder(model, capture_graph=True, ring_dtype=ring_dtype)
        logits = decoder.prefill(ids)
        tokens, all_logits = [], []
        for _ in range(stored):
            token = sampler(logits)
            tokens.append(token)
            all_logits.append(logits.clone())
            logits = decoder.step(token)
        assert decoder._dstate.ring_dtype == ring_dtype
        runs.append((torch.cat(tokens, 1), torch.stack(all_logits, 1)))
    (t0, l0), (t1, l1) = runs
    assert torch.equal(t1.cpu(), fx["decode_tokens"][:, :stored])
    assert torch.equal(t1, t0)
    torch.testing.assert_close(l1, l0, rtol=2e-2, atol=2e-2)


def test_bf16_ring_needs_in_place_path():
    fx, model = _build("c1_t065", "float32")
    with pytest.raises(ValueError, match="in-place"):
        BatchDecoder(model, in_place=False, ring_dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="ring_dtype"):
        BatchDecoder(model, ring_dtype=torch.float16)


def test_state_round_trip_through_decode_state(cuda):
    fx, model = _build("c1_t065", "float32")
    out = model(fx["ids"].cuda())
    from koemi_5hom_b200.runtime import to_static_state
    static = to_static_state(out.state, 32, 32)
    back = to_koemi_state(from_koemi_state(static, 32, 32))
    for field in ("working_state", "local_keys", "local_values", "local_valid", "last_token_ids"):
        assert torch.equal(getattr(back, field), getattr(static, field)), field
    for (mk, mv), (rk, rv) in zip(ops.admitted_sequence(back.salient_keys, back.salient_values, back.salient_valid),
                                  ops.admitted_sequence(static.salient_keys, static.salient_values,
                                                        static.salient_valid)):
        assert torch.equal(mk, rk) and torch.equal(mv, rv)


@pytest.mark.parametrize("batch,length,d,m", [(3, 70, 256, 16), (2, 200, 100, 16), (4, 1, 64, 16), (5, 129, 2048, 16),
                                              (3, 70, 256, 4), (2, 90, 300, 8), (2, 70, 256, 32), (3, 65, 128, 12),
                                              (2, 40, 96, 20), (1, 33, 64, 5)])
def test_window_associative_kernel_matches_oracle(batch, length, d, m, cuda):
    """Prefill (window) associative read and update, fp32, against the oracle's
    sequential form; padded positions carry decay 1 and write 0 as the model
    passes them."""
    from oracle.herm import HermOracle
    from koemi_5hom_b200.cuda_kernels import _ops
    g = torch.Generator().manual_seed(batch * 1000 + length + m)
    basis = torch.randn(batch, d, m, generator=g) * 0.1
    normalizer = torch.rand(batch, m, generator=g)
    decay = 2.0 ** -12 + (1 - 2.0 ** -11) * torch.sigmoid(torch.randn(batch, length, generator=g))
    write = torch.sigmoid(torch.randn(batch, length, generator=g))
    pad = torch.rand(batch, length, generator=g) < 0.1
    decay, write = torch.where(pad, 1.0, decay), torch.where(pad, 0.0, write)
    value = torch.tanh(torch.randn(batch, length, d, generator=g))
    features = torch.softmax(torch.randn(batch, length, m, generator=g), -1)
    query = torch.softmax(torch.randn(batch, length, m, generator=g), -1)
    inputs = (basis, normalizer, decay, value, features, write, query)
    from koemi_5hom_b200.model.network import _associative_scan_read
    # 4, 8, 16, 32 features run the kernel directly, other counts zero-padded
    read, new_basis, new_norm = _associative_scan_read(*(t.to(cuda) for t in inputs))
    assert new_basis.shape == basis.shape and new_norm.shape == normalizer.shape
    expected = HermOracle._scan_read(None, *(t.double() for t in inputs))
    torch.testing.assert_close(read.cpu().double(), expected[0], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(new_basis.cpu().double(), expected[1], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(new_norm.cpu().double(), expected[2], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("carried,length", [(128, 128), (0, 128), (37, 100)])
def test_window_ring_reads_on_tensor_cores_match_fp32(carried, length, cuda):
    """The bf16 models' window ring reads (tcgen05 products with bf16
    operands, fp32 results) against the fp32 reads of the same stored values:
    within bf16 rounding of queries, keys, values and weights."""
    from koemi_5hom_b200.model.network import _local_read, _salient_read
    g = torch.Generator(device=cuda).manual_seed(carried + length)
    batch, d = 5, 256
    t = lambda *shape: torch.randn(*shape, generator=g, device=cuda)  # noqa: E731
    ck, cv, k, v, q = t(batch, carried, d), t(batch, carried, d), t(batch, length, d), t(batch, length, d), t(batch, length, d)
    cvalid = torch.rand(batch, carried, generator=g, device=cuda) > 0.3
    valid = torch.rand(batch, length, generator=g, device=cuda) > 0.2
    admission = torch.rand(batch, length, generator=g, device=cuda) > 0.5
    low = q.bfloat16()
    for low_q in (None, low):
        value, novelty = _local_read(ck, cv, cvalid, k, v, valid, q, 64, low_q)
        salient = _salient_read(ck, cv, cvalid, k, v, admission, q, low_q)
        if low_q is None:
            reference = (value, novelty, salient)
    for got, want in zip((value, novelty, salient), reference):
        assert (got - want).abs().max() <= 2e-2 * max(1.0, want.abs().max().item())
