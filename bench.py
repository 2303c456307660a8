"""HERM batched-decode benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (config 5): HERM stack with vocabulary 32768, d_model 2048, 24
blocks, memory features 16, 128 local + 128 salient ring slots, 64 experts
top-2 (d_ff 4096), bf16 weights, fp32 state, bf16 ring storage; 256 streams
in total, each with a 2048-token prompt of uniform random ids (PAD excluded),
prefilled untimed, then greedy decode (the native greedy sampler, PAD
masked). Weights are seeded random (N(0, 0.02)), inputs synthetic. One step =
one decode step of every stream (256 tokens) plus its sampler. The timed
region is K CUDA-graph replays of that step between barriers, timed with CUDA
events on the decode stream, max over ranks; every step reads far more than
the 126 MB L2, so no flush is needed.

Multi-GPU (config 5): one process per GPU (torchrun); the 256 streams are
split data-parallel (256/N per rank) and the 64 experts expert-parallel
(64/N per rank): per MoE block and step the expert rows go to their owners
and the outputs come back through peer-memory stores (CUDA IPC buffers and
epoch flags, inside the step's CUDA graph). The total work is fixed, so
``scaling`` is "strong". ``--weak`` keeps 256 streams per GPU with a full
replica per rank instead (no exchange on the step).

``--impl reference`` times the CPU oracle port of the same decode step on the
host cores (rank 0 only; the reference is Python and does not travel to the
GPU box) and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# ~140 GB stay live during the config-5 prefill; let the allocator grow segments
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

METRIC = "decode tokens/s at 1/2/4/8 B200; per-kernel % of HBM / tensor-core roofline"
UNIT = "tokens/s"


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--layers", type=int, default=24)
    p.add_argument("--streams", type=int, default=256,
                   help="decode streams in total (split over the ranks); per GPU with --weak")
    p.add_argument("--weak", action="store_true",
                   help="weak scaling: --streams per GPU, full model replica per rank, no expert parallelism")
    p.add_argument("--prompt-len", type=int, default=2048)
    p.add_argument("--vocab", type=int, default=32768)
    p.add_argument("--width", type=int, default=2048)
    p.add_argument("--experts", type=int, default=64)
    p.add_argument("--top-k", type=int, default=2)
    p.add_argument("--threshold", type=float, default=0.64,
                   help="salience threshold (fixed rule of network.py:349; ~mean+1 sigma at random init)")
    p.add_argument("--ring-dtype", choices=("bf16", "fp32"), default="bf16",
                   help="storage type of the exact-memory rings (arithmetic stays fp32)")
    p.add_argument("--cpu-sample-streams", type=int, default=4)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--out", type=str, default=None, help="also write the JSON line to this file")
    p.add_argument("--breakdown", type=str, default=None,
                   help="after the measurement, write per-kernel device times of 3 profiled decode steps "
                        "(torch profiler, CUDA activity) to this JSON file")
    p.add_argument("--op", choices=("scan", "rmsnorm", "moe", "moe_ep", "permute", "expert_decode", "surprise_decode",
                                    "surprise_prefill", "dense_decode", "window", "ring_decode"),
                   default=None, help="time one operator at its BASELINE shape instead of the decode step")
    p.add_argument("--op-rows", type=int, default=None,
                   help="activation rows of --op dense_decode (default 256; 32 is one rank's share at 8 GPUs)")
    p.add_argument("--op-tokens", type=int, default=None,
                   help="token count of --op moe (default: config 4's 131072; smaller for profiler captures)")
    return p.parse_args(argv)


def settings_for(args):
    from koemi_5hom_b200.model import ModelSettings
    return ModelSettings(vocabulary_size=args.vocab, embedding_size=args.width, memory_features=16,
                         local_memory_size=128, salience_memory_size=128, salience_threshold=args.threshold,
                         expert_count=args.experts, expert_top_k=args.top_k, scan_chunk=128,
                         layer_count=args.layers, compute_dtype="bfloat16")


def streams_per_rank(args, world: int) -> int:
    if args.weak:
        return args.streams
    if args.streams % world != 0:
        raise SystemExit(f"--streams {args.streams} does not split over {world} ranks")
    return args.streams // world


def expert_parallel(args, world: int) -> bool:
    return world > 1 and not args.weak


def workload_config(args, world):
    per_rank = streams_per_rank(args, world)
    parallelism = f"dp{world}+ep{world}" if expert_parallel(args, world) else f"dp{world}"
    return {"workload": "config5_herm_batched_decode", "model": "HERM (random init, N(0,0.02))",
            "layers": args.layers, "vocab": args.vocab, "d_model": args.width, "d_ff": 2 * args.width,
            "experts": args.experts, "top_k": args.top_k, "local_slots": 128, "salient_slots": 128,
            "streams_per_gpu": per_rank, "global_batch": per_rank * world, "prompt_len": args.prompt_len,
            "seq_len": 1, "salience_threshold": args.threshold, "parallelism": parallelism,
            "experts_per_gpu": args.experts // world if expert_parallel(args, world) else args.experts,
            "weights": "bf16", "state": "fp32", "rings": args.ring_dtype, "l2": "per-step reads >> 126 MB L2 (no flush needed)"}


def prompts_for(args, rank, world, device):
    """This rank's streams: rows [rank * n, (rank + 1) * n) of one seeded set
    of prompts for all streams (weak scaling: a seeded set per rank)."""
    import torch
    per_rank = streams_per_rank(args, world)
    if args.weak:
        g = torch.Generator().manual_seed(1000 + rank)
        ids = torch.randint(0, args.vocab - 1, (per_rank, args.prompt_len), generator=g)
    else:
        g = torch.Generator().manual_seed(1000)
        ids = torch.randint(0, args.vocab - 1, (per_rank * world, args.prompt_len), generator=g)
        ids = ids[rank * per_rank:(rank + 1) * per_rank]
    return torch.where(ids >= 256, ids + 1, ids).to(device)


# ------------------------------------------------------------ clock sampling
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.process = None

    def __enter__(self):
        try:
            self.process = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                             "--format=csv,noheader,nounits", "-lms", "50"],
                                            stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.process = None
        # nvidia-smi needs a few hundred ms before its first row: wait for it, so
        # that a short timed region (20 steps at 8 GPUs is ~0.1 s) is sampled,
        # and count only the rows written after this point
        deadline = time.perf_counter() + 3.0
        while self.process is not None and time.perf_counter() < deadline and os.path.getsize(self.file.name) == 0:
            time.sleep(0.01)
        self.mark()
        return self

    def mark(self) -> None:
        """The timed region starts here: rows written so far are not counted
        as inside it (call it after any barrier that follows ``__enter__``)."""
        self.start_offset = os.path.getsize(self.file.name)

    def __exit__(self, *exc):
        if self.process is not None:
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()
        self.file.flush()

    def summary(self) -> dict:
        rows, before = [], []
        with open(self.file.name) as handle:
            text = handle.read()
        for chunk, into in ((text[getattr(self, "start_offset", 0):], rows), (text[:getattr(self, "start_offset", 0)], before)):
            for line in chunk.splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    into.append(parts)
        os.unlink(self.file.name)
        adjacent = not rows and bool(before)
        if adjacent:  # no row inside the region: the last one taken just before it starts
            rows = before[-1:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower().startswith("active")})
        summary = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                   "reasons": reasons, "samples": 0 if adjacent else len(rows),
                   "power_w_max": max(float(r[3]) for r in rows)}
        if adjacent:
            summary["sampled"] = "the last row before the timed region (none fell inside it)"
        return summary


# ----------------------------------------------------------------- CPU side
class CpuBaseline:
    """The oracle port of the decode step on the host cores: a stack of
    ``layers`` HERM blocks of config-5 width for ``streams`` streams, each
    block with its own state (rings full of seeded random content), all blocks
    sharing one block's parameters (a host cannot hold 24 distinct fp32 expert
    sets of 6.4 GB; the work per block is the same). One step = one decode
    step of every sampled stream through every block and the head, then the
    greedy choice. Every parameter is drawn before any timing (one seeded
    generator per tensor, tensors drawn in parallel threads), so no step pays
    for materialising weights."""

    def __init__(self, args, streams: int):
        import concurrent.futures
        import zlib
        import torch
        sys.path.insert(0, str(ROOT / "tests" / "golden"))
        from herm_weights import HermShape, parameter_shapes
        from oracle.herm import HermConfig, HermOracle

        torch.set_num_threads(os.cpu_count() or 1)
        self.args, self.streams = args, streams
        s = settings_for(args)
        config = HermConfig(vocabulary_size=s.vocabulary_size, embedding_size=s.embedding_size,
                            memory_features=s.memory_features, local_memory_size=s.local_memory_size,
                            salience_memory_size=s.salience_memory_size, salience_threshold=s.salience_threshold,
                            expert_count=s.expert_count, expert_top_k=s.expert_top_k)
        shapes = {name: dims for name, dims, _ in
                  parameter_shapes(HermShape(s.vocabulary_size, s.embedding_size, s.memory_features, s.expert_count))}

        def draw(name):
            g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
            return (torch.randn(shapes[name], generator=g) * 0.02).bfloat16().float()

        started = time.perf_counter()
        with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as pool:
            params = dict(zip(shapes, pool.map(draw, list(shapes))))
        oracle = HermOracle.__new__(HermOracle)
        oracle.config, oracle.dtype, oracle.p = config, torch.float32, params
        keep = [i for i in range(s.vocabulary_size) if i != 256]
        oracle.content_w = params["token_predictor.weight"][keep]
        oracle.content_b = params["token_predictor.bias"][keep]
        g = torch.Generator().manual_seed(7)
        d = s.embedding_size
        self.states = []
        for _ in range(args.layers):
            state = oracle.initial_state(streams)
            for ring, size in (("local", s.local_memory_size), ("salient", s.salience_memory_size)):
                state[f"{ring}_keys"] = torch.randn(streams, size, d, generator=g)
                state[f"{ring}_values"] = torch.randn(streams, size, d, generator=g)
                state[f"{ring}_valid"] = torch.ones(streams, size, dtype=torch.bool)
            state["working_state"] = torch.randn(streams, d, generator=g) * 0.1
            self.states.append(state)
        self.oracle = oracle
        self.token = torch.randint(0, 255, (streams, 1), generator=g)
        self.cores = torch.get_num_threads()
        self.setup_s = time.perf_counter() - started

    def step(self) -> float:
        """One decode step of the sampled streams through the whole stack."""
        started = time.perf_counter()
        context = None
        top = len(self.states) - 1
        for layer, state in enumerate(self.states):
            out = self.oracle.window(self.token, state, context=context, logits=layer == top)
            self.states[layer] = out["state"]
            context = out["final"]
        self.token = self.oracle.greedy(out["logits"][:, -1])
        return time.perf_counter() - started

    def measure(self, warmup: int, steps: int) -> dict:
        for _ in range(warmup):
            self.step()
        times = [self.step() for _ in range(steps)]
        per_step = statistics.median(times)
        return {"value": self.streams / per_step, "unit": UNIT, "cores": self.cores, "kind": "port",
                "seconds_per_step": per_step, "timed_s": sum(times),
                "sample": (f"oracle port (torch CPU fp32, {self.cores} threads): {self.streams} of the 256 streams "
                           f"through all {self.args.layers} config-5 blocks (one block's parameters shared by every "
                           f"block, each block its own state) and the head, median of {steps} decode steps after "
                           f"{warmup} warm-up = {per_step:.2f} s per step; parameters drawn before timing")}


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    started = time.perf_counter()
    baseline = CpuBaseline(args, args.cpu_sample_streams)
    result = baseline.measure(args.warmup, args.steps)
    value = result["value"]
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": result["seconds_per_step"] * 1000.0,
            "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": workload_config(args, world),
            "cpu_baseline": {"kind": "port", "cores": result["cores"], "sample": result["sample"], "value": value,
                             "unit": UNIT},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "streams_sampled": args.cpu_sample_streams, "timed_region_s": result["timed_s"],
            "setup_s": baseline.setup_s, "wall_s": time.perf_counter() - started}
    emit(line, args)


def emit(line: dict, args) -> None:
    text = json.dumps(line)
    print(text, flush=True)
    if args.out:
        Path(args.out).write_text(text + "\n")


# ----------------------------------------------------------------- GPU side
class GreedyTokens:
    """The greedy sampler of the decode loop: TokenSampler's greedy path (PAD
    masked, first index among equal maxima) as one native pass over the
    logits, called through the C ABI into a reused output (no op dispatch on
    the host between steps)."""

    def __init__(self):
        self._out = None

    def __call__(self, logits):
        import torch
        from koemi_5hom_b200 import _native
        from koemi_5hom_b200.model.settings import PAD_TOKEN_ID
        flat = logits.reshape(-1, logits.shape[-1])
        if flat.dtype != torch.float32 or not flat.is_contiguous():
            flat = flat.float().contiguous()
        rows, vocab = flat.shape
        if self._out is None or self._out.shape[0] != rows or self._out.device != flat.device:
            self._out = torch.empty(rows, 1, dtype=torch.int64, device=flat.device)
        _native.call("koemi_sampler_greedy", flat.data_ptr(), rows, vocab, vocab, PAD_TOKEN_ID,
                     self._out.data_ptr(), torch.cuda.current_stream(flat.device).cuda_stream)
        return self._out



def count_native_kernels(model, decoder, token) -> int:
    """Kernels of libkoemi_b200 launched by one eager decode step (on a copy of
    the decoder's state, so the measured run is not advanced)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    from koemi_5hom_b200.model.decode import decode_step
    from koemi_5hom_b200.runtime.fast_decode import clone_state
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        if decoder._dstate is not None:
            decode_step(model, token, decoder._dstate.clone())
        else:
            model(token, clone_state(decoder._state), trusted_inputs=True)
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "koemi" in e.name)


def measure_expert_mlp(model, args, world: int, repeats: int = 20) -> dict:
    """Time the dominant kernel (grouped expert MLP of block 0, this rank's
    experts) alone, CUDA events on its stream, on the pairs a decode step of
    all streams routes to those experts (a seeded draw of ids: the owner's
    rows under expert parallelism, all pairs on one GPU)."""
    import torch
    from koemi_5hom_b200.cuda_kernels import _ops
    s = model.settings
    block = model.blocks[0]
    local = block.expert_gate_weight.shape[0]
    first = block.expert_first
    tokens = streams_per_rank(args, world) * world if expert_parallel(args, world) else streams_per_rank(args, world)
    g = torch.Generator(device="cuda").manual_seed(5)
    context = torch.randn(tokens, s.embedding_size, device="cuda", generator=g).bfloat16()
    ids = torch.randint(0, s.vocabulary_size, (tokens,), device="cuda", generator=g)
    prev = torch.randint(0, s.vocabulary_size, (tokens,), device="cuda", generator=g)
    valid = torch.ones(tokens, dtype=torch.bool, device="cuda")
    assignments = _ops.route_topk(ids, prev, valid, s.expert_count, s.expert_top_k)
    owned = (assignments >= first) & (assignments < first + local)
    local_ids = torch.where(owned, assignments - first, -1)
    sc, _, se, offsets, _ = _ops.permute_topk(context, local_ids, valid, local, True)
    args_mlp = (sc, se, offsets) + block.expert_weights()
    for _ in range(3):
        _ops.grouped_expert_mlp(*args_mlp)
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(repeats):
        _ops.grouped_expert_mlp(*args_mlp)
    stop.record(stream)
    torch.cuda.synchronize()
    seconds = start.elapsed_time(stop) / 1000.0 / repeats
    counts = torch.diff(offsets).cpu()
    touched = int((counts > 0).sum())
    d, h = s.embedding_size, 2 * s.embedding_size
    pairs = int(offsets[-1])
    weight_bytes = touched * 3 * d * h * 2 + touched * (2 * h + d) * 2
    activation_bytes = pairs * d * 2 * 2 + pairs * h * 2 * 2
    algorithmic = weight_bytes + activation_bytes
    return {"seconds": seconds, "bytes": algorithmic, "touched_experts": touched, "pairs": pairs}


def prefill_roofline(args, streams: int, seconds: float, world: int) -> dict:
    """Prefill rate and its fraction of the tensor-core bound: per token and
    block the surprise head (2 d C), the two expert pairs (2 x 6 d d_ff) and the
    dense projections (gates 4 d^2, local 4 d^2, associative 2 (3d + 2) d,
    fusion 8 d^2) in FLOPs, at the sustained bf16 peak of every GPU."""
    d, c = args.width, args.vocab - 1
    per_token_block = 2 * d * c + args.top_k * 6 * d * (2 * d) + (4 + 4 + 8) * d * d + 2 * (3 * d + 2) * d
    tokens = streams * args.prompt_len
    flop = per_token_block * args.layers * tokens
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    peak = peaks.get("bf16_tflops_sustained", 1409.6) * 1e12 * world
    return {"tokens_per_s": tokens / seconds, "tensor_flop": flop, "bound_s": flop / peak,
            "frac_of_tensor_bound": flop / peak / seconds,
            "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained" if peaks else "fallback 1409.6 TFLOP/s"}


def write_breakdown(path: str, rank: int, world: int, step, steps: int = 3) -> None:
    """Per-kernel device time of ``steps`` decode steps under the torch
    profiler (CUDA activity only), averaged per step, largest first; one file
    per rank (``path`` gets ``.rank<r>`` inserted when world > 1)."""
    import torch
    from collections import defaultdict
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
    totals = defaultdict(lambda: [0, 0.0])
    for event in prof.events():
        if event.device_type.name == "CUDA":
            totals[event.name][0] += 1
            totals[event.name][1] += event.device_time_total
    rows = sorted(totals.items(), key=lambda kv: -kv[1][1])
    out = {"steps": steps, "kernel_us_per_step": sum(v[1] for v in totals.values()) / steps,
           "kernels": [{"name": name, "launches_per_step": count / steps, "us_per_step": us / steps}
                       for name, (count, us) in rows]}
    target = Path(path) if world == 1 else Path(path).with_suffix(f".rank{rank}{Path(path).suffix}")
    target.write_text(json.dumps(out, indent=1))


def progress(rank: int, message: str) -> None:
    """Timestamped, rank-tagged progress on stderr (the JSON line stays alone on stdout)."""
    print(f"[bench rank {rank} {time.strftime('%H:%M:%S')}] {message}", file=sys.stderr, flush=True)


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.model import KoemiModel
    from koemi_5hom_b200.runtime import BatchDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    _native.ensure_device(device)
    wall_start = time.perf_counter()

    shard = None
    if expert_parallel(args, world):
        from koemi_5hom_b200.model.expert_parallel import ExpertShard
        shard = ExpertShard.from_group(args.experts)
    per_rank = streams_per_rank(args, world)
    model = KoemiModel(settings_for(args), device=device, expert_shard=shard)
    model.initialize_parameters(seed=0)
    prompts = prompts_for(args, rank, world, device)
    ring_dtype = torch.bfloat16 if args.ring_dtype == "bf16" else torch.float32
    decoder = BatchDecoder(model, capture_graph=True, ring_dtype=ring_dtype)
    # the process's first forward pays one-time costs (kernel loading, library
    # handles, the caching allocator growing to the window's working set):
    # run two windows once, untimed for the prefill rate, reported apart
    torch.cuda.synchronize()
    first_start = time.perf_counter()
    with torch.no_grad():
        warm = model(prompts[:, :2 * model.settings.scan_chunk], trusted_inputs=True, last_logits_only=True)
    del warm
    torch.cuda.synchronize()
    first_call_seconds = time.perf_counter() - first_start
    prefill_start = time.perf_counter()
    logits = decoder.prefill(prompts)
    torch.cuda.synchronize()
    prefill_seconds = time.perf_counter() - prefill_start
    progress(rank, f"prefill done in {prefill_seconds:.1f} s (first two windows of the process: {first_call_seconds:.1f} s)")
    del prompts

    greedy = GreedyTokens()
    token = greedy(logits)
    eager_kernels = count_native_kernels(model, decoder, token)
    progress(rank, f"eager step counted {eager_kernels} native launches")
    for _ in range(max(args.warmup, 1)):
        logits = decoder.step(token)
        token = greedy(logits)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the sampler starts (and waits for its first row) before the barrier, so
    # the ranks leave the barrier together and enter the timed region at once
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        progress(rank, "graph captured and warmed up; timing")
        clocks.mark()
        torch.cuda.nvtx.range_push("decode_timed")
        start.record(stream)
        for _ in range(args.steps):
            logits = decoder.step(token)
            token = greedy(logits)
        stop.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    seconds = start.elapsed_time(stop) / 1000.0
    clock_summary = clocks.summary()
    if world > 1:
        t = torch.tensor([seconds], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        seconds = float(t.item())
    ms_per_step = seconds / args.steps * 1000.0
    value = per_rank * world * args.steps / seconds

    # end to end: pinned host ids in, sampled ids back to the host, every step
    host_in = torch.empty(per_rank, 1, dtype=torch.long).pin_memory()
    host_out = torch.empty(per_rank, 1, dtype=torch.long).pin_memory()
    host_in.copy_(token.cpu())
    device_ids = torch.empty_like(token)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    progress(rank, "timed steps done; end-to-end steps")
    e2e_start = time.perf_counter()
    for _ in range(args.steps):
        device_ids.copy_(host_in, non_blocking=True)
        logits = decoder.step(device_ids)
        host_out.copy_(greedy(logits), non_blocking=True)
        stream.synchronize()
        host_in.copy_(host_out)
    e2e_seconds = time.perf_counter() - e2e_start
    if world > 1:
        t = torch.tensor([e2e_seconds], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_seconds = float(t.item())
    e2e_value = per_rank * world * args.steps / e2e_seconds

    # the config's sampled variant: temperature 0.8, seeded per stream (the
    # native counter-based sampler; stream ids are global across ranks)
    from koemi_5hom_b200.runtime import SamplingPolicy, TokenSampler
    sampler = TokenSampler(SamplingPolicy(temperature=0.8), device, stream_seed=2024, stream_offset=rank * per_rank)
    token = sampler(logits)
    for _ in range(max(args.warmup, 1)):
        token = sampler(decoder.step(token))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        token = sampler(decoder.step(token))
    stop.record(stream)
    torch.cuda.synchronize()
    sampled_seconds = start.elapsed_time(stop) / 1000.0
    if world > 1:
        t = torch.tensor([sampled_seconds], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sampled_seconds = float(t.item())

    if args.breakdown:
        write_breakdown(args.breakdown, rank, world, lambda: greedy(decoder.step(token)))

    progress(rank, "end-to-end done; expert kernel roofline")
    mlp = measure_expert_mlp(model, args, world)
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    achieved = mlp["bytes"] / mlp["seconds"] / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": workload_config(args, world),
        "clocks": clock_summary,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": host_in.numel() * 8,
                "d2h_bytes_per_step": host_out.numel() * 8},
        "gpu_launches": eager_kernels * args.steps,
        "roofline": {"kernel": "koemi_moe_grouped_expert_mlp (decode step, one block)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm_peak,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650 GB/s",
                     "unit": "GB/s", "frac": achieved / hbm_peak,
                     # dram__bytes_read.sum + dram__bytes_write.sum of both expert GEMMs for one call at this
                     # workload's pair distribution (512 pairs, 64 experts), from one ncu capture of
                     # `bench.py --op expert_decode` (2,163,557,888 B for the gated GEMM, 1,082,892,544 B for
                     # the output GEMM, first launches under ncu); none was taken of an expert-parallel
                     # owner's share
                     "traffic": 3246450432 if not expert_parallel(args, world) else None,
                     "traffic_unit": "bytes per launch",
                     "algorithmic_bytes": mlp["bytes"], "launch_us": mlp["seconds"] * 1e6,
                     "touched_experts": mlp["touched_experts"], "pairs": mlp["pairs"]},
        "prefill_s": prefill_seconds,
        "prefill_first_call_s": first_call_seconds,
        "prefill": prefill_roofline(args, per_rank * world, prefill_seconds, world),
        "sampled": {"policy": "temperature 0.8, seeded per stream (native Gumbel-max)",
                    "value": per_rank * world * args.steps / sampled_seconds,
                    "ms_per_step": sampled_seconds / args.steps * 1000.0},
    }
    # the step graph (which may hold collectives) and the peer buffers go
    # before the process group
    del decoder, logits
    torch.cuda.synchronize()
    model.close_exchanges()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.cuda.empty_cache()
        # a bounded sample (about 20 s of CPU work): the same step as the
        # reference arm, fewer of them
        line["cpu_baseline"] = CpuBaseline(args, args.cpu_sample_streams).measure(1, 4)
    line["wall_s"] = time.perf_counter() - wall_start
    if rank == 0:
        emit(line, args)
    progress(rank, "done")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------- operators
def _time_op(fn, steps: int, warmup: int, graph: bool = False) -> float:
    """Seconds per call of fn, CUDA events on the current stream. With
    graph=True the calls are captured into one CUDA graph and replayed, so
    host dispatch cost does not hide the kernel time of short launches."""
    import torch
    for _ in range(max(warmup, 1)):
        fn()
    stream = torch.cuda.current_stream()
    if graph:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            with torch.cuda.graph(g):
                for _ in range(steps):
                    fn()
        stream.wait_stream(side)
        g.replay()
        run = g.replay
    else:
        def run():
            for _ in range(steps):
                fn()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    run()
    stop.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / 1000.0 / steps


def run_op(args) -> None:
    """One operator at its BASELINE.json shape, CUDA-event timed; inputs are
    larger than L2 (stated per op), so back-to-back launches read HBM."""
    import torch
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.cuda_kernels import _ops
    device = torch.device("cuda", 0)
    _native.ensure_device(device)
    g = torch.Generator(device=device).manual_seed(0)
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    hbm, tensor = peaks.get("hbm_gbs", 6650.0), peaks.get("bf16_tflops", 1590.0)
    if args.op == "scan":  # config 2: B=8, T=4096, D=1024, a = sigmoid(N(0,1)), b ~ N(0,1), h0 = 0
        a = torch.sigmoid(torch.randn(8, 4096, 1024, device=device, generator=g)).bfloat16()
        b = torch.randn(8, 4096, 1024, device=device, generator=g).bfloat16()
        h0 = torch.zeros(8, 1024, device=device, dtype=torch.bfloat16)
        seconds = _time_op(lambda: _ops.affine_scan_forward(a, b, h0, False), args.steps, args.warmup, graph=True)
        work, unit, peak, bound = 3 * a.numel() * 2 / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = "B=8 T=4096 D=1024 bf16 (201 MB per launch > L2)"
    elif args.op == "rmsnorm":  # config 3: 65536 x 2048 bf16, gated form silu(gate) * rmsnorm(x) * w
        x = torch.randn(65536, 2048, device=device, generator=g).bfloat16()
        gate = torch.randn(65536, 2048, device=device, generator=g).bfloat16()
        w = (1.0 + 0.02 * torch.randn(2048, device=device, generator=g)).bfloat16()
        seconds = _time_op(lambda: _ops.gated_rmsnorm_silu(x, gate, w, 1e-6), args.steps, args.warmup, graph=True)
        work, unit, peak, bound = 3 * x.numel() * 2 / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = "65536 x 2048 bf16, gated (805 MB per launch > L2)"
    elif args.op in ("moe", "expert_decode"):
        tokens, d, e = (args.op_tokens or 131072, 1024, 64) if args.op == "moe" else (256, 2048, 64)
        h = 2 * d
        x = torch.randn(tokens, d, device=device, generator=g).bfloat16()
        ids = torch.randint(0, 256, (tokens,), device=device, generator=g)
        prev = torch.randint(0, 256, (tokens,), device=device, generator=g)
        valid = torch.ones(tokens, dtype=torch.bool, device=device)
        weights = [(torch.randn(*s, device=device, generator=g) * 0.02).bfloat16() for s in
                   ((e, h, d), (e, h), (e, h, d), (e, h), (e, d, h), (e, d))]
        assignments = _ops.route_topk(ids, prev, valid, e, 2)
        sc, _, se, offsets, _ = _ops.permute_topk(x, assignments, valid, e, True)
        seconds = _time_op(lambda: _ops.grouped_expert_mlp(sc, se, offsets, *weights), args.steps, args.warmup)
        pairs = int(offsets[-1])
        if args.op == "moe":
            work, unit, peak, bound = pairs * 6 * d * h / seconds / 1e12, "TFLOP/s", tensor, "tensor"
            shape = f"config 4: {tokens} tokens, {pairs} pairs, d={d}, d_ff={h}, E={e}, top-2 (hash route)"
        else:
            touched = int((torch.diff(offsets) > 0).sum())
            moved = touched * 3 * d * h * 2 + pairs * (2 * d + 4 * h) * 2
            work, unit, peak, bound = moved / seconds / 1e9, "GB/s", hbm, "hbm"
            shape = f"config 5 decode step: {pairs} pairs, {touched} experts touched, d={d}, d_ff={h} (3.2 GB weights > L2)"
    elif args.op == "permute":  # config 4's stable permutation with the row gather (262144 pairs, d=1024 bf16)
        tokens, d, e = args.op_tokens or 131072, 1024, 64
        x = torch.randn(tokens, d, device=device, generator=g).bfloat16()
        ids = torch.randint(0, 256, (tokens,), device=device, generator=g)
        prev = torch.randint(0, 256, (tokens,), device=device, generator=g)
        valid = torch.ones(tokens, dtype=torch.bool, device=device)
        assignments = _ops.route_topk(ids, prev, valid, e, 2)
        seconds = _time_op(lambda: _ops.permute_topk(x, assignments, valid, e, True), args.steps, args.warmup,
                           graph=True)
        pairs = tokens * 2
        # context read once, sorted rows written, assignments read, sorted rows / experts / positions written
        moved = tokens * d * 2 + pairs * d * 2 + pairs * 8 + 3 * pairs * 8 + (e + 1) * 8
        work, unit, peak, bound = moved / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = f"config 4: {tokens} tokens x d={d} bf16, hash top-2 over {e} experts ({moved / 1e6:.0f} MB per call)"
    elif args.op == "dense_decode":  # the four dense projections of one config-5 decode block
        shapes = {"gates": (4096, 2048), "local": (4096, 2048), "assoc": (6146, 2048), "fusion": (2048, 8192),
                  "local_assoc": (10242, 2048)}  # the last: local and assoc as one GEMM (not in the block total)
        sets = 4  # weight sets cycled so each launch reads its weights from HBM (4 x 75 MB > L2)
        layers = [{name: ((torch.randn(n, k, device=device, generator=g) * 0.02).bfloat16(),
                          torch.zeros(n, device=device, dtype=torch.bfloat16)) for name, (n, k) in shapes.items()}
                  for _ in range(sets)]
        rows = args.op_rows or 256
        inputs = {k: torch.randn(rows, k, device=device, generator=g).bfloat16() for k in (2048, 8192)}
        per = {}
        for name, (n, k) in shapes.items():
            counter = iter(range(1 << 30))
            # as the model calls it: parameters, so the next launch may load its
            # weights while the previous one finishes
            fn = lambda name=name, k=k: _ops.dense_projection(  # noqa: E731
                inputs[k], *layers[next(counter) % sets][name], True)
            t = _time_op(fn, args.steps, args.warmup, graph=True)
            counter_plain = iter(range(1 << 30))
            plain = lambda name=name, k=k: _ops.dense_projection(  # noqa: E731
                inputs[k], *layers[next(counter_plain) % sets][name])
            t_plain = _time_op(plain, args.steps, args.warmup, graph=True)
            counter_lib = iter(range(1 << 30))
            library = lambda name=name, k=k: torch.mm(  # noqa: E731
                inputs[k], layers[next(counter_lib) % sets][name][0].t(), out_dtype=torch.float32)
            t_lib = _time_op(library, args.steps, args.warmup, graph=True)
            per[name] = {"us": t * 1e6, "gbs": (n * k * 2 + rows * k * 2 + rows * n * 4) / t / 1e9,
                         "us_without_early_weights": t_plain * 1e6, "cublas_us_no_bias": t_lib * 1e6}
        block = ("gates", "local", "assoc", "fusion")
        seconds = sum(per[name]["us"] for name in block) / 1e6
        moved = sum(n * k * 2 + rows * k * 2 + rows * n * 4 for name, (n, k) in shapes.items() if name in block)
        work, unit, peak, bound = moved / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = f"config 5 decode block: {rows} rows; gates 4096x2048, local 4096x2048, assoc 6146x2048, " \
                "fusion 2048x8192 bf16 -> fp32"
        extra = {"per_projection": per}
    elif args.op == "ring_decode":  # both exact-memory rings of one config-5 decode block, full, bf16
        batch, d, slots = 256, 2048, 128
        rings = [(torch.randn(batch, slots, d, device=device, generator=g) * 0.1).bfloat16() for _ in range(4)]
        valid_slots = [torch.ones(batch, slots, dtype=torch.uint8, device=device) for _ in range(2)]
        head = torch.zeros(1, dtype=torch.int64, device=device)
        s_head = torch.zeros(batch, dtype=torch.int32, device=device)
        s_count = torch.full((batch,), slots, dtype=torch.int32, device=device)
        queries = torch.randn(batch, d, device=device, generator=g)
        entries = torch.randn(batch, 2 * d, device=device, generator=g) * 0.1
        valid = torch.ones(batch, dtype=torch.uint8, device=device)
        surprise = torch.zeros(batch, device=device)  # nothing admitted: the salient ring stays full
        out = torch.empty(batch, 2 * d, dtype=torch.bfloat16, device=device)
        novelty = torch.empty(batch, device=device)
        seconds = _time_op(lambda: _native.call(
            "koemi_think_ring_decode_step", queries.data_ptr(), d, entries.data_ptr(), 2 * d, valid.data_ptr(),
            surprise.data_ptr(), 0.64, rings[0].data_ptr(), rings[1].data_ptr(), valid_slots[0].data_ptr(),
            head.data_ptr(), rings[2].data_ptr(), rings[3].data_ptr(), valid_slots[1].data_ptr(), s_head.data_ptr(),
            s_count.data_ptr(), out.data_ptr(), out[:, d:].data_ptr(), 2 * d, novelty.data_ptr(), None, batch, d,
            slots, slots, _native.BF16, _native.BF16, _native.stream_of(queries)), args.steps, args.warmup, graph=True)
        moved = 4 * batch * slots * d * 2 + batch * d * 4 + batch * 2 * d * 2
        work, unit, peak, bound = moved / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = f"config-5 decode block: {batch} streams, local + salient rings of {slots} bf16 slots, d={d}, all valid"
    elif args.op == "window":  # the prefill window's bandwidth kernels, config-5 window shape
        batch, length, d, m, carried = 256, 128, 2048, 16, 128
        rows, padded = batch * length, carried + length
        t = lambda *shape: torch.randn(*shape, device=device, generator=g)  # noqa: E731
        ring_k, ring_v, keys, values = t(batch, carried, d), t(batch, carried, d), t(batch, length, d), t(batch, length, d)
        basis, norm = t(batch, d, m) * 0.1, torch.rand(batch, m, device=device, generator=g)
        decay = torch.sigmoid(t(batch, length)) * 0.5 + 0.5
        write = torch.sigmoid(t(batch, length))
        feats = torch.softmax(t(batch, length, m), -1)
        query = torch.softmax(t(batch, length, m), -1)
        pre = t(rows, 2 * d)
        valid = torch.ones(rows, dtype=torch.bool, device=device)
        parts = [t(rows, d) for _ in range(4)]
        fusion_in = torch.empty(rows, 4 * d, dtype=torch.bfloat16, device=device)
        queries = t(rows, d).bfloat16()
        weights = torch.softmax(t(rows, padded), -1).bfloat16()
        stacked, transposed = _ops.window_slot_operands(ring_k, ring_v, keys, values, padded, torch.bfloat16)
        read_out = torch.empty_like(values)
        f32, b16 = 4, 2
        kernels = {
            # name: (call, algorithmic bytes per launch)
            # through the C ABI in place (the op clones the state first)
            "assoc_window_scan_read": (
                lambda: _native.call("koemi_assoc_window_scan_read", decay.data_ptr(), write.data_ptr(),
                                     values.data_ptr(), feats.data_ptr(), query.data_ptr(), basis.data_ptr(),
                                     norm.data_ptr(), read_out.data_ptr(), batch, length, d, m,
                                     _native.stream_of(values)),
                2 * rows * d * f32 + 2 * batch * d * m * f32 + 2 * rows * m * f32 + 2 * rows * f32),
            "window_slot_operands": (
                lambda: _ops.window_slot_operands(ring_k, ring_v, keys, values, padded, torch.bfloat16),
                2 * batch * padded * d * f32 + 2 * batch * padded * d * b16),
            "pack_rows_fusion_input": (lambda: _ops.pack_rows(fusion_in, parts), 4 * rows * d * (f32 + b16)),
            "bounded_gates": (lambda: _ops.bounded_gates(pre, valid, 0.05, 0.995),
                              rows * 2 * d * f32 + 2 * rows * d * f32 + rows),
            "ring_scores_grouped_projection": (
                lambda: _ops.grouped_projection(queries, stacked.view(batch * padded, d), batch),
                rows * d * b16 + batch * padded * d * b16 + rows * padded * f32),
            "ring_read_grouped_projection": (
                lambda: _ops.grouped_projection(weights, transposed.view(batch * d, padded), batch),
                rows * padded * b16 + batch * d * padded * b16 + rows * d * f32),
        }
        per = {}
        for name, (fn, nbytes) in kernels.items():
            t_op = _time_op(fn, args.steps, args.warmup, graph=True)
            per[name] = {"us": t_op * 1e6, "gbs": nbytes / t_op / 1e9, "frac": nbytes / t_op / 1e9 / hbm,
                         "bytes": nbytes}
        seconds = sum(v["us"] for v in per.values()) / 1e6
        moved = sum(v["bytes"] for v in per.values())
        work, unit, peak, bound = moved / seconds / 1e9, "GB/s", hbm, "hbm"
        shape = (f"config-5 prefill window: {batch} streams x {length} positions, d={d}, {m} memory features, "
                 f"{carried} carried ring slots (every input > L2)")
        extra = {"per_kernel": per}
    else:  # surprise head: decode (256 rows) or one prefill window (32768 rows) of config 5
        rows = 256 if args.op == "surprise_decode" else 32768
        prior = torch.randn(rows, 2048, device=device, generator=g).bfloat16()
        weight = (torch.randn(32767, 2048, device=device, generator=g) * 0.02).bfloat16()
        bias = (torch.randn(32767, device=device, generator=g) * 0.002).bfloat16()
        targets = torch.randint(0, 32767, (rows,), device=device, generator=g)
        valid = torch.ones(rows, dtype=torch.bool, device=device)
        seconds = _time_op(lambda: _ops.causal_surprise_forward(prior, weight, bias, targets, valid, torch.float32),
                           args.steps, args.warmup)
        if args.op == "surprise_decode":
            work, unit, peak, bound = (weight.numel() * 2 + prior.numel() * 2) / seconds / 1e9, "GB/s", hbm, "hbm"
        else:
            work, unit, peak, bound = 2 * rows * 32767 * 2048 / seconds / 1e12, "TFLOP/s", tensor, "tensor"
        shape = f"{rows} rows x d=2048 against the 32767-row content head (134 MB bf16 > L2)"
    line = {"op": args.op, "shape": shape, "us_per_launch": seconds * 1e6, **locals().get("extra", {}),
            "roofline": {"bound": bound, "achieved": work, "peak": peak, "unit": unit, "frac": work / peak,
                         "peak_source": "MEASURED_PEAKS.json (burst)" if peaks else "fallback"}}
    emit(line, args)


def run_op_moe_parallel(args) -> None:
    """Config 4 (MoE dispatch + experts) over N ranks: 131072 tokens in total
    split data-parallel (131072 / N per rank), the 64 experts split
    expert-parallel (64 / N per rank, 8 per GPU at N = 8). One step per rank =
    hash route -> stable permutation -> NCCL all-to-all of the rows to their
    experts' owners (exact per-owner counts) -> grouped expert MLP of the
    owner's experts -> all-to-all back -> combine (sum / k). Before timing,
    every rank checks its step's output bit for bit against the grouped MLP
    of all 64 experts on one GPU (each rank also draws the full expert set,
    805 MB, for that check). Timed with CUDA events over K steps between
    barriers, max over ranks; the job's rate counts every rank's pairs."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.cuda_kernels import _ops
    from koemi_5hom_b200.model.expert_parallel import ExpertShard, expert_parallel_mlp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    _native.ensure_device(device)
    total_tokens = args.op_tokens or 131072
    if total_tokens % world or 64 % world:
        raise SystemExit(f"{total_tokens} tokens / 64 experts do not split over {world} ranks")
    tokens, d, h, e, k = total_tokens // world, 1024, 2048, 64, 2
    shard = ExpertShard.from_group(e) if world > 1 else None
    first, held = (shard.first, shard.local_count) if shard is not None else (0, e)

    def expert_tensors(lo: int, hi: int) -> tuple:
        """Experts [lo, hi) in grouped-MLP order, each drawn from its own seed
        (a shard holds exactly the rows of the full set)."""
        shapes = ((h, d), (h,), (h, d), (h,), (d, h), (d,))
        out = [torch.empty(hi - lo, *shape, dtype=torch.bfloat16, device=device) for shape in shapes]
        for j, expert in enumerate(range(lo, hi)):
            g = torch.Generator(device=device).manual_seed(4000 + expert)
            for tensor, scale in zip(out, (0.02, 0.002, 0.02, 0.002, 0.02, 0.002)):
                tensor[j].copy_(torch.randn(tensor.shape[1:], generator=g, device=device) * scale)
        return tuple(out)

    weights = expert_tensors(first, first + held)
    g = torch.Generator(device=device).manual_seed(100 + rank)
    x = torch.randn(tokens, d, device=device, generator=g).bfloat16()
    ids = torch.randint(0, 256, (tokens,), device=device, generator=g)
    prev = torch.randint(0, 256, (tokens,), device=device, generator=g)
    valid = torch.ones(tokens, dtype=torch.bool, device=device)

    def step(expert_set=weights, sharded=shard):
        assignments = _ops.route_topk(ids, prev, valid, e, k)
        sc, rows, se, offsets, _ = _ops.permute_topk(x, assignments, valid, e, True)
        if sharded is not None:
            y = expert_parallel_mlp(sharded, sc, se, offsets, expert_set, mode="exact")
        else:
            y = _ops.grouped_expert_mlp(sc, se, offsets, *expert_set)
        return _ops.combine_topk(y, rows, offsets, tokens, k)

    full = expert_tensors(0, e)
    expected = step(full, None)
    got = step()
    exact = bool(torch.equal(got, expected))
    del full, expected, got
    torch.cuda.empty_cache()
    for _ in range(max(args.warmup, 1)):
        step()
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    seconds = start.elapsed_time(stop) / 1000.0 / args.steps
    flags = torch.tensor([seconds, 0.0 if exact else 1.0], device=device)
    if world > 1:
        dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    seconds, mismatch = float(flags[0]), bool(flags[1] > 0)
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    peak = peaks.get("bf16_tflops_sustained", 1409.6)
    pairs_total = total_tokens * k
    job_tflops = pairs_total * 6 * d * h / seconds / 1e12
    line = {"op": "moe_ep", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "shape": f"config 4: {total_tokens} tokens x d={d} bf16, hash top-2 over {e} experts (d_ff {h}); "
                     f"{tokens} tokens and {held} experts per GPU",
            "parallelism": f"dp{world}+ep{world}" if world > 1 else "dp1",
            "exchange": "NCCL all_to_all_single, exact per-owner counts" if world > 1 else "none",
            "us_per_step": seconds * 1e6, "pairs_total": pairs_total, "job_tflops": job_tflops,
            "parity": "bit-exact with the single-GPU grouped MLP of all experts on every rank's tokens"
                      if not mismatch else "MISMATCH against the single-GPU grouped MLP",
            "roofline": {"bound": "tensor", "achieved": job_tflops / world, "peak": peak, "unit": "TFLOP/s per GPU",
                         "frac": job_tflops / world / peak,
                         "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained" if peaks else "fallback",
                         "work": "expert FLOPs only (6 d d_ff per pair); route, permutation, exchange and combine "
                                 "are inside the timed step"}}
    if rank == 0:
        emit(line, args)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if mismatch:
        raise SystemExit("expert-parallel MoE step differs from the single-GPU result")


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.op == "moe_ep":
        run_op_moe_parallel(args)
        return
    if args.op is not None:
        run_op(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
