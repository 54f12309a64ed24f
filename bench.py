"""Benchmark: qwen3tts talker decode on B200 — codec frames/s at 48 lanes (benchmark config[2]).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One step = one talker decode step for 48 lanes: 28 Qwen3 layers (dim 2048, 16/8 heads,
head_dim 128, SwiGLU 6144, f16 weights ~N(0, 0.02), RMSNorm, RoPE theta 1e6, paged KV with
lane lengths ~U[64, 1024]), the final norm, 16 codebook heads x 2048 with a greedy pick, and the
next input as the sum of the picked codes' embedding rows. Every lane emits one 12.5 Hz codec
frame per step, so frames/s = lanes x steps/s. The step runs as one captured CUDA graph.

Under torchrun each rank drives its own GPU with its own 48 lanes (data parallel, weights
replicated, no collective on the data path): `value` is frames/s over all ranks, timed on the
device as the max over ranks. `--impl reference` times the CPU restatement of the reference's
CPU path (oracle/, the only runnable form of the reference here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "dream-tts_b200"))
sys.path.insert(0, ROOT)

METRIC = "codec frames/sec (48-lane decode, whole box)"
UNIT = "frames/s"
LANES, LAYERS, DIM, HEADS, N_KV, HD, FFN, CB, VOCAB = 48, 28, 2048, 16, 8, 128, 6144, 16, 2048
BLOCK = 32
# DRAM bytes (read + write) of one gate/up launch at 48 lanes, from its ncu capture
GATEUP_NCU_TRAFFIC = 50_606_336 + 6_912
# the same for one attention launch of the config[2] step (KV lengths U[64,1024] seed 0 + 1)
ATTN_NCU_TRAFFIC = 103_285_760 + 3_062_016
ATTN_BYTES_PER_POS = N_KV * HD * 2 * 2  # K and V rows of one position, all kv heads, f16
KV_LO, KV_HI = 64, 1024
WORKLOAD = ("config[2]: full talker decode step, 28 layers, hidden 2048, 16q/8kv heads x 128, "
            "SwiGLU 6144, f16 weights N(0,0.02), 16 codebook heads x 2048, greedy; 48 lanes, "
            "KV lengths U[64,1024] seed 0, paged (32-position pages)")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def clocks_path(args, rank):
    """Where the nvidia-smi samples of this rank go: --clocks-dir (default /tmp)."""
    d = getattr(args, "clocks_dir", None) or "/tmp"
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, f"clocks_rank{rank}.csv")


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def kv_lengths(seed=0):
    return np.random.default_rng(seed).integers(KV_LO, KV_HI + 1, LANES).astype(np.int32)


# ---------------------------------------------------------------- reference (CPU) arm
_F16_BASE: dict = {}


def normal_f16_bits(rng, shape, std=1.0):
    """~N(0, std^2) as f16 bit patterns for the CPU arm's multi-GB weights and caches: a seeded
    block of 2^24 normal values is drawn once per std, and each array is that block repeated
    from a random offset (memcpy speed; the values are only read for timing)."""
    import oracle as orc
    base = _F16_BASE.get(std)
    if base is None:
        base = orc.f16_bits(np.random.default_rng(12345).standard_normal(1 << 24, dtype=np.float32)
                            * np.float32(std))
        _F16_BASE[std] = base
    n = int(np.prod(shape))
    off = int(rng.integers(0, base.size))
    reps = -(-(n + off) // base.size)
    return np.tile(base, reps)[off:off + n].reshape(shape)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuSample:
    """The oracle's decode step at config[2]: all 28 layers at 48 lanes with the workload's KV
    lengths, then the 16 heads and the greedy pick. The oracle's projection runs 4 x 4 blocks of
    outputs on AVX2/FMA with F16C conversions and its attention scores 8 positions per SIMD
    vector, over all host cores (OpenMP). `time()` returns seconds per step."""

    def __init__(self, threads=None, seed=0):
        import oracle as orc
        self.orc = orc
        if threads:
            orc.set_threads(threads)
        rng = np.random.default_rng(seed)
        self.g = orc.Geometry()
        self.lengths = kv_lengths(seed)
        cap = int(self.lengths.max()) + 2
        g = self.g
        nq = (HEADS + 2 * N_KV) * HD

        def layer():
            qk = np.stack([rng.uniform(0.8, 1.2, HD).astype(np.float32) / np.sqrt(HD),
                           rng.uniform(0.8, 1.2, HD).astype(np.float32)]).astype(np.float32)
            return orc.Layer(attn_norm=rng.uniform(0.8, 1.2, DIM).astype(np.float32),
                             ffn_norm=rng.uniform(0.8, 1.2, DIM).astype(np.float32),
                             wqkv=normal_f16_bits(rng, (nq, DIM), 0.02), qk_norms=qk,
                             wo=normal_f16_bits(rng, (DIM, HEADS * HD), 0.02),
                             gate=normal_f16_bits(rng, (FFN, DIM), 0.02),
                             up=normal_f16_bits(rng, (FFN, DIM), 0.02),
                             down=normal_f16_bits(rng, (DIM, FFN), 0.02))

        self.layers = [layer() for _ in range(g.layers)]
        self.final = np.ones(DIM, np.float32)
        shape = (LANES, N_KV, cap, HD)
        self.kc = [normal_f16_bits(rng, shape) for _ in range(g.layers)]
        self.vc = [normal_f16_bits(rng, shape) for _ in range(g.layers)]
        self.heads = normal_f16_bits(rng, (CB * VOCAB, DIM), 0.02)
        self.x = rng.standard_normal((LANES, DIM), dtype=np.float32)
        self.cos, self.sin = orc.rope_table(cap + 64, HD, 1e6)
        self.sample = (f"28 of 28 layers + 16 heads at 48 lanes, KV lengths U[64,1024] seed 0 "
                       f"(contiguous per-lane caches); one full step per sample on "
                       f"{orc.threads()} threads of {cpu_model()}")

    def threads(self):
        return self.orc.threads()

    def time(self):
        orc = self.orc
        t0 = time.perf_counter()
        h = orc.decode_step(self.x, self.layers, self.final, self.kc, self.vc, self.lengths,
                            self.cos, self.sin, self.g)
        orc.heads_pick(h, self.heads, self.g)
        return time.perf_counter() - t0


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    cs = CpuSample(threads=cores)
    for _ in range(min(args.warmup, 1)):
        cs.time()
    per_steps = [cs.time() for _ in range(args.steps)]
    sec = statistics.median(per_steps)
    sample, used = cs.sample, cs.threads()
    value = LANES / sec
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": "host cores"},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": used, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- B200 arm
class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index, path, interval_ms=200):
        self.path = path
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms",
                                          str(int(interval_ms))],
                                         stdout=open(path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        pw = []
        for r in rows:
            try:
                pw.append(float(r[3]))
            except ValueError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(pw) if pw else None}


def build_device_talker(device, seed=0, extra_positions=256, lanes_override=None, codebooks=CB,
                        vocab=VOCAB):
    import torch
    import ttsnn
    from qwen3tts import Geometry, LayerTensors, PagedKv, Stack
    gen = torch.Generator(device=device).manual_seed(seed)

    def w(n, k):
        return (torch.randn(n, k, generator=gen, device=device) * 0.02).half()

    geo = Geometry(dim=DIM, layers=LAYERS, heads=HEADS, n_kv=N_KV, head_dim=HD, ffn=FFN,
                   rope_len=max(KV_HI + extra_positions + 64, 1600), codebooks=codebooks,
                   vocab=vocab)
    ones = torch.ones(DIM, device=device)
    qk = torch.stack([torch.full((HD,), 1.0 / HD ** 0.5, device=device), torch.ones(HD, device=device)])
    layers = []
    for _ in range(LAYERS):
        layers.append(LayerTensors.from_plain(ones, ones, w((HEADS + 2 * N_KV) * HD, DIM), qk,
                                              w(DIM, HEADS * HD),
                                              ttsnn.interleave_gate_up(w(FFN, DIM), w(FFN, DIM)),
                                              w(DIM, FFN)))
    heads = w(codebooks * vocab, DIM)
    embed = (torch.randn(codebooks, vocab, DIM, generator=gen, device=device) * 0.02).half()
    stack = Stack(geo, layers, ones, heads, embed)
    if lanes_override == 0:
        return stack, None, None, None
    lengths = kv_lengths(seed)
    cap = KV_HI + extra_positions
    per_lane = -(-cap // BLOCK)
    kv = PagedKv(geo, LANES, LANES * per_lane, BLOCK, per_lane, device)
    for i in range(LANES):
        kv.admit(i, cap, int(lengths[i]))
    for li in range(LAYERS):
        kv.k[li].normal_(generator=gen)
        kv.v[li].normal_(generator=gen)
    return stack, kv, lengths, cap


def time_dominant_gemm(stack, device, reps=3):
    """The gate/up GEMM (SwiGLU epilogue) alone, over the 28 layers' weights in turn (1.4 GB, so
    nothing is served from L2): CUDA-event time per launch on the launching stream."""
    import torch
    import ttsnn
    from ttsnn import _lib as L
    x = torch.randn(LANES, DIM, device=device)
    projs = [ttsnn.Proj(lt.w_gate_up, packed=False) for lt in stack.layers]
    for p in projs:  # the stack's weights are already packed
        p.packed = True
    out = torch.empty(LANES, FFN, device=device, dtype=torch.float16)
    for p in projs:
        p.forward(x, L.EPI_SWIGLU_F16, out=out)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x16 = x.half()
    e0.record(s)
    for _ in range(reps):
        for p in projs:
            L.call("tts_proj_forward_packed", ttsnn.ctx(), ttsnn.ptr(x16), LANES, DIM,
                   ttsnn.ptr(p.w), 2 * FFN, L.EPI_SWIGLU_F16, ttsnn.ptr(out), 0, ttsnn.stream())
    e1.record(s)
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / (reps * len(projs)) * 1e-3
    bytes_ = 2 * FFN * DIM * 2 + LANES * DIM * 2 + LANES * FFN * 2
    return per, bytes_


def time_dominant_attention(stack, kv, device, reps=3):
    """The decode attention alone, as the step launches it (48 lanes, gqa 2, spans = each lane's
    position + 1, f16 output), over the 28 layers' pages in turn (3 GB of K/V, so nothing is
    served from L2): CUDA-event time per launch on the launching stream, and the algorithmic
    bytes of one launch (every K and V row of every lane's span read once, q read, output
    written)."""
    import ctypes as C
    import torch
    import ttsnn
    from ttsnn import _lib as L
    q = torch.randn(LANES, HEADS, HD, device=device) * 0.1
    spans = (kv.positions + 1).to(torch.int32)
    caches = [L.KvCache(kv.k[li].data_ptr(), kv.v[li].data_ptr(), kv.table.data_ptr(),
                        kv.max_blocks, kv.block_size, kv.num_blocks, N_KV, HD)
              for li in range(LAYERS)]
    max_span = kv.max_blocks * kv.block_size
    out = torch.empty(LANES, HEADS * HD, device=device, dtype=torch.float16)
    ctx = ttsnn.ctx()

    def one(c):
        L.call("tts_decode_attention", ctx, ttsnn.ptr(q), LANES, HEADS // N_KV, C.byref(c),
               ttsnn.ptr(spans), max_span, 0, ttsnn.ptr(out), 1, ttsnn.stream())

    for c in caches:
        one(c)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        for c in caches:
            one(c)
    e1.record(s)
    torch.cuda.synchronize()
    ttsnn.check()
    per = e0.elapsed_time(e1) / (reps * LAYERS) * 1e-3
    total = int(spans.sum().item())
    bytes_ = total * ATTN_BYTES_PER_POS + LANES * HEADS * HD * 4 + LANES * HEADS * HD * 2
    return per, bytes_, total


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def build_codec_block(device, b=8, t=24000, c=512, seed=0):
    """Benchmark config[1]: x [8, 512, 24000] f16 ~N(0,1) held channels-last [8, 24000, 512];
    per dilation 1, 3, 9: x = x + conv_k7(snake(x)) with 'same' padding, alpha = exp(U(-1,1)),
    Snake's 1/alpha, weights ~N(0, 0.02), bias 0."""
    import torch
    import ttsnn
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(b, t, c, generator=gen, device=device).half()
    convs = []
    for d in (1, 3, 9):
        w_tap = torch.randn(7, c, c, generator=gen, device=device) * 0.02
        alpha = torch.exp(torch.rand(c, generator=gen, device=device) * 2 - 1)
        convs.append((ttsnn.nlc.device_weight(w_tap), torch.zeros(c, device=device), alpha,
                      1.0 / alpha, d))
    return x, convs


def codec_block(x, convs, bufs):
    import ttsnn
    cur = x
    for i, (w, bias, alpha, brecip, d) in enumerate(convs):
        out = bufs[i % 2]
        ttsnn.nlc.conv1d(cur, w, bias, d, 3 * d, snake=(alpha, brecip), res=cur, out=out)
        cur = out
    return cur


def time_codec_block(device, reps=5):
    import torch
    x, convs = build_codec_block(device)
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    codec_block(x, convs, bufs)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        codec_block(x, convs, bufs)
    e1.record(s)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) * 1e-3 / reps
    b, t, c = x.shape
    flops = 3 * 2 * b * t * c * c * 7
    return sec, flops


def run_sweep(args):
    """Benchmark config[3]: a document of segments with target lengths log-uniform in [40, 1200]
    frames, grouped longest-first into runs of `--lanes` lanes, groups split over the ranks by
    LPT (no collective on the data path), each rank decoding its shard with tail shedding;
    with `--refill` (finished lanes reused) single segments are split by LPT on their frames and
    each rank groups its own. frames/s = all frames / max over ranks of device time."""
    import torch
    import torch.distributed as dist
    from qwen3tts.talker import (Talker, plan_groups, shard_groups, shard_segments,
                                 synthetic_segments)
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    n_segments = args.segments * world
    segs = synthetic_segments(n_segments, seed=0)
    if args.refill:
        mine = plan_groups(shard_segments(segs, world)[rank], args.lanes)
    else:
        mine = shard_groups(plan_groups(segs, args.lanes), world)[rank]
    queue = [s for g in mine for s in g]
    stack, _, _, _ = build_device_talker(device, seed=0, extra_positions=0, lanes_override=0)
    cap = 157 + 1200 + 2
    talker = Talker(stack, max_lanes=args.lanes, capacity=cap)
    # warm-up: capture the graphs of every width this shard will use on a short copy
    talker.run([type(s)(s.index, s.prompt_len, min(s.frames, 2), 0) for s in queue[: args.lanes]])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st = talker.run(queue, refill=args.refill)
    t = torch.tensor([st.seconds, st.frames, st.lane_steps], device=device, dtype=torch.float64)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
        t[0] = tmax[0]
    secs, frames, lane_steps = float(t[0]), int(t[1]), int(t[2])
    if rank == 0:
        line = {"metric": "codec frames/sec (lane sweep, whole box)", "value": round(frames / secs, 2),
                "unit": "frames/s", "n_gpus": world, "higher_is_better": True, "scaling": "weak",
                "dtype": "f16", "data": "synthetic",
                "config": {"workload": "config[3]: talker lane sweep, segments log-U[40,1200] frames, "
                                       "prompt 157, longest-first groups, tail shedding"
                                       + (" + interior refill" if args.refill else ""),
                           "lanes": args.lanes, "segments": n_segments, "refill": bool(args.refill)},
                "frames": frames, "seconds": round(secs, 4), "useful_lane_step_fraction":
                    round(frames / max(1, lane_steps), 4), "rtf": round(secs / (frames / 12.5), 5)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def document_sample(args, rank, world, device):
    """Benchmark config[4] (bounded sample) on this rank: a synthetic document of `--segments`
    segments per GPU (2000 in the config) with target lengths log-uniform in [40, 1200] frames,
    decoded by the talker at `--lanes` lanes with tail shedding and interior refill, then turned
    into 24 kHz audio by the codec decoder stack (x2 x2 pre-upsample, x8 x5 x4 x3 transposed
    convs 1024 -> 64, three snake residual blocks after each, random-init) over each segment's
    chunk windows (300 frames + 25 left context + 8 frames of lookahead for the 'same'-padded
    blocks), all windows of a rank decoded in batches, and the rank's audio copied into pinned
    host memory (the host gather). The codec's RVQ dequantiser and pre-transformer are not on
    this path: seeded random latents stand in for its input. Segments are split over the ranks
    one by one by LPT on their frames (shard_segments: a refilling talker's time follows its
    frames), each rank grouping its own longest-first; no collective on the data path. Returns the
    rank-0 summary (None on other ranks): frames/s = all frames / max over ranks of (talker +
    codec + host copy device time); rtf = that time / audio seconds (12.5 frames per second)."""
    import torch
    import torch.distributed as dist
    from qwen3tts.codec import WaveStack, chunk_plan
    from qwen3tts.talker import Talker, plan_groups, shard_segments, synthetic_segments
    n_segments = args.segments * world
    segs = synthetic_segments(n_segments, seed=0)
    shards = shard_segments(segs, world)
    mine = plan_groups(shards[rank], args.lanes)
    loads = [sum(s.frames for s in sh) for sh in shards]
    queue = [s for g in mine for s in g]
    stack, _, _, _ = build_device_talker(device, seed=0, extra_positions=0, lanes_override=0)
    talker = Talker(stack, max_lanes=args.lanes, capacity=157 + 1200 + 2)
    talker.run([type(s)(s.index, s.prompt_len, min(s.frames, 2), 0) for s in queue[: args.lanes]])

    # codec windows of every segment of this shard, one uniform span
    right = 8
    span = 300 + 25 + right
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    wins = []
    for sg in queue:
        lat = torch.randn(sg.frames, 1024, generator=gen, device=device).half()
        for w in chunk_plan(sg.frames, right=right):
            idx = torch.arange(w.lo, w.lo + span, device=device).clamp(max=w.hi - 1)
            wins.append(lat.index_select(0, idx))
    codec = WaveStack(device, seed=7)
    batch = 16
    xs = [torch.stack(wins[i:i + batch]) for i in range(0, len(wins), batch)]
    outs = [None] * len(xs)
    # warm-up on the timed batches' shapes (a full batch and the last, shorter one), so that
    # one-time per-shape set-up (occupancy queries, kernel attributes) stays out of the timing
    codec(xs[0])
    codec(xs[-1])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st = talker.run(queue, refill=True)
    e0, e1, e2 = torch.cuda.Event(True), torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    samples = 0
    for i, xb in enumerate(xs):
        outs[i] = codec(xb)
        samples += outs[i].numel()
    e1.record()
    # host gather: every window's audio into one pinned host buffer
    host = torch.empty(samples, dtype=torch.float16, pin_memory=True)
    o = 0
    for y in outs:
        n = y.numel()
        host[o:o + n].copy_(y.reshape(-1), non_blocking=True)
        o += n
    e2.record()
    torch.cuda.synchronize()
    codec_s = e0.elapsed_time(e1) * 1e-3
    gather_s = e1.elapsed_time(e2) * 1e-3
    flops = codec.flops_per_frame() * len(wins) * span
    mine_s = st.seconds + codec_s + gather_s
    t = torch.tensor([mine_s, st.seconds, codec_s, gather_s, st.frames, flops, samples],
                     device=device, dtype=torch.float64)
    per_rank = [mine_s]
    if world > 1:
        g = [torch.zeros(1, device=device, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(g, t[:1].clone())
        per_rank = [float(x.item()) for x in g]
        tmax = t[:4].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t[4:].clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        t = torch.cat([tmax, tsum])
    secs, tk_s, cd_s, ga_s, frames, flops, samples = [float(v) for v in t]
    if rank != 0:
        return None
    mean_load = sum(loads) / len(loads)
    return {"metric": "codec frames/sec (end-to-end document, whole box)",
            "value": round(frames / secs, 2), "unit": "frames/s", "n_gpus": world,
            "higher_is_better": True, "scaling": "weak", "dtype": "f16",
            "data": "synthetic (random-init weights; random latents in place of the RVQ front)",
            "config": {"workload": "config[4] sample: talker (lane scheduler, shedding, refill) "
                                   "+ codec stack at 24 kHz over chunk windows + host gather",
                       "segments": n_segments, "segments_per_gpu": args.segments,
                       "lanes": args.lanes, "window_frames": span, "codec_batch_windows": batch},
            "frames": int(frames), "audio_seconds": round(frames / 12.5, 2),
            "seconds": round(secs, 4), "talker_seconds": round(tk_s, 4),
            "codec_seconds": round(cd_s, 4), "host_gather_seconds": round(ga_s, 5),
            "rtf": round(secs / (frames / 12.5), 6),
            "codec_tflops": round(flops / max(cd_s, 1e-9) / 1e12, 1),
            "lpt_planned_imbalance": round(max(loads) / mean_load, 4) if mean_load else 1.0,
            "measured_imbalance": round(max(per_rank) / (sum(per_rank) / len(per_rank)), 4),
            "seconds_per_rank": [round(x, 4) for x in per_rank],
            "samples": int(samples)}


def run_document(args):
    """`--workload document`: config[4]'s sample as its own JSON line (document_sample)."""
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    line = document_sample(args, rank, world, device)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def build_device_predictor(device, seed=0):
    """The depth predictor at the reference's shape (crates/qwen3tts/src/cfg.rs): a 5-layer
    stack at dim 1024 (16/8 heads x 128, SwiGLU 3072), 15 heads [2048, 1024], the 2048 -> 1024
    projection with bias, 15 tables [2048, 2048]; f16 weights ~N(0, 0.02), random init."""
    import torch
    import ttsnn
    from qwen3tts import PREDICTOR_GEOMETRY as g, LayerTensors, Predictor, Stack
    gen = torch.Generator(device=device).manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=gen, device=device) * 0.02).half()

    def norm(n):
        return torch.rand(n, generator=gen, device=device) * 0.4 + 0.8

    nqkv = (g.heads + 2 * g.n_kv) * g.head_dim
    layers = [LayerTensors.from_plain(norm(g.dim), norm(g.dim), w(nqkv, g.dim),
                                      torch.stack([norm(128) / 128 ** 0.5, norm(128)]),
                                      w(g.dim, g.heads * g.head_dim),
                                      ttsnn.interleave_gate_up(w(g.ffn, g.dim), w(g.ffn, g.dim)),
                                      w(g.dim, g.ffn)) for _ in range(g.layers)]
    stack = Stack(g, layers, norm(g.dim))
    return Predictor(stack, w(g.dim, 2048), (torch.randn(g.dim, generator=gen, device=device) * 0.02),
                     w(15 * g.vocab, g.dim), w(15, g.vocab, 2048))


class PredictorCpuSample:
    """The oracle's predictor frame (all 15 depth steps) for `lanes` lanes at the reference's
    shape; seconds per frame of those lanes."""

    def __init__(self, lanes=2, threads=None, seed=0):
        import oracle as orc
        self.orc = orc
        if threads:
            orc.set_threads(threads)
        rng = np.random.default_rng(seed)
        self.g = orc.Geometry(dim=1024, layers=5, heads=16, n_kv=8, ffn=3072, codebooks=1,
                              vocab=2048)
        self.layers = [orc.synthetic_layer(rng, self.g) for _ in range(5)]
        self.final = np.ones(1024, np.float32)
        w = lambda *sh: orc.f16_bits(rng.standard_normal(sh, dtype=np.float32) * 0.02)
        resize, heads, tables = w(1024, 2048), w(15 * 2048, 1024), w(15, 2048, 2048)
        bias = np.zeros(1024, np.float32)
        resized = (orc.f16_value(tables) @ orc.f16_value(resize).T).astype(np.float32)
        self.pw = orc.PredictorWeights(resize, bias, heads, tables, resized)
        self.lanes = lanes
        self.hidden = rng.standard_normal((lanes, 2048), dtype=np.float32)
        self.code0 = orc.f16_value(w(lanes, 2048))
        self.sample = (f"one predictor frame (prefill + 15 depth steps + embedding sum) for "
                       f"{lanes} lanes at the reference's shape")

    def threads(self):
        return self.orc.threads()

    def time(self):
        t0 = time.perf_counter()
        self.orc.predictor_frame(self.hidden, self.code0, self.layers, self.final, self.pw, self.g)
        return time.perf_counter() - t0


def run_predictor(args):
    """The depth predictor (crates/qwen3tts/src/talker.rs:255-550) at `--lanes` lanes per GPU.
    One step = one frame for every lane: the two-position prefill, 15 greedy depth steps, the
    embedding sum at talker width, as one captured graph; frames/s = lanes x frames per second.
    Roofline: HBM, the frame's weight stream (the 5-layer stack once per depth step, one head per
    step, the doubled projection) over the frame time. Weak scaling: each rank its own lanes."""
    import torch
    import torch.distributed as dist
    import ttsnn
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    lanes, steps, warmup = args.lanes, args.steps, args.warmup
    p = build_device_predictor(device, seed=rank)
    kv = p.new_state(lanes)
    h_host = torch.randn(lanes, 2048).pin_memory()
    c_host = (torch.randn(lanes, 2048) * 0.02).half().float().pin_memory()
    codes_host = torch.empty(lanes, 15, dtype=torch.int32).pin_memory()
    sum_host = torch.empty(lanes, 2048).pin_memory()
    h = h_host.to(device)
    c0 = c_host.to(device)
    codes = torch.empty(lanes, 15, dtype=torch.int32, device=device)
    total = torch.empty(lanes, 2048, device=device)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        graph = p.capture(kv, h, c0, codes, total)
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    ttsnn.check(local)

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local, clocks_path(args, rank))
    ttsnn.launch_count(reset=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    launches = ttsnn.launch_count()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ttsnn.check(local)
    # end to end through the public API: the talker's hidden and code-0 embedding in from
    # pinned host memory, the codes and the next-input sum back, every frame
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record(stream)
        for _ in range(steps):
            h.copy_(h_host, non_blocking=True)
            c0.copy_(c_host, non_blocking=True)
            graph.replay()
            codes_host.copy_(codes, non_blocking=True)
            sum_host.copy_(total, non_blocking=True)
            stream.synchronize()
        e3.record(stream)
    stream.synchronize()
    t2 = torch.tensor([e2.elapsed_time(e3)], device=device)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())
    ttsnn.check(local)
    hbm, peak_kind = peaks()
    frame_s = ms / steps * 1e-3
    wbytes = p.weight_bytes()
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cs = PredictorCpuSample(threads=os.cpu_count())
            cs.time()
            cpu_t = statistics.median([cs.time() for _ in range(3)])
            cpu = {"value": round(cs.lanes / cpu_t, 3), "unit": UNIT, "cores": cs.threads(),
                   "kind": "port", "sample": cs.sample}
        line = {
            "metric": "codec frames/sec (depth predictor, whole box)",
            "value": round(world * lanes * steps / (ms * 1e-3), 2), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights)",
            "config": {"workload": "depth predictor frame (talker.rs:407-550): 5 layers dim 1024, "
                                   "16q/8kv heads x 128, SwiGLU 3072, 15 heads x 2048 greedy, "
                                   "resize 2048->1024 + bias, tables 15 x [2048, 2048]",
                       "lanes_per_gpu": lanes, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2: each frame streams 2.4 GB of weights"},
            "roofline": {"bound": "hbm", "kernel": "whole frame (weight stream)",
                         "achieved": round(wbytes / frame_s / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(wbytes / frame_s / 1e9 / hbm, 4),
                         "traffic": None, "peak_source": peak_kind,
                         "algorithmic_bytes_per_frame": int(wbytes)},
            "e2e": {"value": round(world * lanes * steps / (e2e_ms * 1e-3), 2), "unit": UNIT,
                    "h2d_bytes_per_step": lanes * 2048 * 4 * 2,
                    "d2h_bytes_per_step": lanes * (15 * 4 + 2048 * 4)},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_frames(args):
    """The reference's talker loop, greedy (talker.rs:903-1073), at 48 lanes per GPU: one step =
    one frame for every lane = the 28-layer talker step with its codec head (3072 ids) under the
    pick rule (banned top 1024 except eos, eos after 2 frames, repetition penalty 1.05), code 0's
    codec_embed row, the depth predictor's 15 residual codes and the next input (their sum plus
    the lane's text row), as one captured graph. KV lengths U[64, 1024] as config[2]. frames/s =
    lanes x frames per second; e2e adds each frame's text rows in (pinned host -> device) and
    its 16 codes out. Weak scaling: each rank its own lanes."""
    import torch
    import torch.distributed as dist
    import ttsnn
    from qwen3tts import FrameLoop, reference_pick
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    steps, warmup = args.steps, args.warmup
    extra = steps + warmup + 8
    stack, _, _, _ = build_device_talker(device, seed=rank, extra_positions=extra,
                                         lanes_override=0, codebooks=1, vocab=3072)
    pred = build_device_predictor(device, seed=100 + rank)
    lengths = kv_lengths(rank)
    cap = KV_HI + extra + 8
    text_len = 64
    gen = torch.Generator(device=device).manual_seed(200 + rank)
    text = torch.randn(LANES, text_len, DIM, generator=gen, device=device) * 0.1
    pad = torch.randn(DIM, generator=gen, device=device) * 0.1
    loop = FrameLoop(stack, pred, LANES, cap, reference_pick(lanes=LANES, device=device), text,
                     pad, block_size=BLOCK)
    for i in range(LANES):
        loop.admit(i, int(lengths[i]) + 1, extra, torch.randn(DIM, generator=gen, device=device))
    for li in range(LAYERS):
        loop.kv.k[li].normal_(generator=gen)
        loop.kv.v[li].normal_(generator=gen)
    stream = torch.cuda.Stream(device)
    text_host = (torch.randn(LANES, DIM) * 0.1).pin_memory()
    codes_host = torch.empty(LANES, 16, dtype=torch.int32).pin_memory()
    with torch.cuda.stream(stream):
        graph = loop.graph(LANES)
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    ttsnn.check(local)

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local, clocks_path(args, rank))
    ttsnn.launch_count(reset=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    launches = ttsnn.launch_count()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ttsnn.check(local)
    # end to end: each frame's text rows in from pinned host memory, its 16 codes out
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record(stream)
        for i in range(steps):
            f = (warmup + steps + i) % text_len
            loop.text.rows[:, f].copy_(text_host, non_blocking=True)
            graph.replay()
            codes_host[:, 0].copy_(loop.code0[:LANES], non_blocking=True)
            codes_host[:, 1:].copy_(loop.codes[:LANES], non_blocking=True)
            stream.synchronize()
        e3.record(stream)
    stream.synchronize()
    t2 = torch.tensor([e2.elapsed_time(e3)], device=device)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())
    ttsnn.check(local)
    hbm, peak_kind = peaks()
    frame_s = ms / steps * 1e-3
    mean_len = float(lengths.mean()) + warmup + steps / 2.0 + 1
    kv_bytes = LAYERS * N_KV * HD * 2 * 2 * LANES * mean_len
    fbytes = stack.weight_bytes() + kv_bytes + pred.weight_bytes()
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            ts = CpuSample(threads=os.cpu_count())
            ps = PredictorCpuSample(threads=os.cpu_count())
            ts.time()
            ps.time()
            t_talker = statistics.median([ts.time() for _ in range(3)])
            t_pred = statistics.median([ps.time() for _ in range(3)]) * LANES / ps.lanes
            cpu = {"value": round(LANES / (t_talker + t_pred), 3), "unit": UNIT,
                   "cores": ts.threads(), "kind": "port",
                   "sample": ts.sample + "; plus " + ps.sample + ", scaled to 48 lanes"}
        line = {
            "metric": "codec frames/sec (reference talker loop: talker + depth predictor, whole box)",
            "value": round(world * LANES * steps / (ms * 1e-3), 2), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights)",
            "config": {"workload": "talker.rs:903-1073 greedy: 28-layer talker (config[2] shape) "
                                   "with codec head 3072 + pick rule, depth predictor (5 x 1024, "
                                   "15 heads), text rows; 48 lanes, KV lengths U[64,1024]",
                       "lanes_per_gpu": LANES, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2: each frame streams 5.3 GB of weights "
                             "and ~3 GB of KV"},
            "roofline": {"bound": "hbm", "kernel": "whole frame (weights + KV)",
                         "achieved": round(fbytes / frame_s / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(fbytes / frame_s / 1e9 / hbm, 4),
                         "traffic": None, "peak_source": peak_kind,
                         "algorithmic_bytes_per_frame": int(fbytes)},
            "e2e": {"value": round(world * LANES * steps / (e2e_ms * 1e-3), 2), "unit": UNIT,
                    "h2d_bytes_per_step": LANES * DIM * 4, "d2h_bytes_per_step": LANES * 16 * 4},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph
    loop.graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_prefill(args):
    """Prompt prefill (Stack::forward at t > 1, qwen3.rs:294-467) at config[2]'s talker shape:
    48 lanes x 157 prompt positions (the reference's ICL width) through the 28 layers, layer by
    layer over all rows: prefill-shaped projections over the 7,536 rows, each row's attention
    over its lane's pages. value = prompt tokens per second over the whole call (its row plan
    upload included). Roofline: tensor (2 x tokens x 1.41 G weights FLOP, the attention's share
    is < 1 %)."""
    import torch
    import ttsnn
    from qwen3tts import PagedKv
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    prompt = 157
    stack, _, _, _ = build_device_talker(device, seed=rank, extra_positions=0, lanes_override=0)
    cap = prompt + 3
    per = -(-cap // BLOCK)
    kv = PagedKv(stack.geo, LANES, LANES * per, BLOCK, per, device)
    gen = torch.Generator(device=device).manual_seed(rank)
    x = torch.randn(LANES * prompt, DIM, generator=gen, device=device)
    lens = [prompt] * LANES

    def run():
        for i in range(LANES):
            kv.positions[i] = 0
        stack.prefill(kv, lens, x, max_span=cap)

    for i in range(LANES):
        kv.admit(i, cap, 0)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    ttsnn.check(local)
    ttsnn.launch_count(reset=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    launches = ttsnn.launch_count()
    ttsnn.check(local)
    s_per = e0.elapsed_time(e1) * 1e-3 / args.steps
    tokens = LANES * prompt
    flops = 2.0 * tokens * (stack.weight_bytes() - 16 * VOCAB * DIM * 2) / 2
    tpeak, tkind = bf16_peak()
    if rank == 0:
        print(json.dumps({
            "metric": "prompt tokens/sec (prefill, one GPU)", "value": round(tokens / s_per, 1),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(s_per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights)",
            "config": {"workload": "prefill of 48 lanes x 157 positions through the config[2] "
                                   "talker (28 layers), layer-major over all rows",
                       "tokens": tokens},
            "roofline": {"bound": "tensor", "achieved": round(flops / s_per / 1e12, 1),
                         "peak": tpeak, "unit": "TFLOP/s",
                         "frac": round(flops / s_per / 1e12 / tpeak, 4), "traffic": None,
                         "peak_source": tkind + " dense bf16"},
            "gpu_launches": int(launches)}), flush=True)
    return 0


def run_codec(args):
    """The codec decoder at the reference's shape (codec.rs:320-424, random-init): codes
    [T, 16] -> 24 kHz audio through the front (RVQ, pre-conv, 8-layer pre-transformer, x2 x2
    with ConvNeXt) and the waveform stack (1536 -> 96 channels, x8 x5 x4 x3). One step = one
    333-frame chunk window (300 frames + 25 of left context + 8 of lookahead, the chunk plan's
    span); frames/s counts the 300 frames each window contributes."""
    import torch
    import ttsnn
    from qwen3tts.codec_ref import Codec
    device = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    codec = Codec.from_weights(Codec.synthetic_weights(seed=0).__getitem__)
    T = 333
    codes = torch.randint(0, 2048, (T, 16), dtype=torch.int32, device=device)
    for _ in range(args.warmup):
        codec(codes)
    torch.cuda.synchronize()
    ttsnn.check(0)
    ttsnn.launch_count(reset=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        codec(codes)
    e1.record()
    torch.cuda.synchronize()
    launches = ttsnn.launch_count()
    s_per = e0.elapsed_time(e1) * 1e-3 / args.steps
    print(json.dumps({
        "metric": "codec frames/sec (reference-shape decoder, one GPU)",
        "value": round(300 / s_per, 1), "unit": "frames/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(s_per * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (random-init weights, random codes)",
        "config": {"workload": "codec.rs decoder: 16 codebooks x 2048, pre-transformer 8 x 512 "
                               "(16 x 64 heads, window 72), x2 x2 ConvNeXt at 1024, waveform "
                               "stack 1536 -> 96 at x8 x5 x4 x3; one 333-frame window",
                   "window_frames": T},
        "rtf": round(s_per / (300 / 12.5), 6), "gpu_launches": int(launches)}), flush=True)
    return 0


def run_kernel_case(args):
    """Small standalone cases of one kernel, for ncu captures (a few launches, < 1 GB)."""
    import torch
    import ttsnn
    from ttsnn import _lib as L
    device = torch.device("cuda", 0)
    if args.kernel == "gemm":
        gen = torch.Generator(device=device).manual_seed(0)
        ws = [ttsnn.interleave_gate_up((torch.randn(FFN, DIM, generator=gen, device=device) * 0.02).half(),
                                       (torch.randn(FFN, DIM, generator=gen, device=device) * 0.02).half())
              for _ in range(4)]
        x = torch.randn(LANES, DIM, device=device)
        out = torch.empty(LANES, FFN, device=device, dtype=torch.float16)
        for i in range(8):
            ttsnn.Proj(ws[i % 4]).forward(x, L.EPI_SWIGLU_F16, out=out)
    elif args.kernel == "attn":
        from qwen3tts import Geometry, PagedKv
        geo = Geometry(layers=1)
        lengths = kv_lengths(0)
        per = -(-KV_HI // BLOCK) + 1
        kv = PagedKv(geo, LANES, LANES * per, BLOCK, per, device)
        for i in range(LANES):
            kv.admit(i, per * BLOCK, int(lengths[i]))
        kv.k.normal_()
        kv.v.normal_()
        q = torch.randn(LANES, HEADS, HD, device=device) * 0.1
        st = L.KvCache(kv.k.data_ptr(), kv.v.data_ptr(), kv.table.data_ptr(), per, BLOCK,
                       kv.num_blocks, N_KV, HD)
        for _ in range(4):
            ttsnn.attn.decode_attention_paged(q, st, kv.positions, per * BLOCK)
    elif args.kernel == "attn_short":
        # the depth predictor's attention: 48 lanes x 8 kv heads, spans 1..16, 16-position pages
        from qwen3tts import PREDICTOR_GEOMETRY, PagedKv
        kv = PagedKv(PREDICTOR_GEOMETRY, LANES, LANES, 16, 1, device)
        for i in range(LANES):
            kv.admit(i, 16, 1 + i % 16)
        kv.k.normal_()
        kv.v.normal_()
        q = torch.randn(LANES, HEADS, HD, device=device) * 0.1
        st = L.KvCache(kv.k.data_ptr(), kv.v.data_ptr(), kv.table.data_ptr(), 1, 16,
                       kv.num_blocks, N_KV, HD)
        for _ in range(4):
            ttsnn.attn.decode_attention_paged(q, st, kv.positions, 16)
    elif args.kernel == "conv":
        x, convs = build_codec_block(device)
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        codec_block(x, convs, bufs)
    torch.cuda.synchronize()
    ttsnn.check(0)
    print(json.dumps({"kernel_case": args.kernel, "ok": True}))
    return 0


def run_b200(args):
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    import ttsnn
    from ttsnn import _lib as L

    steps, warmup = args.steps, args.warmup
    stack, kv, lengths, cap = build_device_talker(
        device, seed=rank, extra_positions=2 * (steps + warmup) + args.sustained_steps + 16)
    stream = torch.cuda.Stream(device)
    codes = torch.zeros(LANES, CB, dtype=torch.int32, device=device)
    x_dev = torch.empty(LANES, DIM, device=device)
    x_host = torch.randn(LANES, DIM).pin_memory()
    codes_host = torch.empty(LANES, CB, dtype=torch.int32).pin_memory()
    max_span = cap
    with torch.cuda.stream(stream):
        x_dev.copy_(x_host, non_blocking=True)
        stack.decode_step(kv, x_dev, codes=codes, max_span=max_span)  # seeds the embedding input
        graph = stack.capture(kv, None, codes=codes, max_span=max_span)
        graph_e2e = stack.capture(kv, x_dev, codes=codes, max_span=max_span)
    stream.synchronize()
    ttsnn.check(local)
    pos0 = kv.positions.clone()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing (graph replays, inputs already in HBM)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local, clocks_path(args, rank))
    ttsnn.launch_count(reset=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    launches = ttsnn.launch_count()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=device)
    per_rank = [ms]
    if world > 1:
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        per_rank = [float(x.item()) for x in gathered]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ttsnn.check(local)

    # ---- sustained leg: the same replays for long enough (~0.6 s) that the clock sampler sees
    # the GPU under load; positions restart from the timed leg's start so the KV work matches
    sustained = None
    if args.sustained_steps > 0:
        with torch.cuda.stream(stream):
            kv.positions.copy_(pos0)
            for _ in range(warmup):
                graph.replay()
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks_s = Clocks(local, clocks_path(args, rank) + ".sustained", interval_ms=50)
        es0, es1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            es0.record(stream)
            for _ in range(args.sustained_steps):
                graph.replay()
            es1.record(stream)
        stream.synchronize()
        clk_s = clocks_s.stop()
        barrier()
        ts = torch.tensor([es0.elapsed_time(es1)], device=device)
        if world > 1:
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        sustained = {"steps": args.sustained_steps,
                     "ms_per_step": round(float(ts.item()) / args.sustained_steps, 4),
                     "value": round(world * LANES * args.sustained_steps / (float(ts.item()) * 1e-3), 2),
                     "clocks": clk_s}
        ttsnn.check(local)
    with torch.cuda.stream(stream):
        kv.positions.copy_(pos0)
    stream.synchronize()

    # ---- end to end through the public API: pinned host input in, codes out, every step
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            x_dev.copy_(x_host, non_blocking=True)
            graph_e2e.replay()
            codes_host.copy_(codes, non_blocking=True)
            stream.synchronize()
        e2.record(stream)
        for _ in range(steps):
            x_dev.copy_(x_host, non_blocking=True)
            graph_e2e.replay()
            codes_host.copy_(codes, non_blocking=True)
            stream.synchronize()  # the host reads the codes before the next step, as the engine does
        e3.record(stream)
    stream.synchronize()
    t2 = torch.tensor([e2.elapsed_time(e3)], device=device)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())
    ttsnn.check(local)

    # ---- roofline of the dominant kernel and of the whole step
    hbm, peak_kind = peaks()
    gemm_s, gemm_bytes = time_dominant_gemm(stack, device)
    with torch.cuda.stream(stream):
        kv.positions.copy_(pos0)
    stream.synchronize()
    attn_s, attn_bytes, attn_positions = time_dominant_attention(stack, kv, device)
    weights = stack.weight_bytes()
    mean_len = float(lengths.mean()) + warmup + steps / 2.0 + 1
    kv_bytes = LAYERS * N_KV * HD * 2 * 2 * LANES * mean_len
    step_bytes = weights + kv_bytes + CB * LANES * DIM * 2
    step_s = ms_max / steps * 1e-3

    codec_s, codec_flops = time_codec_block(device)
    tpeak, tpeak_kind = bf16_peak()
    # config[4]'s sharded segment queue with host gather, at this N (weak: segments per GPU)
    doc = None
    if args.document_segments > 0:
        import argparse as _ap
        dargs = _ap.Namespace(**vars(args))
        dargs.segments = args.document_segments
        dargs.lanes = LANES
        doc = document_sample(dargs, rank, world, device)

    if rank == 0:
        value = world * LANES * steps / (ms_max * 1e-3)
        e2e_value = world * LANES * steps / (e2e_ms * 1e-3)
        cpu = None
        if world == 1 and not args.no_cpu:
            cs = CpuSample(threads=os.cpu_count())
            cs.time()
            cpu_t = statistics.median([cs.time() for _ in range(3)])
            cpu = {"value": round(LANES / cpu_t, 3), "unit": UNIT, "cores": cs.threads(),
                   "kind": "port", "sample": cs.sample}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(ms_max / steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "lanes_per_gpu": LANES, "global_lanes": LANES * world,
                       "parallelism": f"dp{world} (replicated weights, lanes sharded per GPU)",
                       "l2": "inputs larger than L2: each step streams 2.95 GB of weights and ~3 GB of KV"},
            "roofline": {"bound": "hbm", "kernel": "attn_decode (the step's largest share of time: "
                                                   "48 lanes x 8 kv heads x gqa 2, paged f16 K/V)",
                         "achieved": round(attn_bytes / attn_s / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(attn_bytes / attn_s / 1e9 / hbm, 4),
                         "traffic": ATTN_NCU_TRAFFIC,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of "
                                           "one cold launch of this kernel on this workload "
                                           "(a separate capture, not measured in this run)",
                         "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": attn_bytes,
                         "algorithmic_unit": f"{ATTN_BYTES_PER_POS} B of K/V per cached position "
                                             f"per layer x {attn_positions} positions, + q and "
                                             "output",
                         "launch_us": round(attn_s * 1e6, 2)},
            "roofline_gemm": {"bound": "hbm", "kernel": "gemm_decode (gate/up, SwiGLU epilogue)",
                              "achieved": round(gemm_bytes / gemm_s / 1e9, 1), "peak": hbm,
                              "unit": "GB/s", "frac": round(gemm_bytes / gemm_s / 1e9 / hbm, 4),
                              "traffic": GATEUP_NCU_TRAFFIC,
                              "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                                "of one cold launch (a separate capture, not "
                                                "measured in this run)",
                              "algorithmic_bytes_per_launch": gemm_bytes,
                              "launch_us": round(gemm_s * 1e6, 2)},
            "roofline_step": {"bound": "hbm", "achieved": round(step_bytes / step_s / 1e9, 1),
                              "peak": hbm, "unit": "GB/s",
                              "frac": round(step_bytes / step_s / 1e9 / hbm, 4),
                              "algorithmic_bytes_per_step": int(step_bytes)},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                    "h2d_bytes_per_step": LANES * DIM * 4, "d2h_bytes_per_step": LANES * CB * 4},
            "codec_block": {"workload": "config[1]: [8,512,24000] f16, snake + 3 x conv 512->512 k7 "
                                        "d1/3/9 'same' + residual, implicit GEMM on tcgen05",
                            "ms": round(codec_s * 1e3, 3), "bound": "tensor",
                            "achieved": round(codec_flops / codec_s / 1e12, 1), "unit": "TFLOP/s",
                            "peak": tpeak, "frac": round(codec_flops / codec_s / 1e12 / tpeak, 4),
                            "peak_source": tpeak_kind + " dense bf16 (f16 runs at the same rate)",
                            "flops_per_block": codec_flops},
            "gpu_launches": int(launches),
            "clocks": clk,
            "ms_per_step_per_rank": [round(x / steps, 4) for x in per_rank],
        }
        if sustained is not None:
            line["sustained"] = sustained
        if doc is not None:
            line["document"] = doc
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph, graph_e2e
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_timeline(args):
    """Per-CTA phase timeline of one captured config[2] step, from the tracing library (build
    it with `python dream-tts_b200/build.py --timeline`; run with TTS_LIB=dream-tts_b200/ttsnn/
    libtts_cuda_tl.so). For each kernel of layers 5 and 20: first CTA entry, dependency release
    (first/last CTA), main loop done and cross-CTA reduction done (GEMMs), end (median/max over
    CTAs; for the attention the later of the compute end and the split-pair merges), in us from
    the layer's first record. Each CTA takes its end time before writing its records; the log's
    one atomic per CTA still delays its exit a little, so a traced step runs somewhat long."""
    import ctypes as C

    import torch

    import ttsnn
    from ttsnn import _lib as L
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cnt = C.c_int(0)
    if L.load().tts_timeline_read(None, 0, C.byref(cnt), 1) != 0:
        raise SystemExit("timeline: needs the tracing library (TTS_LIB=.../libtts_cuda_tl.so): "
                         + L.last_error())
    cap_rec = 1 << 21
    buf = (C.c_ulonglong * (cap_rec * 4))()
    GEMM, ATTN = 0x100, 0x200
    if args.workload == "prefill":
        return timeline_prefill(args, dev, L, C, cnt, buf, cap_rec)
    stack, kv, lengths, cap = build_device_talker(dev, seed=0, extra_positions=64)
    codes = torch.zeros(LANES, CB, dtype=torch.int32, device=dev)
    x = torch.randn(LANES, DIM, device=dev)
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        stack.decode_step(kv, x, codes=codes, max_span=cap)
        g = stack.capture(kv, x, codes=codes, max_span=cap)
        for _ in range(3):
            g.replay()
        s.synchronize()
        L.call("tts_timeline_read", None, 0, C.byref(cnt), 1)
        g.replay()
        s.synchronize()
    ttsnn.check(0)
    L.call("tts_timeline_read", buf, cap_rec, C.byref(cnt), 0)
    a = np.frombuffer(buf, dtype=np.uint64).reshape(cap_rec, 4)[:cnt.value].astype(np.int64)
    layers = stack.geo.layers

    def runs(first_kind):
        """[launch][cta][record] of the contiguous runs that start with `first_kind`, launches in
        time order, split evenly (a kernel's grid is the same in every layer)."""
        idx = np.nonzero(a[:, 0] == first_kind)[0]
        idx = idx[np.argsort(a[idx, 2])]
        return idx

    def gemm_phases(epi, n_launch, pick=None):
        idx = runs(GEMM | epi << 4)
        per = len(idx) // n_launch
        out = [idx[i * per:(i + 1) * per] for i in range(n_launch)]
        return out if pick is None else out[pick::2]

    qkv = gemm_phases(4, layers)
    gu = gemm_phases(3, layers)
    o = gemm_phases(2, 2 * layers, 0)
    dn = gemm_phases(2, 2 * layers, 1)
    att = runs(ATTN)
    per = len(att) // layers
    att = [att[i * per:(i + 1) * per] for i in range(layers)]
    mg = np.nonzero(a[:, 0] == ATTN | 4)[0]
    mg = mg[(mg + 1 < len(a)) & (a[np.minimum(mg + 1, len(a) - 1), 0] == ATTN | 5)]
    merged = {}
    for i in mg:  # (cta, time) of merge runs, assigned to a launch by time below
        merged.setdefault(int(a[i, 1]), []).append(int(a[i + 1, 1]))
    out = {"records": int(cnt.value), "layers": {}}
    for li in (5, 20):
        t0 = a[qkv[li], 1].min()
        f = lambda v: round(float((v - t0) / 1e3), 2)
        rows = {}
        for name, idx in (("qkv", qkv[li]), ("attn", att[li]), ("o", o[li]), ("gate/up", gu[li]),
                          ("down", dn[li])):
            row = {"entry": f(a[idx, 1].min()),
                   "released": [f(a[idx + 1, 1].min()), f(a[idx + 1, 1].max())]}
            if name == "attn":
                end = a[idx + 3, 1].copy()
                lo, hi = a[idx + 1, 1].min(), end.max() + 20_000
                for j, c in enumerate(a[idx + 2, 1]):
                    for t in merged.get(int(c), []):
                        if lo <= t <= hi:
                            end[j] = max(end[j], t)
                row["end"] = [f(np.median(end)), f(end.max())]
                row["cta_end_p10_p90"] = [f(np.percentile(end, 10)), f(np.percentile(end, 90))]
                if len(a) > int(idx.max()) + 6 and ((a[idx + 4, 0] & 0xf) == 6).all():
                    row["first_s"] = f(np.median(a[idx + 4, 1]))
                    row["first_p"] = f(np.median(a[idx + 5, 1]))
                    row["last_p"] = [f(np.median(a[idx + 6, 1])), f(a[idx + 6, 1].max())]
                    order = np.argsort(a[idx + 2, 1])  # by CTA index
                    row["per_cta"] = {k: [f(v) for v in a[idx + o, 1][order]]
                                      for k, o in (("released", 1), ("first_s", 4),
                                                   ("first_p", 5), ("last_p", 6))}
                    row["per_cta"]["end"] = [f(v) for v in end[order]]
                    if len(a) > int(idx.max()) + 8 and ((a[idx + 7, 0] & 0xf) == 9).all():
                        row["q_wait"] = f(np.median(a[idx + 7, 1]))
                        row["q_ready"] = f(np.median(a[idx + 8, 1]))
                by_cta = np.zeros(len(idx))
                by_cta[a[idx + 2, 1]] = (end - a[idx + 1, 1].min()) / 1e3
                row["cta_work_us"] = [round(float(x), 2) for x in by_cta]
            else:
                row["main_done"] = [f(np.median(a[idx + 2, 1])), f(a[idx + 2, 1].max())]
                row["reduced"] = [f(np.median(a[idx + 3, 1])), f(a[idx + 3, 1].max())]
                if len(a) > int(idx.max()) + 6 and ((a[idx + 5, 0] & 0xf) == 6).all():
                    ok = a[idx + 5, 1] > 0  # the kPipe form has no first-batch stamp
                    if ok.any():
                        row["epi_first_batch"] = f(np.median(a[idx + 5, 1][ok]))
                    row["epi_loop_done"] = f(np.median(a[idx + 6, 1]))
                    if len(a) > int(idx.max()) + 7 and ((a[idx + 7, 0] & 0xf) == 8).all():
                        ok2 = a[idx + 7, 1] > 0
                        if ok2.any():
                            row["epi_first_again"] = f(np.median(a[idx + 7, 1][ok2]))
                row["end"] = [f(np.median(a[idx + 4, 1])), f(a[idx + 4, 1].max())]
            rows[name] = row
        out["layers"][str(li)] = rows
        print(f"layer {li} (us from the QKV projection's first CTA):", file=sys.stderr)
        for name, row in rows.items():
            print(f"  {name:8s} " + "  ".join(f"{k} {v}" for k, v in row.items()
                                              if k not in ("cta_work_us", "per_cta")),
                  file=sys.stderr)
    out["spans"] = [int(p) for p in kv.positions.cpu().tolist()]  # the traced step's spans
    print(json.dumps({"timeline": "config[2] step", **out}))


def timeline_prefill(args, dev, L, C, cnt, buf, cap_rec):
    """The prefill's GEMM phases (48 lanes x 157 positions in chunks of 448 rows): per
    projection, the median over its launches of dependency release -> main loop done -> cross-CTA
    reduction done -> end (median CTA), in us."""
    import torch

    import ttsnn
    from qwen3tts import PagedKv
    prompt = 157
    stack, _, _, _ = build_device_talker(dev, seed=0, extra_positions=0, lanes_override=0)
    cap = prompt + 3
    per = -(-cap // BLOCK)
    kv = PagedKv(stack.geo, LANES, LANES * per, BLOCK, per, dev)
    x = torch.randn(LANES * prompt, DIM, device=dev)
    for i in range(LANES):
        kv.admit(i, cap, 0)

    def run():
        for i in range(LANES):
            kv.positions[i] = 0
        stack.prefill(kv, [prompt] * LANES, x, max_span=cap)

    run()
    torch.cuda.synchronize()
    L.call("tts_timeline_read", None, 0, C.byref(cnt), 1)
    run()
    torch.cuda.synchronize()
    ttsnn.check(0)
    L.call("tts_timeline_read", buf, cap_rec, C.byref(cnt), 0)
    a = np.frombuffer(buf, dtype=np.uint64).reshape(cap_rec, 4)[:cnt.value].astype(np.int64)
    out = {}
    for name, epi in (("qkv", 4), ("o+down", 2), ("gate/up", 3)):
        idx = np.nonzero(a[:, 0] == (0x100 | epi << 4))[0]
        idx = idx[idx + 4 < len(a)]
        if not len(idx):
            continue
        # launches: a launch's CTAs are released together, launches of one kind >= 10 us apart
        idx = idx[np.argsort(a[idx + 1, 1])]
        rel_t = a[idx + 1, 1]
        cuts = [0] + [i for i in range(1, len(idx)) if rel_t[i] - rel_t[i - 1] > 3000] + [len(idx)]
        ph = []
        for c0, c1 in zip(cuts[:-1], cuts[1:]):
            g = idx[c0:c1]
            rel = a[g + 1, 1].min()
            ph.append([np.median(a[g + 2, 1]) - rel, np.median(a[g + 3, 1]) - rel,
                       np.median(a[g + 4, 1]) - rel, a[g + 4, 1].max() - rel])
        ph = np.median(np.array(ph), 0) / 1e3
        out[name] = {"launches": len(cuts) - 1, "main_done": round(float(ph[0]), 2),
                     "reduced": round(float(ph[1]), 2), "end_median": round(float(ph[2]), 2),
                     "end_max": round(float(ph[3]), 2)}
        print(f"  {name:8s} {out[name]}  (us after the dependency release)", file=sys.stderr)
    print(json.dumps({"timeline": "prefill 48 x 157", "gemm": out}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--clocks-dir", default="/tmp",
                    help="directory for the per-rank nvidia-smi clock samples")
    ap.add_argument("--document-segments", type=int, default=96,
                    help="segments per GPU of the config[4] sample in the default run (0: none)")
    ap.add_argument("--sustained-steps", type=int, default=300,
                    help="graph replays of the sustained leg (clock record under load)")
    ap.add_argument("--workload", default="step",
                    choices=["step", "sweep", "document", "predictor", "frames", "prefill",
                             "codec"],
                    help="step: the config[2] decode step (headline); sweep: config[3]; "
                         "document: a bounded config[4] sample (talker + codec); predictor: "
                         "the depth predictor's frame; frames: the reference's talker loop "
                         "(talker + predictor)")
    ap.add_argument("--lanes", type=int, default=48)
    ap.add_argument("--segments", type=int, default=96, help="segments per GPU (sweep, document)")
    ap.add_argument("--refill", action="store_true")
    ap.add_argument("--kernel", choices=["gemm", "attn", "attn_short", "conv"],
                    help="run a small standalone case of one kernel (for ncu captures)")
    ap.add_argument("--timeline", action="store_true",
                    help="per-CTA phase timeline of one step (needs the tracing library)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel:
        return run_kernel_case(args)
    if args.timeline:
        return run_timeline(args)
    if args.workload == "sweep":
        return run_sweep(args)
    if args.workload == "document":
        return run_document(args)
    if args.workload == "predictor":
        return run_predictor(args)
    if args.workload == "frames":
        return run_frames(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "codec":
        return run_codec(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
