"""Benchmark of Depthformer chunk decoding on B200 (the north-star hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one 2 s chunk of BASELINE.json config 2: the benchmark architecture
("hybrid": d_model 1024, 16 x 64 heads, d_ff 2816, layers 12/20/4, vocab
16388) in bf16 with random-init N(0, 0.02) weights (seed 0), batch 1 with
CFG (cond/uncond rows), guidance 4.0, top-k 40, temperature 1.1, Philox
seed 1 + chunk index: the encoder over 1006 context tokens, 50 temporal steps
and 16 depth steps + sampling per frame = 800 RVQ tokens.

* value: RVQ tokens/s over K chunks with the inputs resident in HBM
  (mrtdf_generate_tokens_dev), CUDA events on the engine's stream,
  max over ranks.
* e2e: the same metric through the reference-facing host API exactly as
  System::generate_chunk drives it (system.cpp:177-333): host context ->
  encoder ids -> mrtdf_generate_tokens (host->device ids, device->host
  tokens) -> llm_to_rvq -> context roll, streaming K chunks.
* roofline: the decode phases, split by stack: the temporal stack against
  the measured HBM peak, the depth stack + lm_head against an L2 read peak
  measured by the engine's own kernel; algorithmic bytes per launch / the
  average launch time, from replaying exactly one stack's launches of a
  chunk (mrtdf_bench_phases).
* cpu_baseline: the CPU oracle (C++ restatement of the reference's eager
  Depthformer, all host threads) on one whole chunk of the same workload.

* codec_decode (rank 0): the next stage of a chunk, the SpectroStream decode
  phase (RVQ codes -> decoder -> iSTFT -> 48 kHz stereo) on the tensor cores;
  `--codec-only` prints just this leg.

Multi-GPU (torchrun, one process per GPU): independent replicas, one stream
per GPU with seed offset by rank, no collective on the data path
(scaling = weak); the barrier and the max-over-ranks reduction use
torch.distributed.

`--impl reference` times the reference's algorithm on the host cores: the
reference (MLX) cannot be built here, so this runs the oracle port, one frame
(16 tokens) per step, without loading the engine library.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200")
sys.path.insert(0, PKG)

METRIC = "RVQ tokens/s (2 s chunk = 800 tokens, bf16, batch 1 + CFG)"
UNIT = "tokens/s"
TOKENS_PER_CHUNK = 800
CHUNK_SECONDS = 2.0
ENC_LEN = 1006


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": "BASELINE config 2: bf16 Depthformer chunk decode, CFG pair (batch 1), guidance 4.0, "
                    "top-k 40, T 1.1, 1006-token context, 50 frames x 16 levels",
        "model": "depthformer-hybrid (d1024 h16x64 ff2816 L12/20/4 V16388)",
        "global_batch": n_gpus,
        "seq_len": ENC_LEN,
        "parallelism": f"replicas x{n_gpus} (no collective)",
        "l2": "inputs larger than L2: 1.2 GB of weights and 165 MB of cross K/V streamed per chunk",
    }


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's eager path)
# ---------------------------------------------------------------------------
def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _oracle():
    """The CPU oracle (test infrastructure; only the CPU legs use it)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py

    oracle_py.set_num_threads(host_cores())
    return oracle_py


def cpu_chunk():
    """One whole chunk of the same workload on the CPU oracle (all host
    threads): random-init weights of seed 0 built in memory, the chunk-0
    encoder ids, encode + 50 frames of (temporal step, 16 x (depth step with
    the level's lm_head rows, CFG mix, top-k 40, T 1.1, Gumbel draws from
    Philox seed 1, embedding feedback)). Returns (tokens/s, ms, threads)."""
    oracle_py = _oracle()
    cfg = oracle_py.preset_ints("hybrid", 1)
    orc = oracle_py.Oracle.from_random(cfg, 0)
    ids = _initial_ids(oracle_py.build_encoder_inputs, 0)
    t0 = time.perf_counter()
    orc.gen_begin(ids)
    for f in range(50):
        orc.gen_frame(f, 4.0, 1.1, 40, True, 1)
    ms = (time.perf_counter() - t0) * 1e3
    orc.close()
    return TOKENS_PER_CHUNK / (ms / 1e3), ms, oracle_py.num_threads()


def _initial_ids(build_encoder_inputs, seed: int) -> np.ndarray:
    """Chunk-0 encoder ids: empty context (all MASK) + 6 style ids drawn
    uniformly from the codec range (stand-in for MusicCoCa tokens)."""
    rng = np.random.default_rng(1000 + seed)
    ctx = -np.ones((250, 16), np.int32)
    style = rng.integers(2, 2 + 16 * 1024, 6).astype(np.int32)
    return build_encoder_inputs(ctx, style, 4, 1024, 2)


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world: int, local: int, backend: str = "nccl"):
    if world <= 1:
        return None
    import torch
    import torch.distributed as dist

    if backend == "nccl":
        torch.cuda.set_device(local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return dist


def max_over_ranks(dist, value: float, device=None) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist, device=None):
    if dist is not None:
        if device is not None and device.type == "cuda":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def run_reference(args):
    """The reference's algorithm on the host cores: the CPU oracle (the
    reference itself needs MLX, which cannot be installed here), all host
    threads, rank 0 only. A step is one frame of the chunk: the temporal
    step and 16 x (depth step with the level's lm_head rows, CFG mix, top-k /
    temperature / Gumbel sampling, embedding feedback) = 16 tokens; value =
    16 / mean step time. The encoder pass runs untimed before frame 0 of
    every 50-frame chunk (its time is reported in the sample text). This
    process never loads libmrtdf.so."""
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    W, K = args.warmup, args.steps
    oracle_py = _oracle()
    cfg = oracle_py.preset_ints("hybrid", 1)
    orc = oracle_py.Oracle.from_random(cfg, 0)
    ids = _initial_ids(oracle_py.build_encoder_inputs, 0)
    t0 = time.perf_counter()
    orc.gen_begin(ids)
    t_enc = time.perf_counter() - t0
    times = []
    chunk = 0
    for s in range(W + K):
        f = s % 50
        if f == 0 and s:
            chunk += 1
            orc.gen_begin(ids)
        t0 = time.perf_counter()
        orc.gen_frame(f, 4.0, 1.1, 40, True, 1 + chunk)
        if s >= W:
            times.append(time.perf_counter() - t0)
    t_frame = float(np.mean(times))
    value = 16 / t_frame
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": t_frame * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init weights N(0,0.02) seed 0; chunk-0 context)",
        "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": oracle_py.num_threads(), "kind": "port",
                         "sample": f"{K} timed frames of config 2 (16 tokens each: temporal step + 16 depth steps "
                                   f"with level-slice lm_head, CFG, top-k 40, T 1.1, Gumbel, feedback); "
                                   f"encoder pass untimed ({t_enc:.2f} s per chunk, not in the value); "
                                   "the reference's MLX build is unavailable here (MLX not installable)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    orc.close()
    return 0


def run_ours(args):
    import torch

    import mrtdf

    rank, world, local = dist_env()
    dist = init_dist(world, local)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg, device=local).load_random(0)
    st = mrtdf.Stream(eng, 1, True)
    ext = torch.cuda.ExternalStream(st.cuda_stream(), device=device)
    W, K = args.warmup, args.steps

    ids = _initial_ids(mrtdf.build_encoder_inputs, rank)
    ids_dev = torch.from_numpy(ids).to(device)
    frames = args.frames
    out_dev = torch.empty((1, 50, cfg.rvq_depth), dtype=torch.int32, device=device)

    def chunk_dev(k):
        o = mrtdf.gen_opts(cfg, frames, temperature=1.1, top_k=40, guidance_weight=4.0, seed=1 + k + 1000 * rank)
        st.generate_tokens_dev(ids_dev.data_ptr(), ENC_LEN, o, out_dev.data_ptr())

    for k in range(W):
        chunk_dev(k)
    st.sync()

    # ---- value: device-resident inputs --------------------------------------
    clocks = ClockSampler(local)
    clocks.start()
    barrier(dist, device)
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" list exactly the timed launches
    e0.record(ext)
    for k in range(K):
        chunk_dev(W + k)
    e1.record(ext)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    st.sync()
    torch.cuda.synchronize(device)
    barrier(dist, device)
    clk = clocks.stop()
    ms_dev = e0.elapsed_time(e1) / K
    ms_dev = max_over_ranks(dist, ms_dev, device)

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    e2e = roofline = None
    if not args.timed_only:
        e2e = e2e_leg(mrtdf, torch, cfg, st, ext, ids, K, rank, dist, device)
        roofline = roofline_leg(mrtdf, eng, cfg, st, peaks)

    value = TOKENS_PER_CHUNK * frames / 50 * world / (ms_dev / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_dev, "rtf": CHUNK_SECONDS * 1e3 / ms_dev, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02) seed 0, RMSNorm scales 1; chunk-0 context + random style)",
        "config": workload_config(world),
        "e2e": e2e,
        "gpu_launches": None,
        "roofline": roofline,
        "clocks": clk,
    }
    # kernels of the chunk graph, counted by the engine from the captured graph
    # (st_launch_count restates the structure and is checked against it)
    launches = st.chunk_kernels()
    if launches <= 0:
        launches = st_launch_count(cfg, frames)
    line["gpu_launches"] = launches * K
    if not args.no_suite and not args.timed_only:
        # BASELINE.json configs 3-5 on the same engine (configs 3 and 4 on rank 0 only)
        if rank == 0:
            line["encoder_microbench"] = encoder_microbench(eng, peaks)
            line["depth_microbench"] = depth_microbench(mrtdf, cfg, st)
        line["multi_stream"] = multi_stream(mrtdf, torch, eng, cfg, device, rank, world, dist)
        if rank == 0:
            # the next stage of a chunk; a failure here is reported in the line
            # (and its traceback on stderr) without losing the headline number
            try:
                line["codec_decode"] = codec_decode(torch, peaks, device, local,
                                                    cpu=world == 1 and not args.no_cpu_baseline)
            except Exception as exc:  # noqa: BLE001
                import traceback

                traceback.print_exc()
                line["codec_decode"] = {"error": f"{type(exc).__name__}: {exc}"}
            try:
                line["style_prompt"] = style_prompt_leg(cpu=world == 1 and not args.no_cpu_baseline, device=local)
            except Exception as exc:  # noqa: BLE001
                import traceback

                traceback.print_exc()
                line["style_prompt"] = {"error": f"{type(exc).__name__}: {exc}"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.timed_only:
        tps, ms_cpu, cores = cpu_chunk()
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": f"one whole chunk of the same workload ({ms_cpu / 1e3:.1f} s: encoder + 50 "
                                          "frames with sampling and feedback) on the CPU oracle"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    st.close()
    eng.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def e2e_leg(mrtdf, torch, cfg, st, ext, ids, K: int, rank: int, dist, device) -> dict:
    """The reference-facing host loop of System::generate_chunk
    (system.cpp:177-333): host context -> encoder ids -> mrtdf_generate_tokens
    (host->device ids, device->host tokens) -> llm_to_rvq -> context roll."""
    ctx = -np.ones((250, cfg.rvq_depth), np.int32)
    style = ids[0, -6:].copy()
    o = mrtdf.gen_opts(cfg, 50, seed=1)
    st.generate_tokens(mrtdf.build_encoder_inputs(ctx, style, 4, cfg.codebook_size, cfg.codec_offset), o)
    barrier(dist, device)
    torch.cuda.synchronize(device)
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(ext)
    for k in range(K):
        enc = mrtdf.build_encoder_inputs(ctx, style, 4, cfg.codebook_size, cfg.codec_offset)
        o = mrtdf.gen_opts(cfg, 50, seed=1 + k + 1000 * rank)
        toks = st.generate_tokens(enc, o)[0]
        rvq = mrtdf.llm_to_rvq(toks, cfg.codebook_size, cfg.codec_offset)
        ctx = mrtdf.context_roll(ctx, rvq)
    e3.record(ext)
    e3.synchronize()
    ms_e2e = max_over_ranks(dist, e2.elapsed_time(e3) / K, device)
    world = dist.get_world_size() if dist is not None else 1
    return {"value": TOKENS_PER_CHUNK * world / (ms_e2e / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": ENC_LEN * 2 * 4 + 8, "d2h_bytes_per_step": TOKENS_PER_CHUNK * 4 + 4,
            "ms_per_chunk": ms_e2e, "rtf": CHUNK_SECONDS * 1e3 / ms_e2e}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch from
# an ncu capture with --cache-control none of a 3-frame chunk
# (bench.py --timed-only --frames 3), frame 1: temporal layer 5 (self, cross,
# FFN) and depth level 3 (self, FFN, self) plus two lm_head slices. Per-launch
# means over a stack's launch mix (temporal: 1 self + 1 cross + 1 FFN per
# layer; depth: 4 self + 4 FFN + 1 lm_head per level).
TRAFFIC_TEMPORAL = (8715008 + 13177088 + 17774336) / 3
TRAFFIC_DEPTH = (4 * (8666624 + 1420800 + 8615424 + 823552) / 2 + 4 * 14456576 + (2048256 + 1632768) / 2) / 9


def roofline_leg(mrtdf, eng, cfg, st, peaks: dict) -> dict:
    """The decode phases split into the temporal stack (fused self / cross /
    FFN phases; weights and cross K/V streamed from HBM) and the depth stack
    + lm_head. Algorithmic bytes per launch / average launch time against the
    measured HBM peak for both: the depth weights carry evict-last hints, but
    the capture shows them read from DRAM again at every level (101 MB of
    depth-layer weights plus the lm_head slices do not stay resident in L2
    when all SMs read them), so HBM bounds both stacks. The L2 read peak,
    measured here with the engine's own read kernel over a 64 MiB buffer, is
    reported beside the depth figure for context. Each stack is timed by
    replaying exactly its launches of one chunk as one CUDA graph between
    CUDA events (mrtdf_bench_phases)."""
    o = mrtdf.gen_opts(cfg, 50, seed=1)
    t_ms, t_n, t_b = st.bench_phases(o, 1, 3)
    d_ms, d_n, d_b = st.bench_phases(o, 2, 3)
    l2_peak = eng.bench_l2_read(64 << 20, 20)
    hbm = peaks.get("hbm_gbs", 6650.0)
    t_ach = t_b / t_n / (t_ms / 1e3 / t_n) / 1e9
    d_ach = d_b / d_n / (d_ms / 1e3 / d_n) / 1e9
    return {"bound": "hbm", "achieved": t_ach, "peak": hbm, "unit": "GB/s", "frac": t_ach / hbm,
            "traffic": TRAFFIC_TEMPORAL, "traffic_unit": "DRAM bytes per launch",
            "traffic_source": "ncu --cache-control none capture of a 3-frame chunk (temporal layer 5 of frame 1)",
            "kernel": "temporal-stack decode phases (fused_self_kernel / fused_cross_kernel / fused_ffn_kernel)",
            "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
            "launches_per_chunk": t_n, "bytes_per_launch": t_b / t_n, "us_per_launch": t_ms * 1e3 / t_n,
            "ms_per_chunk": t_ms,
            "depth": {"bound": "hbm", "achieved": d_ach, "peak": hbm, "unit": "GB/s", "frac": d_ach / hbm,
                      "traffic": TRAFFIC_DEPTH, "traffic_unit": "DRAM bytes per launch",
                      "traffic_source": "ncu --cache-control none capture of a 3-frame chunk (depth level 3 of "
                                        "frame 1: L2 sector hit rate 59-65 %)",
                      "l2_peak": l2_peak, "frac_of_l2_peak": d_ach / l2_peak,
                      "l2_peak_source": "measured: engine L2 read kernel, 64 MiB buffer, 16-byte loads on every SM",
                      "kernel": "depth-stack decode phases + lm_head level slice", "launches_per_chunk": d_n,
                      "bytes_per_launch": d_b / d_n, "us_per_launch": d_ms * 1e3 / d_n, "ms_per_chunk": d_ms}}


def encoder_microbench(eng, peaks: dict) -> dict:
    """the encoder pass + cross-K/V projection of all 20
    temporal layers over 1006 uniform-random ids (seed 2) at 1, 16 and 128
    rows, one CUDA graph per size, against the measured bf16 tensor peak."""
    peak = peaks.get("bf16_tflops", 1590.0)
    out = {"peak_tflops": peak, "peak_source": "measured" if "bf16_tflops" in peaks else "fallback", "rows": {}}
    for rows, reps in ((1, 5), (16, 3), (128, 2)):
        ms, flops = eng.bench_encoder(rows, ENC_LEN, reps)
        tf = flops / (ms / 1e3) / 1e12
        out["rows"][str(rows)] = {"ms": ms, "gflop": flops / 1e9, "tflops": tf, "frac": tf / peak}
    return out


def depth_microbench(mrtdf, cfg, st) -> dict:
    """1000 frames x 16 sequential depth steps (bf16,
    CFG pair, sampler feedback), each frame from an N(0, 1) hidden state
    (seed 3); 50-frame graph replayed 20 times. Achieved GB/s = algorithmic
    bytes per step (depth stack + lm_head level slice + K/V reads) / time;
    the depth weights (103 MB) are held in L2 with evict-last hints."""
    o = mrtdf.gen_opts(cfg, 50, temperature=1.1, top_k=40, guidance_weight=4.0, seed=3)
    us, b, n = st.bench_depth(o, 50, 20)
    return {"frames": 1000, "us_per_step": us, "bytes_per_step": b, "achieved_gbs": b / (us * 1e-6) / 1e9,
            "launches_per_step": n, "us_per_launch": us / n}


# SpectroStream decoder blocks (spectrostream.cpp:328-338): in, out, stride, transposed kernel
CODEC_BLOCKS = [(512, 1024, (2, 1), (4, 3)), (512, 256, (2, 2), (4, 4)), (256, 256, (1, 2), (3, 4)),
                (256, 256, (1, 2), (3, 4)), (256, 128, (1, 3), (3, 6)), (128, 128, (1, 2), (3, 4)),
                (128, 64, (1, 2), (3, 4))]


def codec_flops(S: int, B: int = 1):
    """Multiply-adds x 2 of the decoder's tensor-core convolutions at (B, S)
    (every tap of every kept output, padding taps included, as the GEMMs
    compute them) and of the SIMT 7x7 output convolution."""
    Hs = S + 1
    tc = 2 * B * Hs * (256 * 2560 * 2 + 2560 * 2560)          # input_proj 1x1 convs
    tc += 2 * 2 * B * Hs * 5 * 9 * 512 * 512                   # input_conv
    n, h, w = B, Hs, 5
    for cin, cout, (sh, sw), (kh, kw) in CODEC_BLOCKS:
        if cin != cout:
            tc += 2 * n * h * w * cin * cout                   # shortcut at the input resolution
        cws = (kw - sw) // 2
        for ry in range(sh):
            for rx in range(sw):
                taps = -(-(kh - ry) // sh) * -(-(kw - rx) // sw)
                q0 = -((rx - cws) // sw)
                wq = (w * sw - 1 + cws - rx) // sw - q0 + 1
                tc += 2 * n * h * wq * taps * cin * cout       # transposed-conv phase
        h, w = h * sh, w * sw
        tc += 2 * n * h * w * 9 * cout * cout                  # post conv
        if cout == 1024:
            n *= 2                                             # stereo split
    simt = 2 * n * (h - 4) * w * 49 * 64 * 2
    return tc, simt


def codec_decode(torch, peaks: dict, device, local: int, cpu: bool, S: int = 51, reps: int = 20) -> dict:
    """Codec decode phase of one chunk (system.cpp:372-390): 51 codec frames
    (50 + 1 crossfade) x 16 RVQ levels -> 97,920 stereo samples at 48 kHz.
    Random-init decoder and codebooks (seed 11), codes uniform (seed 12).
    Device-resident codes, one CUDA graph per call, CUDA events on the
    codec's stream (ms); e2e through the host API (codes in, audio out);
    tensor-core roofline against the measured bf16 peak / 2 (dense tf32
    runs at half the bf16 rate). The CPU baseline is the float32 oracle
    (all host threads) on the same chunk."""
    import mrtss

    codec = mrtss.Codec(max_batch=1, max_frames=S, device=local).load_random(11, 16)
    codes = np.random.default_rng(12).integers(0, 1024, size=(1, S, 16), dtype=np.int32)
    dcodes = torch.from_numpy(codes).to(device)
    daudio = torch.empty((1, S * 1920, 2), dtype=torch.float32, device=device)
    ext = torch.cuda.ExternalStream(codec.cuda_stream(), device=device)
    for _ in range(3):
        codec.decode_tokens_dev(dcodes.data_ptr(), 1, S, 16, daudio.data_ptr())
    codec.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(reps):
        codec.decode_tokens_dev(dcodes.data_ptr(), 1, S, 16, daudio.data_ptr())
    e1.record(ext)
    codec.sync()
    ms = e0.elapsed_time(e1) / reps
    t0 = time.perf_counter()
    for _ in range(5):
        codec.decode_tokens(codes[0])
    ms_e2e = (time.perf_counter() - t0) * 1e3 / 5
    tc, simt = codec_flops(S)
    bf16 = peaks.get("bf16_tflops")
    peak = (bf16 if bf16 else 1590.0) / 2
    seconds = S * 1920 / 48000.0
    out = {"frames": S, "levels": 16, "ms": ms, "rtf": seconds * 1e3 / ms, "samples_per_s": S * 1920 / (ms / 1e3),
           "e2e_ms": ms_e2e, "kernels": codec.decode_kernels(1, S),
           "roofline": {"bound": "tensor", "achieved": tc / (ms / 1e3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                        "frac": tc / (ms / 1e3) / 1e12 / peak, "tensor_gflop": tc / 1e9, "simt_gflop": simt / 1e9,
                        "peak_source": ("measured" if bf16 else "fallback") + " bf16 / 2 (tf32)"}}
    codec.close()
    if cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle_py

        oracle_py.set_num_threads(host_cores())
        with tempfile.TemporaryDirectory() as td:
            dec, cb = os.path.join(td, "d.safetensors"), os.path.join(td, "c.safetensors")
            mrtss.write_random_safetensors(11, 16, dec, cb)
            orc = oracle_py.CodecOracle(dec, cb)
        t0 = time.perf_counter()
        orc.decode_tokens(codes[0])
        ms_cpu = (time.perf_counter() - t0) * 1e3
        orc.close()
        out["cpu_baseline"] = {"ms": ms_cpu, "cores": oracle_py.num_threads(), "kind": "port",
                               "sample": f"one full chunk ({S} frames) through the float32 oracle"}
    return out


def style_prompt_leg(cpu: bool, device: int, reps: int = 10) -> dict:
    """The style path once per prompt change (system.cpp:158-161): a 20-piece
    prompt padded to 128 tokens -> MusicCoCa text tower -> 6 style RVQ levels
    -> LLM ids (StyleModel::style_tokens_lm after tokenisation), through the
    host API (ids in, style ids out). Random-init tower with the reference's
    64,000-token vocabulary (numpy seed 13). float32 CUDA-core GEMMs: the
    roofline is against the nominal B200 float32 FMA rate (148 SMs x 128
    lanes x 2 x 1.965 GHz = 74.4 TFLOP/s). CPU baseline: the float32 oracle
    (all host threads) on the same prompt."""
    import mrtmc

    rng = np.random.default_rng(14)
    ids = np.zeros((1, 128), np.int32)
    pad = np.ones((1, 128), np.float32)
    ids[0, 0] = 1
    ids[0, 1:21] = rng.integers(2, 64000, 20)
    pad[0, :21] = 0
    with tempfile.TemporaryDirectory() as td:
        enc, cb = os.path.join(td, "musiccoca_encoder.safetensors"), os.path.join(td, "musiccoca_codebooks.safetensors")
        mrtmc.write_random_safetensors(enc, cb, seed=13)
        model = mrtmc.StyleModel(max_batch=1, device=device).load_safetensors(enc, cb)
        for _ in range(3):
            toks = model.style_tokens_lm(ids, pad)
        t0 = time.perf_counter()
        for _ in range(reps):
            toks = model.style_tokens_lm(ids, pad)
        ms = (time.perf_counter() - t0) * 1e3 / reps
        L, D, FF, P = 128, 768, 3072, 3072
        flops = 2.0 * L * (12 * (3 * D * D + D * D + 2 * D * FF) + 2 * P * D) + 12 * 12 * 4.0 * L * L * 64 \
            + 2.0 * P * D + 12 * 4.0 * L * 256
        out = {"prompt_tokens": 21, "padded_len": L, "ms": ms, "kernels": model.embed_kernels(1, L),
               "gflop": flops / 1e9,
               "roofline": {"bound": "fp32 FMA", "achieved": flops / (ms / 1e3) / 1e12, "peak": 74.4,
                            "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / 74.4,
                            "peak_source": "nominal (no measured fp32 peak)"},
               "style_ids": toks[0].tolist()}
        model.close()
        if cpu:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle_py

            oracle_py.set_num_threads(host_cores())
            orc = oracle_py.StyleOracle(enc, cb)
            t0 = time.perf_counter()
            emb = orc.embed_text(ids, pad)
            orc.quantize(emb, 6)
            ms_cpu = (time.perf_counter() - t0) * 1e3
            orc.close()
            out["cpu_baseline"] = {"ms": ms_cpu, "cores": oracle_py.num_threads(), "kind": "port",
                                   "sample": "the same prompt through the float32 oracle"}
    return out


def multi_stream(mrtdf, torch, eng, cfg, device, rank: int, world: int, dist, n_streams: int = 64,
                 per_group: int = 64, rounds: int = 2) -> dict:
    """64 independent CFG streams per GPU (bf16, top-k 40,
    T 1.1), seeds 100 + global stream index, batched as one engine stream of
    64 CFG pairs (128 rows: RMSNorm + tcgen05 GEMM projections; with
    per_group < 64, several engine streams run concurrently on their own
    CUDA streams). Aggregate tokens/s over all ranks; a stream holds real
    time when its chunk (2 s of audio) takes <= 2 s."""
    groups = n_streams // per_group
    sts = [mrtdf.Stream(eng, per_group, True) for _ in range(groups)]
    exts = [torch.cuda.ExternalStream(s.cuda_stream(), device=device) for s in sts]
    ids_dev, out_dev, seeds = [], [], []
    for g in range(groups):
        base = 100 + rank * n_streams + g * per_group
        ids = np.concatenate([_initial_ids(mrtdf.build_encoder_inputs, base + i) for i in range(per_group)], axis=0)
        ids_dev.append(torch.from_numpy(ids).to(device))
        out_dev.append(torch.empty((per_group, 50, cfg.rvq_depth), dtype=torch.int32, device=device))
        seeds.append([base + i for i in range(per_group)])

    def launch(r):
        for g, st in enumerate(sts):
            o = mrtdf.gen_opts(cfg, 50, temperature=1.1, top_k=40, guidance_weight=4.0)
            st.generate_tokens_dev(ids_dev[g].data_ptr(), ENC_LEN, o, out_dev[g].data_ptr(),
                                   seeds=[sd + 1000 * r for sd in seeds[g]])

    launch(0)  # warm-up: builds every stream's chunk graph
    for st in sts:
        st.sync()
    barrier(dist, device)
    ts = torch.cuda.Stream(device=device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    e0.record(ts)
    for x in exts:
        x.wait_event(e0)
    for r in range(rounds):
        launch(1 + r)
    for x in exts:
        ev = torch.cuda.Event()
        ev.record(x)
        ts.wait_event(ev)
    e1.record(ts)
    e1.synchronize()
    for st in sts:
        st.sync()
    ms_round = max_over_ranks(dist, e0.elapsed_time(e1) / rounds, device)
    for st in sts:
        st.close()
    total = n_streams * world
    return {"streams_per_gpu": n_streams, "streams": total, "engine_streams_per_gpu": groups,
            "rows_per_engine_stream": 2 * per_group, "rounds": rounds, "ms_per_chunk": ms_round,
            "tokens_per_s": TOKENS_PER_CHUNK * total / (ms_round / 1e3), "rtf_per_stream": CHUNK_SECONDS * 1e3 / ms_round,
            "streams_rtf_ge_1": total if ms_round <= CHUNK_SECONDS * 1e3 else 0}


def st_launch_count(cfg, frames: int = 50, fused: bool = True) -> int:
    """Kernels of one bf16 chunk graph (our own) for one CFG pair: encoder +
    PAD embedding + 50 x (temporal layers + 16 x (depth layers + lm_head +
    sampler)). Fused phases: 3 launches per temporal layer (self, cross,
    FFN), 2 per depth layer; otherwise 7 and 4 (the self-attention inside
    the q/k/v cluster launch)."""
    enc = 1 + cfg.num_encoder_layers * 7 + 2
    temporal = cfg.num_temporal_layers * (3 if fused else 7)
    depth = cfg.num_depth_layers * (2 if fused else 4) + 1 + 1
    return enc + 1 + frames * (temporal + cfg.rvq_depth * depth)


def run_codec_only(args) -> int:
    import torch

    _, _, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = {}
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    out = codec_decode(torch, peaks, device, local, cpu=not args.no_cpu_baseline)
    print(json.dumps({"metric": "SpectroStream decode phase, ms per 2.04 s chunk (51 frames x 16 levels)",
                      "value": out["ms"], "unit": "ms", "higher_is_better": False, "n_gpus": 1, "dtype": "f32/tf32",
                      "data": "synthetic (random-init decoder and codebooks seed 11, codes seed 12)",
                      "codec_decode": out}), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-suite", action="store_true", help="skip the config 3-5 measurements")
    ap.add_argument("--timed-only", action="store_true",
                    help="only the timed chunks (for an ncu launch list): no e2e, roofline, suite or CPU legs")
    ap.add_argument("--frames", type=int, default=50,
                    help="frames per timed chunk with --timed-only (a short chunk for ncu captures)")
    ap.add_argument("--codec-only", action="store_true",
                    help="only the SpectroStream decode-phase leg (one GPU), as its own JSON line")
    args = ap.parse_args(argv)
    if args.frames != 50 and not args.timed_only:
        ap.error("--frames applies to --timed-only runs (the headline chunk is 50 frames)")
    if not 1 <= args.frames <= 50:
        ap.error("--frames must be in [1, 50]")
    if args.codec_only:
        return run_codec_only(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
