"""Throughput of the cuda backend: RTFx (audio seconds per wall second) of the whole path
(log-mel front-end, 24-layer encoder, TDT greedy decode) on the whole-box workload: 4096
synthetic speech-like clips of 2-30 s (durations uniform, seeded), with seeded random-init
weights of the Parakeet-TDT-0.6B-v3 architecture, bf16. One process per GPU: the clips are
dealt to the GPUs in contiguous ranges of the length order, cut where the predicted shard
times balance (tinybark_b200.dp.deal), and each rank
transcribes its shard end to end with no collective on the data path (strong scaling: the
same 4096 clips at every GPU count; one GPU runs them all as one batch).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints one JSON line (rank 0). `value` is device-timed with the samples resident in HBM
(16-bit PCM, as tinybark's transcribe_pcm takes it); `e2e` is the same metric through the
public API (Bark.tokens_batch on host int16 arrays, host<->device copies inside the timed
region). `roofline` is the persistent TDT decoder (the step's largest kernel), timed
inside the timed region; `roofline_kernels` adds the encoder's FFN GEMM, attention,
depthwise conv and LayerNorm timed alone at the step's shapes; `config0` is the batch-1
fp32 end-to-end transcription of one 10 s clip (cold run, then warm runs).
`--impl reference` times the reference path's CPU implementation (the CPU oracle:
tinybark's front-end restated in numpy, transformers' ParakeetEncoder, the TDT loop
restated in torch) on the host cores.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "RTFx (audio-s per wall-s) per box at 1/2/4/8 B200; encoder ms per 10 s clip"
WORKLOAD = ("whole-box: 4096 synthetic clips 2-30 s (uniform, seeded) dealt to the GPUs in contiguous length ranges "
            "balancing predicted time, packed end to end, front-end + encoder + TDT decode")
SEED = 4
CLIPS = 4096
# Algorithmic work of the greedy loop (tinybark/tinygrad/model.py:162-233): the joint on
# every iteration (8193 token + 5 duration logits from 640 inputs) and, for every emitted
# token, the prediction step (two LSTM layers of [x | h] 1280 -> 2560 gates, projector 640 -> 640).
JOINT_FLOP = 2 * (8193 + 5) * 640
STEP_FLOP = 2 * 2 * 2560 * 1280 + 2 * 640 * 640


def args_parser():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--clips", type=int, default=CLIPS, help="clips of the whole-box set, dealt over the GPUs")
    p.add_argument("--layers", type=int, default=24)
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-config0", action="store_true", help="skip the batch-1 fp32 end-to-end line")
    p.add_argument("--micro", action="store_true", help="per-kernel microbenchmarks at encoder shapes")
    p.add_argument("--only", default="", help="--micro: comma-separated cases (layernorm,ffn,mx,conv,mhsa,decode,decode_loop,batch1,longform,load,text; config0 only by name)")
    p.add_argument("--rows", default="125,4000,32000", help="--micro: B*T values")
    p.add_argument("--lengths", default="125,375,1500", help="--micro: T values of the attention cases")
    p.add_argument("--micro-dtypes", default="bf16,fp32")
    p.add_argument("--lanes", default="64,512", help="--micro: decoder lanes")
    p.add_argument("--lane-seconds", default="2,30", help="--micro decode_loop: the lanes' clip lengths, lo,hi seconds")
    p.add_argument("--profile", action="store_true", help="one step of the pipeline, for a profiler")
    p.add_argument("--decode-groups", type=int, default=0, help="concurrent decoder groups (0: by batch size)")
    return p


def rank_info():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def box_frames(count: int) -> list[int]:
    """Feature frames of every clip of the whole-box set (durations uniform in [2, 30) s)."""
    from tinybark_b200 import lengths, synthetic

    return [lengths.frames(int(round(d * 16000))) for d in synthetic.durations(count, SEED * 1000)]


def shard(rank: int, world: int, count: int = CLIPS):
    """This rank's clips of the whole-box set, as int16 PCM, longest first (the order
    Bark.tokens_batch gives a batch), with their durations: the set's clips dealt over
    `world` GPUs by dp.deal; each clip's audio seeded by its index in the set, so a clip
    is the same whichever rank draws it."""
    from tinybark_b200 import dp, synthetic

    durs_all = synthetic.durations(count, SEED * 1000)
    mine = dp.deal(box_frames(count), world)[rank]
    mine = sorted(mine, key=lambda i: (-durs_all[i], i))
    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 4)) as pool:
        pcm = list(pool.map(lambda i: synthetic.clip(float(durs_all[i]), SEED * 10_000_000 + i), mine))
    return pcm, np.asarray([durs_all[i] for i in mine])


def reduce_over_ranks(x: float, op: str, device) -> float:
    """x reduced ("max" or "sum") over the ranks of the default process group, as float64
    on `device`; x itself without a group. Every rank must call it at the same point."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def weights(layers: int):
    from tinybark_b200 import synthetic
    from tinybark_b200 import weights as w

    cfg = synthetic.config(layers)
    return w.convert(synthetic.state_dict(0, layers=layers), cfg), cfg


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 8:
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[4:]))
                except ValueError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for _, _, flags in rows for n, f in zip(names, flags) if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def cpu_pipeline_factory(layers: int):
    """The reference path on the host: tinybark's front-end (restated in numpy),
    transformers' ParakeetEncoder (bf16 when the CPU has AVX512-BF16, as
    tinybark/pytorch/__init__.py:53-58 picks, else fp32), and the TDT loop."""
    import torch

    from oracle import decoder, encoder, frontend
    from tinybark_b200 import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
    sd = synthetic.state_dict(0, layers=layers)
    bf16 = getattr(torch.cpu, "_is_avx512_bf16_supported", lambda: False)()
    dtype = torch.bfloat16 if bf16 else torch.float32
    try:
        enc_model = encoder.hf_encoder(sd, layers).to(dtype)
    except Exception:  # transformers without Parakeet: the restated encoder
        enc_model = None
    proj_w = torch.from_numpy(sd["encoder_projector.weight"]).to(dtype)
    proj_b = torch.from_numpy(sd["encoder_projector.bias"]).to(dtype)
    dec = decoder.Decoder(sd)

    def run(samples: np.ndarray) -> list[int]:
        if samples.dtype == np.int16:
            samples = synthetic.to_float(samples)
        feats = frontend.features(samples)
        if len(feats) < 2:
            return []
        with torch.inference_mode():
            if enc_model is not None:
                hidden = enc_model(torch.from_numpy(feats)[None].to(dtype)).last_hidden_state[0]
                enc = torch.nn.functional.linear(hidden, proj_w, proj_b).float().numpy()
            else:
                enc = encoder.encode(sd, feats)
        return dec.greedy(enc, len(feats))

    return run, ("bf16" if bf16 else "fp32"), torch.get_num_threads()


def cpu_baseline(clips, durs, layers: int, budget_s: float):
    run, dtype, threads = cpu_pipeline_factory(layers)
    run(clips[0][:16000])  # warm-up
    # Clips spread over the shard's lengths (it is ordered longest first), until the budget.
    pick = np.unique(np.linspace(0, len(clips) - 1, min(len(clips), 64)).round().astype(int))
    order = [int(i) for k in range(4) for i in pick[k::4]]
    audio, start, n = 0.0, time.perf_counter(), 0
    while n < len(order) and (n == 0 or time.perf_counter() - start < budget_s):
        run(clips[order[n]])
        audio += durs[order[n]]
        n += 1
    wall = time.perf_counter() - start
    return {"value": audio / wall, "unit": "audio-s/s", "cores": threads, "kind": "port",
            "sample": f"{n} clips ({audio:.1f} s of audio) spread over the lengths of the same workload, one at a "
                      f"time, {dtype}, tinybark front-end restated + transformers ParakeetEncoder + TDT loop restated"}


def run_reference(args):
    rank, world, _ = rank_info()
    if rank != 0:
        return
    # A bounded sample of the same set: the first clips of rank 0's shard at this GPU
    # count, one clip per step.
    from tinybark_b200 import dp

    n = max(8, args.steps + args.warmup)
    clips, durs = shard(0, 1, args.clips) if world == 1 else shard(0, world, args.clips)
    pick = np.linspace(0, len(clips) - 1, n).round().astype(int)
    clips, durs = [clips[i] for i in pick], durs[pick]
    run, dtype, threads = cpu_pipeline_factory(args.layers)
    for i in range(args.warmup):
        run(clips[i % len(clips)][:32000])
    audio, times = 0.0, []
    for i in range(args.steps):
        t0 = time.perf_counter()
        run(clips[i % len(clips)])
        times.append(time.perf_counter() - t0)
        audio += durs[i % len(clips)]
    wall = sum(times)
    value = audio / wall
    del dp
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * wall / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": {"workload": WORKLOAD, "clips": args.clips, "layers": args.layers,
                   "sample": "one clip per step, spread over the lengths of rank 0's shard, on one host process"},
        "cpu_baseline": {"value": value, "unit": "audio-s/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} clips ({audio:.1f} s audio), {dtype}"},
        "e2e": {"value": value, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = rank_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(minutes=10), device_id=dev)

    import tinybark_b200
    from tinybark_b200 import _lib as L
    from tinybark_b200.engine import Engine

    clips, durs = shard(rank, world, args.clips)
    tensors, cfg = weights(args.layers)
    bark = tinybark_b200.load("gpu", dtype="bf16", weights=(tensors, cfg))
    eng: Engine = bark.engine
    audio_rank = float(np.sum(durs))
    plan = eng.plan([len(c) // 160 for c in clips])
    samples, sample_off = eng.upload(clips)
    torch.cuda.synchronize()
    dec_ev = []  # (start, end) of each decode in the timed region

    def step(events=None):
        feats = eng.features(samples, sample_off, plan)
        enc = eng.encode(feats, plan)
        if events is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        out = eng.decode(enc, plan, groups=args.decode_groups or None)
        if events is not None:
            b.record()
            events.append((a, b))
        return out

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        return reduce_over_ranks(x, "max", dev)

    for _ in range(args.warmup):
        step()
    eng.check()

    # Device-timed region, inputs resident.
    barrier()
    launches0 = L.lib.tb_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record()
        for _ in range(args.steps):
            tokens, counts = step(dec_ev)
        end.record()
        torch.cuda.synchronize()
    launches = (L.lib.tb_launch_count() - launches0) // args.steps
    eng.check()
    ms = max_over_ranks(start.elapsed_time(end)) / args.steps
    decode_s = sum(a.elapsed_time(b) for a, b in dec_ev) / len(dec_ev) / 1000
    iters = int(eng.lane_iterations().sum().item()) if not args.decode_groups else None
    emitted = int(counts.sum().item())
    barrier()
    stages = stage_split(eng, samples, sample_off, plan, args.decode_groups or None)
    total_audio = reduce_over_ranks(audio_rank, "sum", dev)
    value = total_audio / (ms / 1000.0)

    # End to end through the public API: host int16 arrays in, token lists out.
    bark.tokens_batch(clips)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        bark.tokens_batch(clips)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    h2d = int(sum(len(c) for c in clips) * 2 + (len(clips) + 1) * 8 + plan.meta.numel() * 4)
    d2h = int(len(clips) * plan.max_cap * 4 + len(clips) * 4)

    # Encoder ms per 10 s clip, batch 1 (bf16).
    from tinybark_b200 import synthetic

    one = [synthetic.clip(10.0, 0)]
    p1 = eng.plan([1000])
    s1, o1 = eng.upload(one)
    f1 = eng.features(s1, o1, p1)
    for _ in range(3):
        eng.encode(f1, p1)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(10):
        eng.encode(f1, p1)
    b.record()
    torch.cuda.synchronize()
    enc10_ms = a.elapsed_time(b) / 10

    hbm, tflops, kind = peaks()
    sustained = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops_sustained") \
        if (ROOT / "MEASURED_PEAKS.json").exists() else None
    dec_flop = (iters * JOINT_FLOP + emitted * STEP_FLOP) if iters is not None else None
    roof_peak = sustained or 1400.0
    roofline = {
        "bound": "tensor", "unit": "TFLOP/s", "peak": roof_peak,
        "peak_kind": f"{'measured' if sustained else 'fallback'} sustained bf16 (timed inside the step)",
        "kernel": f"decode_tc_kernel (persistent TDT greedy decode, {len(clips)} lanes)",
        "achieved": None if dec_flop is None else dec_flop / decode_s / 1e12,
        "frac": None if dec_flop is None else dec_flop / decode_s / 1e12 / roof_peak,
        "traffic": traffic_of("decode_tc_kernel_bytes_per_lane_iter", iters),
        "work": {"lane_iterations": iters, "emitted_tokens": emitted, "flop": dec_flop,
                 "flop_per_iteration": JOINT_FLOP, "flop_per_token": STEP_FLOP},
        "launch_ms": decode_s * 1000,
    }
    kernels = roofline_kernels(eng, plan, dev, hbm, tflops, kind)

    if world > 1:
        dist.barrier()
    if rank == 0:
        base = None
        if world == 1 and not args.no_cpu_baseline:
            base = cpu_baseline(clips, durs, args.layers, args.cpu_seconds)
        config0 = None if (world > 1 or args.no_config0) else run_config0(args, tensors, cfg)
        line = {
            "metric": METRIC, "value": value, "unit": "audio-s/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "clips": args.clips, "clips_rank0": len(clips),
                       "audio_s_rank0": round(audio_rank, 2), "audio_s_total": round(total_audio, 2),
                       "encoder_frames_rank0": int(plan.batch.t3_total), "layers": args.layers,
                       "parallelism": f"dp{world}", "input": "int16 PCM",
                       "l2": "inputs larger than L2 (samples and weights, >126 MB per step)"},
            "encoder_ms_per_10s_clip": enc10_ms,
            "stages_ms_rank0": stages,
            "roofline": roofline,
            "roofline_kernels": kernels,
            "cpu_baseline": base,
            "e2e": {"value": total_audio / (e2e_ms / 1000.0), "unit": "audio-s/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "config0": config0,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def traffic_of(key: str, units):
    """DRAM bytes per launch from profiles/traffic.json (bytes per unit, from one ncu
    capture) scaled to `units`, or None."""
    path = ROOT / "profiles" / "traffic.json"
    if units is None or not path.exists():
        return None
    per = json.loads(path.read_text()).get(key)
    return None if per is None else per * units


def roofline_kernels(eng, plan, dev, hbm, tflops, kind):
    """The encoder's kernels timed alone (median of launches with L2 flushed) at this
    step's shapes: FFN up (tcgen05 GEMM, SiLU epilogue), rel-pos attention over the step's
    clips, depthwise conv + SiLU, LayerNorm; each against its roofline (burst bf16 peak or
    HBM copy bandwidth)."""
    import torch

    from tinybark_b200 import _lib as L
    from tinybark_b200 import kernels as K

    M = plan.batch.t3_total
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *s, dt=torch.bfloat16: torch.randn(*s, device=dev, generator=g).to(dt)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = []
    x, w1 = rnd(M, 1024), rnd(4096, 1024) / 32
    h = torch.empty(M, 4096, device=dev, dtype=torch.bfloat16)
    ep = L.Epilogue(kind=L.EPI_SILU, out_dtype=L.BF16, out=h.data_ptr(), ldo=4096)
    s = timed(lambda: K.gemm(x, w1, ep), iters=10, flush=flush)
    fl = 2.0 * M * 4096 * 1024
    out.append({"kernel": "gemm_tc2_kernel FFN up + SiLU" if M >= 2048 else "gemm_tc_kernel FFN up + SiLU",
                "rows": M, "bound": "tensor", "us": s * 1e6, "achieved": fl / s / 1e12, "peak": tflops,
                "unit": "TFLOP/s", "frac": fl / s / 1e12 / tflops, "peak_kind": f"{kind} burst bf16",
                "traffic": traffic_of("gemm_ffn_up_bytes_per_row", M)})
    del h
    t3 = [int(t) for t in plan.t3]
    frames = K.Frames(t3, L.BF16, dev)
    qu, qv, k, v = (rnd(M, 1024) for _ in range(4))
    T = max(t3)
    eng.ensure_len(T)
    rel = rnd(2 * eng.max_len - 1, 1024)
    rel_c = K.rel_bias(rel, rnd(1024, dt=torch.float32), rnd(1024, dt=torch.float32))
    att = torch.empty(M, 1024, device=dev, dtype=torch.bfloat16)
    s = timed(lambda: K.attention(qu, qv, k, v, rel, eng.max_len, frames, att, rel_c), iters=5, flush=flush)
    fl = 6.0 * 1024 * sum(t * t for t in t3)
    out.append({"kernel": "relpos_attention_tc", "rows": M, "clips": len(t3), "bound": "tensor", "us": s * 1e6,
                "achieved": fl / s / 1e12, "peak": tflops, "unit": "TFLOP/s", "frac": fl / s / 1e12 / tflops,
                "peak_kind": f"{kind} burst bf16", "work": "6 T^2 1024 FLOP per clip (QK, banded position scores, PV)"})
    del qu, qv, k, v, att
    glu, dwo = rnd(M, 1024), torch.empty(M, 1024, device=dev, dtype=torch.bfloat16)
    dww, dwb = rnd(1024, 9, dt=torch.float32), rnd(1024, dt=torch.float32)
    s = timed(lambda: K.depthwise(glu, dww, dwb, frames, dwo), iters=10, flush=flush)
    nb = 2.0 * M * 1024 * 2
    out.append({"kernel": "depthwise_stream_kernel (k=9, folded BN, SiLU)", "rows": M, "bound": "hbm",
                "us": s * 1e6, "achieved": nb / s / 1e9, "peak": hbm, "unit": "GB/s", "frac": nb / s / 1e9 / hbm,
                "work": "bf16 rows read once and written once"})
    del glu, dwo
    xf, lw, lb = rnd(M, 1024, dt=torch.float32), rnd(1024, dt=torch.float32), rnd(1024, dt=torch.float32)
    y = torch.empty(M, 1024, device=dev, dtype=torch.bfloat16)
    s = timed(lambda: K.layernorm(xf, lw, lb, y), iters=10, flush=flush)
    nb = M * 1024 * (4.0 + 2.0)
    out.append({"kernel": "layernorm_kernel (fp32 in, bf16 out)", "rows": M, "bound": "hbm", "us": s * 1e6,
                "achieved": nb / s / 1e9, "peak": hbm, "unit": "GB/s", "frac": nb / s / 1e9 / hbm})
    K.check(dev)
    return out


def run_config0(args, tensors, cfg):
    """Config 0: batch 1, fp32, one 10 s clip (seed 0) end to end through Bark.tokens, timed
    as tinybark's benchmark worker times a clip (a first, cold call after loading, then warm
    calls; tinybark/bench/worker.py:37-44); plus the fp32 encoder alone."""
    import torch

    import tinybark_b200
    from tinybark_b200 import synthetic

    bark = tinybark_b200.load("gpu", dtype="fp32", weights=(tensors, cfg))
    clip = synthetic.to_float(synthetic.clip(10.0, 0))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = bark.tokens(clip)
    cold = time.perf_counter() - t0
    warm = []
    for _ in range(5):
        t0 = time.perf_counter()
        tokens = bark.tokens(clip)
        warm.append(time.perf_counter() - t0)
    assert tokens == first
    eng = bark.engine
    plan = eng.plan([1000])
    s1, o1 = eng.upload([clip])
    f1 = eng.features(s1, o1, plan)
    for _ in range(2):
        eng.encode(f1, plan)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        eng.encode(f1, plan)
    b.record()
    torch.cuda.synchronize()
    enc_ms = a.elapsed_time(b) / 5
    del bark
    torch.cuda.empty_cache()
    return {"workload": "batch 1, fp32, one 10 s clip (seed 0), Bark.tokens from a host float32 array",
            "cold_ms": cold * 1000, "warm_ms_best": min(warm) * 1000, "warm_ms_mean": statistics.mean(warm) * 1000,
            "rtfx_warm": 10.0 / min(warm), "encoder_ms": enc_ms, "tokens": len(first)}


def timed(fn, iters: int = 10, flush=None) -> float:
    """Median seconds of fn() over `iters` launches, each timed alone with CUDA events on
    the current stream, L2 flushed before each (a write larger than L2)."""
    import torch

    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) / 1000)
    return statistics.median(times)


def run_micro(args):
    """Per-kernel microbenchmarks at encoder shapes, inputs N(0, 1) from a seed: LayerNorm
    over [B*T, 1024]; the SiLU FFN 1024->4096->1024; the conv module (pointwise 1024->2048
    + GLU, depthwise k=9 + SiLU, pointwise 1024->1024); rel-pos MHSA with q/k/v
    [B, 8, T, 128] and positions [2T-1, 1024]. One JSON line per case."""
    import torch

    from tinybark_b200 import _lib as L
    from tinybark_b200 import kernels as K

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    hbm, tflops, kind = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    only = set(filter(None, args.only.split(",")))
    want = lambda k: not only or k in only
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *s, dt=torch.float32: torch.randn(*s, device=dev, generator=g).to(dt)

    def emit(**kw):
        print(json.dumps(kw), flush=True)

    for dt_name in args.micro_dtypes.split(","):
        dt = torch.bfloat16 if dt_name == "bf16" else torch.float32
        esz = 2 if dt == torch.bfloat16 else 4
        code = L.BF16 if dt == torch.bfloat16 else L.F32
        for bt in map(int, filter(None, args.rows.split(","))):
            if want("layernorm"):
                x, w, b = rnd(bt, 1024), rnd(1024), rnd(1024)
                y = torch.empty(bt, 1024, device=dev, dtype=dt)
                s = timed(lambda: K.layernorm(x, w, b, y), flush=flush)
                nbytes = bt * 1024 * (4 + esz)
                emit(kernel="layernorm", dtype=dt_name, rows=bt, us=s * 1e6, gbs=nbytes / s / 1e9,
                     frac=nbytes / s / 1e9 / hbm, bound="hbm")
            if want("ffn"):
                x = rnd(bt, 1024, dt=dt)
                w1, w2 = rnd(4096, 1024, dt=dt) / 32, rnd(1024, 4096, dt=dt) / 64
                h = torch.empty(bt, 4096, device=dev, dtype=dt)
                res = rnd(bt, 1024)
                e1 = L.Epilogue(kind=L.EPI_SILU, out_dtype=code, out=h.data_ptr(), ldo=4096)
                e2 = L.Epilogue(kind=L.EPI_RESIDUAL, out=res.data_ptr(), ldo=1024, alpha=0.5)
                s1 = timed(lambda: K.gemm(x, w1, e1), flush=flush)
                s2 = timed(lambda: K.gemm(h, w2, e2), flush=flush)
                fl = 2 * bt * 1024 * 4096
                for name, s in (("ffn_up_silu", s1), ("ffn_down_residual", s2)):
                    emit(kernel=name, dtype=dt_name, rows=bt, us=s * 1e6, tflops=fl / s / 1e12,
                         frac=fl / s / 1e12 / tflops, bound="tensor" if code == L.BF16 else "fma")
            if want("mx") and code == L.BF16:
                # The FFN-up GEMM on block-scaled FP8 (the ffn="mxfp8" option): activations
                # quantized (tb_mx_quantize), then the kind::mxf8f6f4 GEMM with SiLU.
                x = rnd(bt, 1024, dt=dt)
                xa, wa = K.MX(x), K.MX(rnd(4096, 1024, dt=dt) / 32)
                h = torch.empty(bt, 4096, device=dev, dtype=dt)
                e1 = L.Epilogue(kind=L.EPI_SILU, out_dtype=code, out=h.data_ptr(), ldo=4096)
                quant = lambda: L.check(L.lib.tb_mx_quantize(code, x.data_ptr(), x.stride(0), bt, 1024,
                                                             xa.codes.data_ptr(), xa.scales.data_ptr(),
                                                             torch.cuda.current_stream().cuda_stream), "tb_mx_quantize")
                sq = timed(quant, flush=flush)
                sg = timed(lambda: K.gemm_mx(xa, wa, e1), flush=flush)
                nbytes = bt * 1024 * (2 + 1) + bt * 1024 // 32
                emit(kernel="mx_quantize", dtype="bf16->mxfp8", rows=bt, us=sq * 1e6, gbs=nbytes / sq / 1e9,
                     frac=nbytes / sq / 1e9 / hbm, bound="hbm")
                fl = 2 * bt * 1024 * 4096
                emit(kernel="ffn_up_silu_mxfp8", dtype="mxfp8", rows=bt, us=sg * 1e6, tflops=fl / sg / 1e12,
                     frac_of_2x_bf16=fl / sg / 1e12 / (2 * tflops), bound="tensor")
            if want("conv"):
                x = rnd(bt, 1024, dt=dt)
                pw1, pw2 = rnd(2048, 1024, dt=dt) / 32, rnd(1024, 1024, dt=dt) / 32
                glu = torch.empty(bt, 1024, device=dev, dtype=dt)
                dwo = torch.empty(bt, 1024, device=dev, dtype=dt)
                res = rnd(bt, 1024)
                frames = K.Frames([bt], code, dev)
                dww, dwb = rnd(1024, 9), rnd(1024)
                e1 = L.Epilogue(kind=L.EPI_GLU, out_dtype=code, out=glu.data_ptr(), ldo=1024)
                e2 = L.Epilogue(kind=L.EPI_RESIDUAL, out=res.data_ptr(), ldo=1024, alpha=1.0)
                s1 = timed(lambda: K.gemm(x, pw1, e1), flush=flush)
                s2 = timed(lambda: K.depthwise(glu, dww, dwb, frames, dwo), flush=flush)
                s3 = timed(lambda: K.gemm(dwo, pw2, e2), flush=flush)
                emit(kernel="conv_pw1_glu", dtype=dt_name, rows=bt, us=s1 * 1e6,
                     tflops=2 * bt * 1024 * 2048 / s1 / 1e12)
                nbytes = 2 * bt * 1024 * esz
                emit(kernel="conv_depthwise_silu", dtype=dt_name, rows=bt, us=s2 * 1e6, gbs=nbytes / s2 / 1e9,
                     frac=nbytes / s2 / 1e9 / hbm, bound="hbm")
                emit(kernel="conv_pw2_residual", dtype=dt_name, rows=bt, us=s3 * 1e6,
                     tflops=2 * bt * 1024 * 1024 / s3 / 1e12)
            if want("decode") and code == L.BF16 and bt == max(map(int, args.rows.split(","))):
                # The decoder's GEMMs at `--lanes` lanes, weights resident in L2 as in the
                # greedy loop (back-to-back launches, no flush).
                for lanes in map(int, args.lanes.split(",")):
                    z, x0 = rnd(lanes, 640, dt=dt), rnd(lanes, 1280, dt=dt)
                    wj, wl, wp = rnd(8448, 640, dt=dt) / 25, rnd(2560, 1280, dt=dt) / 36, rnd(640, 640, dt=dt) / 25
                    bj, bl, bp = rnd(8448), rnd(2560), rnd(640)
                    keys = torch.zeros(2, lanes, dtype=torch.int64, device=dev)
                    c, h, mask = rnd(lanes, 640), rnd(lanes, 640), torch.ones(lanes, dtype=torch.int32, device=dev)
                    dec, zz = torch.empty(lanes, 640, device=dev), torch.empty(lanes, 640, device=dev, dtype=dt)
                    enc, erow = rnd(lanes, 640), torch.arange(lanes, dtype=torch.int32, device=dev)
                    hout = torch.empty(lanes, 1280, device=dev, dtype=dt)
                    cases = {
                        "decode_joint_argmax": (z, wj, L.Epilogue(kind=L.EPI_ARGMAX, bias=bj.data_ptr(),
                                                                   keys=keys[0].data_ptr(), keys2=keys[1].data_ptr(),
                                                                   split=8256, split_end=8261)),
                        "decode_lstm": (x0, wl, L.Epilogue(kind=L.EPI_LSTM, out_dtype=code, bias=bl.data_ptr(),
                                                           c=c.data_ptr(), h=h.data_ptr(), mask=mask.data_ptr(),
                                                           out=hout.data_ptr(), ldo=1280)),
                        "decode_proj_joint_in": (h.to(dt), wp, L.Epilogue(kind=L.EPI_JOINT_IN, out_dtype=code,
                                                                          bias=bp.data_ptr(), out=dec.data_ptr(),
                                                                          ldo=640, out2=zz.data_ptr(), ldo2=640,
                                                                          gather=enc.data_ptr(),
                                                                          gather_row=erow.data_ptr())),
                    }
                    for name, (a, w, ep) in cases.items():
                        for _ in range(3):
                            K.gemm(a, w, ep)
                        s = timed(lambda: K.gemm(a, w, ep), iters=50)
                        fl = 2 * lanes * w.shape[0] * w.shape[1]
                        emit(kernel=name, dtype=dt_name, lanes=lanes, us=s * 1e6, tflops=fl / s / 1e12,
                             weight_gbs=w.numel() * 2 / s / 1e9)
            if want("mhsa"):
                for t in map(int, filter(None, args.lengths.split(","))):
                    if t > bt and bt != min(map(int, args.rows.split(","))):
                        continue
                    clips = max(1, bt // t)
                    rows = clips * t
                    qu, qv, k, v = (rnd(rows, 1024, dt=dt) for _ in range(4))
                    rel = rnd(2 * t - 1, 1024, dt=dt)
                    rel_c = K.rel_bias(rel, rnd(1024), rnd(1024)) if code == L.BF16 else None
                    out = torch.empty(rows, 1024, device=dev, dtype=dt)
                    frames = K.Frames([t] * clips, code, dev)
                    s = timed(lambda: K.attention(qu, qv, k, v, rel, t, frames, out, rel_c), flush=flush)
                    fl = 6.0 * t * t * 1024 * clips
                    emit(kernel="relpos_attention", dtype=dt_name, rows=rows, T=t, clips=clips, us=s * 1e6,
                         tflops=fl / s / 1e12, frac=fl / s / 1e12 / tflops)
    K.check(dev)
    if want("decode_loop"):
        run_decode_loop(args, dev)
    if want("batch1"):
        run_batch1(args, dev)
    if "config0" in only:
        print(json.dumps({"kernel": "config0_fp32", **run_config0(args, *weights(args.layers))}), flush=True)
    if want("longform"):
        run_longform(args, dev, tflops)
    if want("load"):
        run_load(args, dev, hbm)
    if want("text"):
        run_text(args, dev)


def run_batch1(args, dev):
    """Batch 1: the bf16 encoder of one 10 s clip (the metric's "encoder ms per 10 s clip"),
    and config 0 (fp32, Bark.tokens of the 10 s seed-0 clip, cold and warm)."""
    import torch

    import tinybark_b200
    from tinybark_b200 import synthetic

    tensors, cfg = weights(args.layers)
    eng = tinybark_b200.load("gpu", dtype="bf16", weights=(tensors, cfg)).engine
    plan = eng.plan([1000])
    s1, o1 = eng.upload([synthetic.clip(10.0, 0)])
    f1 = eng.features(s1, o1, plan)
    for _ in range(3):
        eng.encode(f1, plan)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(20):
        eng.encode(f1, plan)
    b.record()
    torch.cuda.synchronize()
    eng.check()
    ms = a.elapsed_time(b) / 20
    print(json.dumps({"kernel": "encoder_batch1_bf16", "layers": args.layers, "T": 125, "ms": ms,
                      "weights_gbs": eng.layout.size / ms / 1e6}), flush=True)
    del eng
    print(json.dumps({"kernel": "config0_fp32", **run_config0(args, tensors, cfg)}), flush=True)


def run_decode_loop(args, dev):
    """The whole persistent greedy loop (2-layer model, bf16) for `--lanes` lanes whose
    lengths are those of clips of `--lane-seconds` (uniform; 2-30 s by default), on seeded
    N(0, 1) encoder frames (every lane then runs to its cap): milliseconds per loop, per
    iteration and per lane-iteration."""
    import torch

    from tinybark_b200 import lengths, synthetic
    from tinybark_b200 import weights as w
    from tinybark_b200.engine import Engine

    cfg = synthetic.config(2)
    eng = Engine(w.convert(synthetic.state_dict(0, layers=2), cfg), cfg, dtype="bf16", device=dev)
    for lanes in map(int, args.lanes.split(",")):
        lo, hi = map(float, args.lane_seconds.split(","))
        durs = np.sort(synthetic.durations(lanes, 4000 + lanes, lo, hi))[::-1]
        plan = eng.plan([lengths.frames(int(round(d * 16000))) for d in durs])
        enc = torch.randn(plan.batch.t3_total, 640, device=dev, generator=torch.Generator(device=dev).manual_seed(0))
        eng.decode(enc, plan)
        eng.check()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(2):
            eng.decode(enc, plan, early_exit=False)
        b.record()
        torch.cuda.synchronize()
        eng.check()
        ms = a.elapsed_time(b) / 2
        caps = plan.caps.cpu().numpy()
        print(json.dumps({"kernel": "decode_loop", "lanes": lanes, "ms": ms, "max_cap": int(caps.max()),
                          "lane_iterations": int(caps.sum()), "us_per_iteration": 1000 * ms / int(caps.max()),
                          "ns_per_lane_iteration": 1e6 * ms / int(caps.sum())}), flush=True)


def run_text(args, dev):
    """Transcripts as text for a batch of 512 lanes of 50-300 tokens (seeded ids of a seeded
    8193-id tokenizer): joined into bytes on the GPU (tb_text_offsets, tb_text_bytes, one
    copy back, one UTF-8 decode per lane), against the host path (token rows copied back,
    then the tokenizer's decode per lane). Best of 5 each, wall clock."""
    import tempfile

    import torch

    from tinybark_b200 import synthetic
    from tinybark_b200 import weights as w
    from tinybark_b200.engine import Engine
    from tinybark_b200.text import Tokenizer, finish

    cfg = synthetic.config(2)
    eng = Engine(w.convert(synthetic.state_dict(0, layers=2), cfg), cfg, dtype="bf16", device=dev)
    with tempfile.TemporaryDirectory() as d:
        tok = Tokenizer(synthetic.tokenizer(Path(d) / "tokenizer.json"))
    table = eng.text_table(*tok.table())
    rng = np.random.default_rng(0)
    lanes, ld = 512, 400
    counts = torch.from_numpy(rng.integers(50, 301, lanes).astype(np.int32)).to(dev)
    tokens = torch.from_numpy(rng.integers(3, 8192, (lanes, ld)).astype(np.int32)).to(dev)

    def gpu():
        return [finish(raw) for raw in eng.texts(tokens, counts, table)]

    def host():
        tk, cn = tokens.cpu().numpy(), counts.cpu().numpy()
        return [tok.decode(tk[j, : cn[j]].tolist()) for j in range(lanes)]

    assert gpu() == host()
    times = {}
    for name, fn in (("gpu_join_ms", gpu), ("host_decode_ms", host)):
        best = float("inf")
        for _ in range(5):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            best = min(best, time.perf_counter() - t0)
        times[name] = best * 1e3
    print(json.dumps({"kernel": "text_join", "lanes": lanes, "tokens": int(counts.sum()), **times}), flush=True)


def run_load(args, dev, hbm):
    """Weight loading, tinybark's every-start cost: the converted weights written as
    tinybark's fp16 cache file (1.25 GB at 24 layers), then that file to a ready bf16
    engine (data block read into pinned slices and copied to the GPU, one repack kernel,
    the decoder's input table, position tables up to 30 s), page cache warm from the
    write. Then the repack kernel on its own against the HBM roofline: algorithmic bytes =
    the f16 elements read plus the bf16 / f32 elements written."""
    import tempfile

    import torch

    from tinybark_b200 import _lib as L
    from tinybark_b200 import lengths, pack
    from tinybark_b200 import weights as w
    from tinybark_b200.engine import Engine

    tensors, cfg = weights(args.layers)
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "bark.safetensors"
        w.save(tensors, path)
        del tensors
        size = path.stat().st_size
        runs = []
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            eng = Engine(path, cfg, dtype="bf16", device=dev, max_len=lengths.subsampled(3000, 3))
            torch.cuda.synchronize()
            runs.append({"total_s": time.perf_counter() - t0, **{k + "_s": v for k, v in eng.load_seconds.items()}})
            del eng
        best = min(runs, key=lambda r: r["total_s"])
        print(json.dumps({"kernel": "load_cache_file", "layers": args.layers, "file_gb": size / 1e9,
                          "runs_s": [round(r["total_s"], 4) for r in runs], **{k: round(v, 4) for k, v in best.items()},
                          "read_copy_gbs": size / 1e9 / best["upload_s"]}), flush=True)
        src, index = pack.upload_cache(path, dev)
    lay = pack.model_layout(index, args.layers, L.BF16)
    out = torch.empty(lay.size, dtype=torch.uint8, device=dev)
    table = lay.table()
    jobs_dev = torch.empty(ctypes.sizeof(table), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def call():
        L.check(L.lib.tb_repack(table, len(lay.jobs), jobs_dev.data_ptr(), src.data_ptr(), src.numel(), out.data_ptr(),
                                out.numel(), stream), "tb_repack")

    for _ in range(3):
        call()
    s = timed(call, iters=10)
    moved = sum(int(np.prod(j[3])) * ((0 if j[6] else (2 if j[4] == L.SRC_F16 else 4)) + (2 if j[5] == L.BF16 else 4))
                for j in lay.jobs)
    print(json.dumps({"kernel": "repack_kernel", "layers": args.layers, "jobs": len(lay.jobs), "bytes": moved,
                      "us": s * 1e6, "gbs": moved / s / 1e9, "frac": moved / s / 1e9 / hbm}), flush=True)


def run_longform(args, dev, tflops):
    """The long-form workload: one 10-minute clip (f0 redrawn every 2 s, T = 7500 encoder
    frames) through front-end, encoder with full-context attention, and decode, bf16."""
    import torch

    import tinybark_b200
    from tinybark_b200 import synthetic

    seconds = 600.0
    clip = synthetic.to_float(synthetic.clip(seconds, 3, segment=2.0))
    tensors, cfg = weights(args.layers)
    bark = tinybark_b200.load("gpu", dtype="bf16", weights=(tensors, cfg))
    eng = bark.engine
    plan = eng.plan([len(clip) // 160])
    eng.ensure_len(int(plan.t3.max()))
    samples, off = eng.upload([clip])
    split = {}
    for _ in range(3):
        split = stage_split(eng, samples, off, plan)
    eng.check()
    T = int(plan.t3[0])
    enc_flop = args.layers * (48.2e6 * T + 6.0 * T * T * 1024)
    total = sum(split.values())
    print(json.dumps({"kernel": "longform_10min", "dtype": "bf16", "audio_s": seconds, "T": T, "layers": args.layers,
                      "stages_ms": split, "rtfx": seconds / (total / 1000), "encoder_tflops": enc_flop / split["encoder"] / 1e9,
                      "encoder_frac": enc_flop / split["encoder"] / 1e9 / tflops}), flush=True)
    # The same recording in pieces of at most 30 s (Bark.tokens_long), end to end from the
    # host array: front-end, encoder and decode of all pieces as one batch.
    from tinybark_b200 import longform

    cuts = longform.cut_points(clip)
    for _ in range(2):
        bark.tokens_long(clip)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        bark.tokens_long(clip)
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1000 / reps
    print(json.dumps({"kernel": "longform_10min_pieces", "dtype": "bf16", "audio_s": seconds, "pieces": len(cuts) - 1,
                      "layers": args.layers, "e2e_ms": ms, "rtfx": seconds / (ms / 1000)}), flush=True)


def stage_split(eng, samples, sample_off, plan, groups=None):
    """Milliseconds of front-end, encoder and decode in one untimed extra step."""
    import torch

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record()
    feats = eng.features(samples, sample_off, plan)
    ev[1].record()
    enc = eng.encode(feats, plan)
    ev[2].record()
    eng.decode(enc, plan, groups=groups)
    ev[3].record()
    torch.cuda.synchronize()
    return {k: ev[i].elapsed_time(ev[i + 1]) for i, k in enumerate(("frontend", "encoder", "decode"))}


def run_profile(args):
    """One pipeline step on this rank's shard after one warm-up step: for ncu."""
    import torch

    import tinybark_b200

    torch.cuda.set_device(0)
    from tinybark_b200.engine import lane_order

    groups = args.decode_groups or None
    clips, durs = shard(0, 1, args.clips)
    order = lane_order(list(range(len(clips))), [len(c) // 160 for c in clips], groups)
    clips, durs = [clips[i] for i in order], durs[order]
    tensors, cfg = weights(args.layers)
    bark = tinybark_b200.load("gpu", dtype="bf16", weights=(tensors, cfg))
    eng = bark.engine
    plan = eng.plan([len(c) // 160 for c in clips])
    samples, sample_off = eng.upload(clips)
    for _ in range(args.steps):
        split = stage_split(eng, samples, sample_off, plan, groups)
    eng.check()
    print(json.dumps({"profile_step_ms": split, "clips": len(clips), "audio_s": float(np.sum(durs))}), flush=True)


def main():
    args = args_parser().parse_args()
    if args.micro:
        run_micro(args)
    elif args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
