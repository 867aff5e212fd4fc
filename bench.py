"""Throughput bench of the Kokoro-82M decoder hot path on B200.

Workload: 256 independent utterances, T ~ U[40, 800] asr frames (1-20 s of
24 kHz audio), decoder weights F16 random-init seed 2, inputs seeded per
utterance; each GPU runs batches of 64 utterances (one step = decoder encode/
decode + ISTFTNet generator + iSTFT over one batch). Synthetic data: no
checkpoint or dataset exists offline.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Multi-GPU: one process per GPU (torchrun), utterances sharded by
kokopop_b200.shard, no collective on the data path; the timed region is
bracketed by barriers and the max over ranks is reported.
Prints one JSON line on rank 0.
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
sys.path.insert(0, ROOT)

METRIC = "audio-sec/s per B200 (Kokoro-82M decoder, batch 64)"
UNIT = "audio-s/s"
POOL = 256
BATCH = 64
FLOP_PER_AUDIO_S = None  # filled from the model dimensions below
# DRAM bytes of all tensor-core conv launches per audio second, from one ncu
# capture of the batch-8 step (dram__bytes_read.sum + dram__bytes_write.sum of
# one forward); traffic grows with the rows processed.
CONV_DRAM_BYTES_PER_AUDIO_S = 1.483e8
# DRAM bytes measured by ncu per algorithmic byte for the tensor-bound
# convolutions (per-shape captures of single launches); None until measured.
CONV_TENSOR_DRAM_PER_ALGO_BYTE = None


def algorithmic_flop_per_asr_frame() -> float:
    """2 x MACs of the dense convolutions per asr frame T (linear in T):
    decoder (k=3 convs, 1x1 shortcuts, asr_res) + generator (noise convs,
    ups, 4 resblocks per stage, conv_post)."""
    mac = 0.0
    # decoder, per T frame
    mac += 512 * 64                                   # asr_res
    mac += 514 * 1024 * 3 + 1024 * 1024 * 3 + 514 * 1024  # encode
    mac += 3 * (1090 * 1024 * 3 + 1024 * 1024 * 3 + 1090 * 1024)  # decode.0-2
    mac += 2 * (1090 * 512 * 3 + 512 * 512 * 3) + 1090 * 512      # decode.3 (2T) + shortcut at T
    # generator stage 0 (20 rows per T, 256 ch) and stage 1 (120 rows, 128 ch)
    mac += 20 * 256 * 22 * 12                          # noise_convs.0
    mac += 2 * 512 * 256 * 20                          # ups.0: 2 input rows per T, K=20 taps
    mac += 20 * 6 * 256 * 256 * (7 + 3 + 7 + 11)       # noise_res.0 (k7) + resblocks 3/7/11: 6 convs each
    mac += 120 * 128 * 22 * 1                          # noise_convs.1
    mac += 20 * 256 * 128 * 12                         # ups.1: per input row (20 per T) K=12 taps
    mac += 120 * 6 * 128 * 128 * (11 + 3 + 7 + 11)     # noise_res.1 (k11) + resblocks
    mac += 120 * 128 * 22 * 7                          # conv_post
    return 2.0 * mac


def roofline_classes(records, steps, step_ms, pk, pk_kind):
    """Groups the timed launches of the timed region (kk_profile_records) by
    class and sets each class against its roofline: convolutions whose
    arithmetic intensity (algorithmic FLOP per algorithmic DRAM byte) reaches
    the ridge point of the measured peaks are tensor-bound (TFLOP/s against
    the sustained dense bf16 peak), the others HBM-bound (GB/s against the
    measured copy bandwidth), like every memory pass. The LSTM recurrence is
    bound by its sequential steps, not by a pipe. Per step: launches, device
    ms and its share of the step (the source runs on a side stream,
    overlapped with the decoder)."""
    hbm = float(pk["hbm_gbs"])
    tf = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    ridge = tf * 1e12 / (hbm * 1e9)
    names = {"operand": "operand pass (AdaIN + Snake / LeakyReLU -> half operand)",
             "stats": "instance-norm statistics pass", "istft": "conv_post -> iSTFT",
             "source": "harmonic source + STFT (side stream)", "lstm": "LSTM recurrence",
             "other": "packing, upsampling, ConvTranspose edge row",
             "conv_tensor": "dense conv, tensor-bound (k >= 7 and the 1024-channel decoder convs)",
             "conv_hbm": "dense conv, HBM-bound (k = 3 at 128 / 256 channels, 1x1, ConvTranspose phases)"}
    agg = {}
    for r in records:
        k = r["kind"]
        if k == "conv":
            k = "conv_tensor" if r["bytes"] > 0 and r["flop"] / r["bytes"] >= ridge else "conv_hbm"
        a = agg.setdefault(k, {"launches": 0, "ms": 0.0, "flop": 0.0, "bytes": 0.0})
        a["launches"] += 1
        a["ms"] += r["ms"]
        a["flop"] += r["flop"]
        a["bytes"] += r["bytes"]
    out = {}
    for k, a in agg.items():
        s = a["ms"] / 1e3
        c = {"what": names.get(k, k), "launches_per_step": a["launches"] / steps, "ms_per_step": a["ms"] / steps,
             "share_of_step": (a["ms"] / steps) / step_ms if step_ms else None}
        if k == "conv_tensor":
            c.update(bound="tensor", achieved=a["flop"] / s / 1e12 if s else None, peak=tf, unit="TFLOP/s")
        elif k == "lstm":
            c.update(bound="latency (sequential steps)", achieved=a["flop"] / s / 1e12 if s else None,
                     peak=None, unit="TFLOP/s")
        else:
            c.update(bound="hbm", achieved=a["bytes"] / s / 1e9 if s else None, peak=hbm, unit="GB/s")
        c["frac"] = c["achieved"] / c["peak"] if c.get("peak") and c.get("achieved") is not None else None
        c["algorithmic_flop_per_step"] = a["flop"] / steps
        c["algorithmic_bytes_per_step"] = a["bytes"] / steps
        out[k] = c
    out["ridge_flop_per_byte"] = ridge
    out["peak_source"] = f"{pk_kind}: copy {hbm:.0f} GB/s, bf16 dense sustained {tf:.0f} TFLOP/s"
    return out


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region.

    nvidia-smi takes a while to print its first sample, and the timed region
    lasts well under a second, so the sampler starts before the warm-up,
    waits for its first sample, samples every 50 ms, and keeps the samples
    whose timestamps fall inside the timed region (mark() brackets it)."""

    FIELDS = ("timestamp,index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path):
        self.path = path
        self.proc = None
        self.window = None

    def start(self, wait_s=5.0):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                          "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t_end = time.time() + wait_s
        while time.time() < t_end and os.path.getsize(self.path) == 0 and self.proc.poll() is None:
            time.sleep(0.02)

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self, uuid=None):
        import datetime
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 11:
                continue
            if uuid and parts[2] != uuid:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[3].split()[0]), float(parts[4].split()[0]), parts[7:11]))
            except ValueError:
                continue
        if self.window is not None:
            t0, t1 = self.window
            inside = [r for r in rows if t0 <= r[0] <= t1]
            # a region shorter than the sampling period: the samples around it
            rows = inside or [r for r in rows if t0 - 0.1 <= r[0] <= t1 + 0.1]
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in rows for n, v in zip(names, r[3]) if v.lower() == "active"}
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": rows[-1][2],
                "reasons": sorted(reasons), "samples": len(rows)}


def make_pool():
    from kokopop_b200 import workload as W
    return W.config3_utterances(POOL)


def cpu_sample(pool, max_T=240, n=3):
    """A bounded sample of the workload for the CPU baselines: the first n
    pool utterances with T <= max_T (seconds of CPU work, not minutes)."""
    return [u for u in pool if u.T <= max_T][:n]


def run_cpu_oracle(weights, utts):
    """Times the oracle (the CPU restatement of the reference's path) on
    utts; returns (audio seconds, wall seconds, threads)."""
    from oracle import oracle as O
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    m = O.OracleModel(weights)
    t0 = time.perf_counter()
    secs = 0.0
    for u in utts:
        m.decoder_forward(u.asr, u.f0, u.noise, u.style)
        secs += u.T / 40.0
    return secs, time.perf_counter() - t0, threads


def reference_arm(args):
    """--impl reference: the reference's CPU path for this workload on the
    host cores. The reference's generator needs ggml (fetched from the network
    at configure time, absent here), so this is the oracle port of it; its
    iSTFT and LSTM restatements are bit-exact with the reference's own compiled
    istft.cpp / lstm_fused.cpp (tests/test_oracle.py)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    from kokopop_b200 import workload as W
    pool = make_pool()
    sample = [u for u in pool if u.T <= 240]
    weights = W.config2_weights()
    from oracle import oracle as O
    m = O.OracleModel(weights)
    threads = int(os.environ["OMP_NUM_THREADS"])
    secs_tot, wall_tot = 0.0, 0.0
    for k in range(args.warmup + args.steps):
        u = sample[k % len(sample)]
        t0 = time.perf_counter()
        m.decoder_forward(u.asr, u.f0, u.noise, u.style)
        dt = time.perf_counter() - t0
        if k >= args.warmup:
            secs_tot += u.T / 40.0
            wall_tot += dt
    value = secs_tot / wall_tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall_tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config_dict(),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "one utterance per step, cycling over the pool's utterances with T<=240 asr "
                                   "frames (not the pool's U[40,800] length mix); the oracle port of the "
                                   "reference's ggml CPU path (C, -O3 without -march: scalar, no SIMD, like the "
                                   "reference's own flags), OpenMP over output channels"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def parity_vs_c_library(kb, W, device, pool):
    """The device waveform against the oracle in its two modes for the
    harmonic source's sin / cos / tanh / atan2: correctly rounded (what the
    kernels compute) and the C library's float functions (what the
    reference's compiled fill_harmonic_stft calls; the oracle's C-library
    mode equals it bit for bit). Cases: config 0 (T = 200, F32 weights seed
    0) and the pool's first utterance with T <= 240 (F16 weights seed 2).
    The two oracle modes differ from each other by about as much as the
    device differs from the C-library mode: near-silent STFT bins feed atan2,
    whose branch flips with the last bit of the source."""
    from oracle import oracle as O
    out = {"cases": []}
    u3 = next(u for u in pool if u.T <= 240)
    for name, w, u in (("config 0: T=200, F32 weights seed 0", W.config0_weights(), W.config0_inputs(200)),
                       (f"pool utterance T={u3.T}, F16 weights seed 2", W.config2_weights(), u3)):
        c = kb.Context(device)
        c.upload(w)
        got = c.decoder_forward([u])[0]
        c.close()
        m = O.OracleModel(w)
        cr = m.decoder_forward(u.asr, u.f0, u.noise, u.style)
        m.set_source_libm(True)
        lm = m.decoder_forward(u.asr, u.f0, u.noise, u.style)
        out["cases"].append({
            "case": name,
            "max_abs_vs_oracle_correctly_rounded": float(np.abs(got - cr).max()),
            "max_abs_vs_oracle_c_library": float(np.abs(got - lm).max()),
            "mean_abs_vs_oracle_c_library": float(np.abs(got - lm).mean()),
            "oracle_modes_max_abs": float(np.abs(cr - lm).max()),
        })
    return out


def bench_lstm(kb, W, device, runs):
    """The prosody duration encoder (3 x biLSTM 640 -> 2x256 + AdaLayerNorm),
    seed-1 weights U(-1/16, 1/16), inputs N(0, 1), device-resident, timed with
    CUDA events on the launch stream: ms per call, us per sequential step
    (3 layers x L steps), tokens/s, and the W_ih projection's TFLOP/s."""
    import torch
    cases = [(32, 512, False), (1, 512, False), (32, 512, True)]
    out = {"workload": "duration encoder: 3 x (biLSTM 640 -> 2x256, AdaLayerNorm 512), seed 1 U(-1/16,1/16)",
           "cases": []}
    stream = torch.cuda.Stream()
    for B, L, f16 in cases:
        c = kb.Context(device)
        c.upload(W.config1_weights(f16=f16))
        g = torch.Generator(device="cuda").manual_seed(101)
        x = torch.randn(B * L, 512, device="cuda", generator=g)
        st = torch.randn(B, 128, device="cuda", generator=g)
        o = torch.empty(B * L, 640, device="cuda")
        lens = np.full(B, L, np.int32)
        call = lambda: c.duration_encoder_device(lens, x.data_ptr(), st.data_ptr(), o.data_ptr(), stream.cuda_stream)
        for _ in range(2):
            call()
        torch.cuda.synchronize()
        c.profile_read(reset=True)
        c.profile_enable(True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(runs):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        c.profile_enable(False)
        prof = c.profile_read(reset=True)
        ms = e0.elapsed_time(e1) / runs
        gemm_tf = prof["conv_flop"] / (prof["conv_ms"] / 1e3) / 1e12 if prof["conv_ms"] > 0 else None
        out["cases"].append({
            "batch": B, "steps": L, "weights": "f16" if f16 else "f32",
            "wih_path": "tcgen05 f16" if f16 else "tcgen05 split f32 (hi + lo halves, 3 products)",
            "ms_per_call": ms, "us_per_step": 1e3 * ms / (3 * L), "tokens_per_s": B * L / (ms / 1e3),
            "wih_gemm_tflops": gemm_tf, "wih_share": (prof["conv_ms"] / runs) / ms if ms > 0 else None,
        })
        c.close()
    return out


def bench_prosody(kb, W, device, runs, pool, batch):
    """The prosody predictor's F0 / N chain (biLSTM 640 -> 2x256, then per
    branch 3 x AdainResBlk1d and the 1x1 projection) over one batch of the
    pool's lengths as aligned frames, seed-2 F16 weights (config 2's draw),
    inputs N(0, 1) / style N(0, 0.1), device-resident, timed with CUDA
    events on the launch stream: ms per call and frames/s."""
    import torch
    lens = np.array([u.T for u in pool[:batch]], np.int32)
    c = kb.Context(device)
    c.upload(W.prosody_weights(f16=True))
    g = torch.Generator(device="cuda").manual_seed(102)
    rows = int(lens.sum())
    en = torch.randn(rows, 640, device="cuda", generator=g)
    st = 0.1 * torch.randn(len(lens), 128, device="cuda", generator=g)
    f0 = torch.empty(2 * rows, device="cuda")
    nn = torch.empty(2 * rows, device="cuda")
    stream = torch.cuda.Stream()
    call = lambda: c.prosody_f0n_device(lens, en.data_ptr(), st.data_ptr(), f0.data_ptr(), nn.data_ptr(),
                                        stream.cuda_stream)
    for _ in range(2):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(runs):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / runs
    c.close()
    return {"workload": f"prosody F0/N chain: biLSTM 640->2x256 + 2 x (3 AdainResBlk1d + 1x1 proj), "
                        f"batch {len(lens)} utterances T~U[40,800] frames, F16 weights seed 2",
            "frames": rows, "ms_per_call": ms, "frames_per_s": rows / (ms / 1e3),
            "audio_s_per_s": rows / 40.0 / (ms / 1e3)}


def bench_vocos(kb, W, device, runs, batch=64):
    """The sanoTTS Vocos decoder: `batch` chunks of 10 s (938 frames at hop
    256), F32 weights seed 3 at the stand-in dimensions of
    workload.VOCOS_DIMS, inputs N(0, 1), device-resident, timed with CUDA
    events on the launch stream (the median of `runs` calls): ms per call,
    audio-s/s, and the tensor-core linears' TFLOP/s from the profile
    records of one call."""
    import statistics
    import torch
    d = W.VOCOS_DIMS
    frames = 938
    c = kb.Context(device)
    c.upload(W.vocos_weights(f16=False))
    g = torch.Generator(device="cuda").manual_seed(104)
    lens = np.full(batch, frames, np.int32)
    mel = torch.randn(batch * d["mels"] * frames, device="cuda", generator=g)
    noise = torch.randn(batch * d["noise_ch"] * frames, device="cuda", generator=g)
    out = torch.empty(batch * d["hop"] * (frames - 1), device="cuda")
    stream = torch.cuda.Stream()
    call = lambda: c.vocos_forward_device(W.VOCOS_PREFIX, d, lens, mel.data_ptr(), noise.data_ptr(), out.data_ptr(),
                                          stream.cuda_stream)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    ts = []
    for _ in range(runs):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call()
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    c.profile_read(reset=True)
    c.profile_enable(True)
    call()
    torch.cuda.synchronize()
    c.profile_enable(False)
    recs = c.profile_records()
    c.profile_read(reset=True)
    c.close()
    ms = statistics.median(ts)
    secs = batch * d["hop"] * (frames - 1) / 24000.0
    kinds = {}
    for r in recs:
        k = kinds.setdefault(r["kind"], {"ms": 0.0, "flop": 0.0, "bytes": 0.0, "launches": 0})
        k["ms"] += r["ms"]
        k["flop"] += r["flop"]
        k["bytes"] += r["bytes"]
        k["launches"] += 1
    conv = kinds.get("conv", {"ms": 0.0, "flop": 0.0})
    return {"workload": f"sanoTTS Vocos decoder, {batch} chunks of {frames} frames (10 s each), F32 weights seed 3, "
                        f"dims {d} (stand-ins: the heart voice's are not available)",
            "ms_per_call": ms, "audio_s_per_s": secs / (ms / 1e3),
            "linears_tflops": conv["flop"] / (conv["ms"] / 1e3) / 1e12 if conv["ms"] else None,
            "ms_by_kind": {k: round(v["ms"], 4) for k, v in kinds.items()}}


def bench_frontend(kb, W, device, runs):
    """Config 2's front end for one utterance of 128 phoneme ids (130 with the
    pads), F16 weights seed 2, device-resident, each stage timed with CUDA
    events on the launch stream: ALBERT + bert_encoder, the duration encoder,
    the duration head (predictor biLSTM + projection), the text encoder; ms
    per call (median of `runs`)."""
    import statistics
    import torch
    c = kb.Context(device)
    c.upload(W.config2_frontend_weights())
    ids = W.token_ids(np.random.default_rng(7), 128)
    lens = np.array([len(ids)], np.int32)
    n = int(lens[0])
    g = torch.Generator(device="cuda").manual_seed(103)
    d_ids = torch.from_numpy(ids).cuda()
    style = 0.1 * torch.randn(1, 128, device="cuda", generator=g)
    bert = torch.empty(n, 512, device="cuda")
    d = torch.empty(n, 640, device="cuda")
    dur = torch.empty(n, device="cuda")
    ten = torch.empty(n, 512, device="cuda")
    stream = torch.cuda.Stream()
    stages = {
        "albert_ms": lambda: c.albert_device(lens, d_ids.data_ptr(), bert.data_ptr(), stream.cuda_stream),
        "duration_encoder_ms": lambda: c.duration_encoder_device(lens, bert.data_ptr(), style.data_ptr(),
                                                                 d.data_ptr(), stream.cuda_stream),
        "duration_head_ms": lambda: c.duration_head_device(lens, d.data_ptr(), dur.data_ptr(), stream.cuda_stream),
        "text_encoder_ms": lambda: c.text_encoder_device(lens, d_ids.data_ptr(), ten.data_ptr(), stream.cuda_stream),
    }
    for f in stages.values():
        f()
        f()
    torch.cuda.synchronize()
    out = {"workload": "config-2 front end, one utterance of 128 phoneme ids + 2 pads, F16 weights seed 2",
           "tokens": n}
    total = 0.0
    for k, f in stages.items():
        ts = []
        for _ in range(runs):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            f()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        out[k] = statistics.median(ts)
        total += out[k]
    out["total_ms"] = total
    c.close()
    return out


def bench_queue(kb, device, weights, pool, batch):
    """The rank's pool through the batching queue (one worker on a second
    context of this GPU, max_batch = the bench batch, 2 ms batching wait): all
    chunks submitted at once from the host, wall time until the last result is
    in host memory (the second of two passes); audio-s/s and the batches
    formed over both passes. The output buffers are the caller's, allocated
    and touched once before both passes (as a C caller of kk_queue_submit
    passes its own)."""
    ctx = kb.Context(device)
    ctx.upload(weights)
    q = kb.Queue(contexts=[ctx], max_batch=batch, max_batch_frames=batch * 800, max_wait_us=2000)
    outs = [np.zeros(600 * int(u.T), np.float32) for u in pool]
    for o in outs:
        o.fill(0.0)
    try:
        for timed in (False, True):  # one untimed pass: workspace and staging allocated
            t0 = time.perf_counter()
            tickets = [q.submit(i, u, outs[i]) for i, u in enumerate(pool)]
            for t in tickets:
                rc, _ = q.wait(t, 600000)
                if rc != 0:
                    raise RuntimeError(f"queue result {rc}")
            wall = time.perf_counter() - t0
        st = q.stats()
    finally:
        q.close()
        ctx.close()
    secs = sum(u.T for u in pool) / 40.0
    return {"workload": f"{len(pool)} utterances of the pool submitted at once, one worker, max batch {batch}",
            "value": secs / wall, "unit": UNIT, "wall_s": wall, "batches": st["batches"], "max_batch": st["max_batch"]}


def bench_stream(kb, W, device, weights, runs):
    """First audio through a streaming session (kk_stream over a one-worker
    GPU queue, adaptative preset): a request of four chunks (T = 40, 120,
    120, 120 asr frames: a short first chunk, as the reference's adaptative
    chunker makes it) pushed at once on an idle GPU; wall time from the
    push to the first post-processed chunk in host memory (kk_stream_next),
    and to the last. p50 over `runs` requests after two untimed ones."""
    ctx = kb.Context(device)
    ctx.upload(weights)
    q = kb.Queue(contexts=[ctx], max_batch=8, max_batch_frames=8 * 800, max_wait_us=0)
    rng = np.random.default_rng(77)
    chunks = [W.make_utterance(rng, t) for t in (40, 120, 120, 120)]
    first, total = [], []
    try:
        for r in range(runs + 2):
            s = kb.Stream(q, kb.StreamConfig.preset(0))
            t0 = time.perf_counter()
            for i, u in enumerate(chunks):
                s.push(u, kb.BOUNDARY_CLAUSE_WEAK, i == len(chunks) - 1)
            t_first = None
            while True:
                rc, _, _ = s.next(60000)
                if rc == kb.STREAM_END:
                    break
                if rc != 0:
                    raise RuntimeError(f"stream result {rc}")
                if t_first is None:
                    t_first = time.perf_counter() - t0
            t_all = time.perf_counter() - t0
            s.close()
            if r >= 2:
                first.append(1e3 * t_first)
                total.append(1e3 * t_all)
    finally:
        q.close()
        ctx.close()
    return {"workload": "one request of 4 chunks (T = 40, 120, 120, 120), idle GPU, adaptative preset",
            "ttfa_p50_ms": statistics.median(first), "all_chunks_p50_ms": statistics.median(total),
            "runs": runs, "audio_s": sum(u.T for u in chunks) / 40.0}


def config_dict(batch=BATCH):
    return {
        "workload": "Kokoro-82M decoder (AdainResBlk1d encode/decode) + ISTFTNet generator + iSTFT; "
                    f"256 utterances T~U[40,800] asr frames, F16 weights seed 2, batch {batch} per GPU",
        "batch_per_gpu": batch, "pool": POOL, "weights": "F16 (converter policy), N(0,0.02), seed 2",
        "l2": "no flush: per-step working set (activations ~15 GB) is >100x the 126 MB L2",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the device-vs-C-library-mode parity key")
    ap.add_argument("--ttfa-runs", type=int, default=50, help="0 skips the TTFA measurement")
    ap.add_argument("--batch", type=int, default=BATCH, help="utterances per GPU step (profiling cases)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling cases)")
    ap.add_argument("--lstm-runs", type=int, default=5, help="timed calls per LSTM-stack case (0 skips)")
    ap.add_argument("--prosody-runs", type=int, default=3, help="timed calls of the prosody F0/N chain (0 skips)")
    ap.add_argument("--frontend-runs", type=int, default=5, help="timed calls per front-end stage (0 skips)")
    ap.add_argument("--vocos-runs", type=int, default=5, help="timed calls of the Vocos decoder (0 skips)")
    ap.add_argument("--no-queue", action="store_true", help="skip the batching-queue leg")
    ap.add_argument("--stream-runs", type=int, default=20, help="timed requests of the streaming-session leg (0 skips)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist
    import kokopop_b200 as kb
    from kokopop_b200 import workload as W
    from kokopop_b200.shard import rank_batches

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    pool = make_pool()
    weights = W.config2_weights()
    ctx = kb.Context(local)
    ctx.upload(weights)
    batches = rank_batches(POOL, rank, world, args.batch)
    dev = []
    host = []
    for idx in batches:
        utts = [pool[i] for i in idx]
        n_frames, asr, f0, noise, style = W.pack(utts)
        t = lambda a: torch.from_numpy(a).cuda()
        d = {"n": n_frames, "asr": t(asr), "f0": t(f0), "noise": t(noise), "style": t(style),
             "audio": torch.empty(600 * int(n_frames.sum()), dtype=torch.float32, device="cuda")}
        dev.append(d)
        p = lambda a: torch.from_numpy(a).pin_memory()
        host.append({"n": n_frames, "asr": p(asr), "f0": p(f0), "noise": p(noise), "style": p(style),
                     "audio": torch.empty(600 * int(n_frames.sum()), dtype=torch.float32).pin_memory()})

    # A dedicated stream: the C ABI runs the path on the stream it is given,
    # and the CUDA events below are recorded on that same stream.
    stream = torch.cuda.Stream()

    def step_device(k):
        d = dev[k % len(dev)]
        ctx.decoder_forward_device(d["n"], d["asr"].data_ptr(), d["f0"].data_ptr(), d["noise"].data_ptr(),
                                   d["style"].data_ptr(), d["audio"].data_ptr(), stream.cuda_stream)
        return float(d["n"].sum()) / 40.0

    import ctypes

    def step_host(k):
        h = host[k % len(host)]
        f = ctypes.POINTER(ctypes.c_float)
        cast = lambda tt: ctypes.cast(tt.data_ptr(), f)
        rc = ctx.L.kk_decoder_forward(ctx.h, len(h["n"]), h["n"].ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                      cast(h["asr"]), cast(h["f0"]), cast(h["noise"]), cast(h["style"]),
                                      cast(h["audio"]))
        ctx._check(rc)
        return float(h["n"].sum()) / 40.0

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # Setup: one untimed pass over every batch of this rank through both
    # entry points, so the context's workspaces (grown on first sight of a
    # larger batch) reach their final sizes before any warm-up or timing.
    for k in range(len(dev)):
        step_device(k)
    torch.cuda.synchronize()
    if not args.no_e2e:
        for k in range(len(host)):
            step_host(k)

    # ---- device-resident throughput (value) ----
    clocks = ClockSampler(os.path.join("/tmp", f"kk_clocks_{rank}.csv"))
    if rank == 0:
        clocks.start()
    for k in range(args.warmup):
        step_device(k)
    torch.cuda.synchronize()
    ctx.profile_read(reset=True)
    ctx.profile_enable(True)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    tw0 = time.time()
    ev0.record(stream)
    secs = 0.0
    th0 = time.perf_counter()
    for k in range(args.steps):
        secs += step_device(args.warmup + k)
    host_enqueue_ms = (time.perf_counter() - th0) * 1e3 / max(1, args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(tw0, time.time())
    barrier()
    elapsed = ev0.elapsed_time(ev1) / 1e3
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        if not uuid.startswith("GPU-"):
            uuid = "GPU-" + uuid
    except Exception:
        uuid = None
    clk = clocks.stop(uuid) if rank == 0 else None
    ctx.profile_enable(False)
    records = ctx.profile_records()
    prof = ctx.profile_read(reset=True)
    t_max = max_over_ranks(elapsed)
    secs_all = sum_over_ranks(secs)
    value = secs_all / t_max

    # Host cost of enqueueing, from an idle GPU: two device-buffer steps in a
    # row. A call that waited for the stream would take a whole step here
    # (the loop above also includes the launch queue's back-pressure once
    # the host runs a few steps ahead).
    torch.cuda.synchronize()
    th0 = time.perf_counter()
    step_device(0)
    step_device(1)
    enqueue_idle_ms = (time.perf_counter() - th0) * 1e3 / 2
    torch.cuda.synchronize()

    # ---- end to end through the host-buffer C ABI (pinned host memory) ----
    e2e_value = None
    if not args.no_e2e:
        for k in range(min(args.warmup, 2)):
            step_host(k)
        barrier()
        t0 = time.perf_counter()
        e2e_secs = 0.0
        e2e_steps_ms = []
        for k in range(args.steps):
            ts = time.perf_counter()
            e2e_secs += step_host(k)
            e2e_steps_ms.append(round((time.perf_counter() - ts) * 1e3, 2))
        e2e_t = time.perf_counter() - t0
        barrier()
        e2e_value = sum_over_ranks(e2e_secs) / max_over_ranks(e2e_t)
    tot_frames = [int(h["n"].sum()) for h in host]
    h2d = statistics.mean([(512 + 2 + 2) * 4 * f + 4 * 128 * args.batch + 4 * args.batch for f in tot_frames])
    d2h = statistics.mean([600 * 4 * f for f in tot_frames])

    ttfa = None
    cpu = None
    parity = None
    # The single-GPU legs below (TTFA, LSTM stack, prosody, queue, stream,
    # front end, Vocos) run at N = 1 only: at N > 1 the other ranks have left
    # by then while this rank's NCCL communicator lives on, which slowed the
    # host-driven legs (the queue leg measured 457 audio-s/s at N = 2 against
    # 8066 at N = 1), and their single-GPU figures are those of the N = 1 run.
    single = rank == 0 and world == 1
    if single and args.ttfa_runs > 0:
        # p50 time to first audio: one config-0 utterance (T=200, F32 weights
        # seed 0), submitted alone on an idle GPU, until its samples are in
        # host memory; the whole utterance is returned in one piece.
        c0 = kb.Context(local)
        c0.upload(W.config0_weights())
        u = W.config0_inputs(200)
        for _ in range(3):
            c0.decoder_forward([u])
        lat = []
        for _ in range(args.ttfa_runs):
            t = time.perf_counter()
            c0.decoder_forward([u])
            lat.append(time.perf_counter() - t)
        ttfa = 1e3 * statistics.median(lat)
        c0.close()
    def leg(name, fn, *a):
        # an NVTX range per leg, so that a profiler can select one leg's
        # launches (ncu --nvtx --nvtx-include "<name>/")
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*a)
        finally:
            torch.cuda.nvtx.range_pop()

    lstm = None
    if single and args.lstm_runs > 0:
        lstm = leg("lstm", bench_lstm, kb, W, local, args.lstm_runs)
    prosody = None
    if single and args.prosody_runs > 0:
        prosody = leg("prosody", bench_prosody, kb, W, local, args.prosody_runs, pool, args.batch)
    queue = None
    if single and not args.no_queue:
        queue = leg("queue", bench_queue, kb, local, weights, [pool[i] for idx in batches for i in idx], args.batch)
    stream = None
    if single and args.stream_runs > 0:
        stream = leg("stream", bench_stream, kb, W, local, weights, args.stream_runs)
    frontend = None
    if single and args.frontend_runs > 0:
        frontend = leg("frontend", bench_frontend, kb, W, local, args.frontend_runs)
    vocos = None
    if single and args.vocos_runs > 0:
        vocos = leg("vocos", bench_vocos, kb, W, local, args.vocos_runs)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            sample = cpu_sample(pool)
            s_audio, s_wall, thr = run_cpu_oracle(weights, sample)
            cpu = {"value": s_audio / s_wall, "unit": UNIT, "cores": thr, "kind": "port",
                   "sample": f"the first {len(sample)} pool utterances with T<=240 ({s_audio:.1f} s of audio; not "
                             f"the pool's U[40,800] length mix); the oracle port of the reference's ggml CPU path "
                             f"(C, -O3 without -march: scalar, no SIMD, like the reference's own flags), OpenMP "
                             f"over output channels"}
        if world == 1 and not args.no_parity:
            parity = parity_vs_c_library(kb, W, local, pool)

    pk, pk_kind = peaks()
    achieved_all = prof["conv_flop"] / (prof["conv_ms"] / 1e3) / 1e12 if prof["conv_ms"] > 0 else 0.0
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    classes = roofline_classes(records, args.steps, 1e3 * elapsed / args.steps, pk, pk_kind)
    ct = classes.get("conv_tensor", {})
    ct_launches = ct.get("launches_per_step") or 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config_dict(args.batch),
        "e2e": ({"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                 "step_ms": e2e_steps_ms}
                if e2e_value is not None else None),
        # the dominant kernel class: the tensor-bound convolutions (CUDA
        # events around each launch in the timed region); per launch
        "roofline": {"bound": "tensor", "kernel": "k_conv_tct / k_conv_tc launches at or above the ridge point",
                     "achieved": ct.get("achieved"), "peak": peak, "unit": "TFLOP/s", "frac": ct.get("frac"),
                     "traffic": (CONV_TENSOR_DRAM_PER_ALGO_BYTE * ct["algorithmic_bytes_per_step"] / ct_launches
                                 if ct_launches and CONV_TENSOR_DRAM_PER_ALGO_BYTE else None),
                     "traffic_unit": "DRAM bytes per launch (ncu per-shape captures: measured / algorithmic bytes, "
                                     "applied to this class's algorithmic bytes)",
                     "algorithmic_bytes_per_launch": (ct["algorithmic_bytes_per_step"] / ct_launches
                                                      if ct_launches else None),
                     "share_of_step": ct.get("share_of_step"),
                     "peak_source": f"{pk_kind} bf16 dense, sustained",
                     "all_conv": {"achieved": achieved_all, "unit": "TFLOP/s",
                                  "frac": achieved_all / peak if peak else None,
                                  "share_of_step": (prof["conv_ms"] / 1e3) / elapsed if elapsed else None,
                                  "dram_bytes_per_step": CONV_DRAM_BYTES_PER_AUDIO_S * secs_all / world / args.steps,
                                  "dram_source": "ncu, batch-8 step, all conv launches, scaled by audio seconds"}},
        "roofline_classes": classes,
        "cpu_baseline": cpu,
        "clocks": clk,
        "host_enqueue_ms_per_step": round(host_enqueue_ms, 2),
        "host_enqueue_ms_from_idle": round(enqueue_idle_ms, 3),
        "gpu_launches": prof["launches"],
        "ttfa_p50_ms": ttfa,
        "lstm": lstm,
        "prosody": prosody,
        "frontend": frontend,
        "vocos": vocos,
        "queue": queue,
        "stream": stream,
        "parity_vs_c_library": parity,
        "single_gpu_legs": "measured" if world == 1 else "N = 1 only (ttfa, lstm, prosody, queue, stream, frontend, "
                                                         "vocos, cpu_baseline, parity: see the N = 1 line)",
        "pipeline_tflops": value / world * algorithmic_flop_per_asr_frame() * 40.0 / 1e12,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
