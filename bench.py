"""Benchmark of the decoder token loop: decoder tokens/s on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

One bench step is one pass of the hot path over one batch of synthetic input:
for every window on the GPU, the sequence start (cross-attention keys and
values from the encoder rows), the prompt step, and greedy single-token steps
until `steps` tokens per window are sampled -- WhisperEACP's decodeTranscript
with no end-of-text stop.  The metric counts sampled tokens.

The default configuration is medium.en with 64 windows (bf16).  Multi-GPU
(torchrun, one process per GPU): the batch's windows are split evenly over
the ranks (strong scaling; every rank holds the weights and decodes its own
windows, no collective on the data path); the time is the maximum over
ranks and the value is the batch's tokens over that time.  Rank 0 also
times base.en at one window (the batch-1 milliseconds per token step).

`--impl reference` times the reference's own CPU decoder (its scalar test
decoder, compiled from its sources into oracle/_ref/libref_decoder.so) on the
host cores, on rank 0 only, on a bounded sample of the configuration.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decoder tokens/s"
UNIT = "tokens/s"
DEFAULT_CONFIG = "medium_en_b64"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default=DEFAULT_CONFIG)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-batch1", action="store_true", help="skip the extra base.en batch-1 timing")
    p.add_argument("--no-audio", action="store_true",
                   help="skip the base.en audio -> log-mel -> encoder -> greedy tokens timing")
    p.add_argument("--tokens", type=int, default=0,
                   help="tokens per window (default: the config's); smaller for profiler captures")
    p.add_argument("--windows", type=int, default=0,
                   help="windows per GPU (default: the config's); fewer for profiler captures")
    p.add_argument("--products", default="auto", choices=["auto", "mma", "tcgen05"],
                   help="the products' form (default: the decoder's choice for the window count)")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, sm_max, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.file.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.file.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(sm_max),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- measurement

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(kernel: str, config: str):
    """DRAM bytes (read + write) per single-token step of `kernel` from the
    committed ncu summary of that kernel and config, if there is one."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    if not os.path.exists(path):
        return None
    match = re.search(r"traffic_bytes_per_step:\s*([0-9.eE+]+)", open(path).read())
    return float(match.group(1)) if match else None


def step_bytes(run, windows: int, mean_keys: float) -> dict:
    """Algorithmic bytes of one single-token step of `windows` windows on one
    GPU (16-bit weights and caches): w_b*(L*(6d^2 + 2dF) + V*d) +
    B*L*2d*(X + t + 1)*kv_b."""
    s = run.shape
    d, L, F, V, X = s.width, s.layers, s.feed_forward_width, s.vocabulary_size, s.cross_positions
    weights = 2 * (L * (6 * d * d + 2 * d * F) + V * d)
    kv = windows * L * 2 * d * (X + mean_keys) * 2
    return {"weights": weights, "kv": kv}


def cpu_baseline_port(run, tensors, encoder, threads: int) -> dict:
    """The oracle (the reference's decoder restated, KV-cached, threaded) on a
    bounded sample: the sequence start and 8 single-token steps of one window."""
    from oracle import oracle as O
    shape = O.Shape(**run.shape.__dict__)
    session = O.Session(shape, tensors, threads=threads)
    t0 = time.perf_counter()
    session.begin(encoder[0])
    t_begin = time.perf_counter() - t0
    session.step(list(run.prompt), want_logits=True)
    sample = 8
    t0 = time.perf_counter()
    for k in range(sample):
        session.step([int(50 + k)], want_logits=True)
    t_step = (time.perf_counter() - t0) / sample
    per_window = t_begin + run.steps * t_step
    return {"value": run.steps / per_window, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"oracle/wsp_oracle.c on one window: sequence start ({t_begin:.2f} s) + "
                       f"{sample} single-token steps ({t_step * 1e3:.1f} ms each), extrapolated to "
                       f"{run.steps} tokens per window")}


# --------------------------------------------------------------------- ours

def rank_encoder_rows(run, windows) -> np.ndarray:
    """This rank's encoder rows: window w of the batch is seeded by w alone, so
    a window's rows do not depend on how the batch is split across ranks."""
    from whispereacp_b200 import synthetic as S
    shape = run.shape
    out = np.empty((len(windows), shape.cross_positions, shape.width), np.float32)
    for i, w in enumerate(windows):
        out[i] = S.encoder_output(1, shape.cross_positions, shape.width, seed=1000 + w)[0]
    return out


def time_transcriptions(decoder, device_rows, tokens_per_window, steps, stream, flush):
    """Device-timed transcriptions (CUDA events on the decoder's stream, the L2
    flushed before each, outside the timed interval) and each one's phases."""
    import torch
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    phases = []
    for i in range(steps):
        with torch.cuda.stream(stream):
            flush.zero_()
            starts[i].record(stream)
        decoder.enqueue_transcribe(device_rows.data_ptr(), tokens_per_window)
        stops[i].record(stream)
        # The step's own launches, from the decoder's CUDA events on the same
        # stream (this waits for the step; the next flush is queued after).
        phases.append(decoder.phase_ms())
    decoder.synchronize()
    return sum(a.elapsed_time(b) for a, b in zip(starts, stops)), phases


def batch1_line(args, local, flush, peak):
    """base.en at one window (configuration C2's decoder), timed on this GPU:
    the batch-1 milliseconds per single-token step and their roofline share."""
    import torch
    from whispereacp_b200 import Decoder, synthetic as S
    run = S.CONFIGS["base_en_b1"]
    shape = run.shape
    decoder = Decoder(shape, windows=1, device=local, storage=run.storage)
    decoder.load_weights(S.normal_weights(shape, seed=0))
    first, later = S.suppression_masks(shape.vocabulary_size)
    decoder.set_generation(run.prompt, first, later, maximum_tokens=run.steps,
                           end_of_text=S.END_OF_TEXT, stop_at_end_of_text=False)
    stream = torch.cuda.ExternalStream(decoder.stream, device=local)
    rows = torch.from_numpy(S.encoder_output(1, shape.cross_positions, shape.width, seed=1)).to(f"cuda:{local}")
    for _ in range(3):
        decoder.enqueue_transcribe(rows.data_ptr(), run.steps)
    decoder.synchronize()
    _, phases = time_transcriptions(decoder, rows, run.steps, max(3, min(args.steps, 10)), stream, flush)
    decoder.close()
    later_steps = run.steps - 1
    launch_ms = statistics.median(p["steps"] for p in phases)
    per_step = sum(step_bytes(run, 1, len(run.prompt) + later_steps / 2).values())
    ms = launch_ms / later_steps
    return {"workload": run.description, "ms_per_token_step": ms, "tokens_per_s": 1e3 / ms,
            "algorithmic_bytes_per_token_step": per_step,
            "roofline_frac": per_step / (ms * 1e-3) / 1e9 / peak}


def audio_line(args, local):
    """Configuration C2 end to end on one GPU: 30 s of audio (three seeded
    sinusoids and N(0, 0.05) noise) through the log-mel spectrogram and the
    base.en encoder (random-init weights), then 224 greedy tokens: host
    samples in, token ids out, through the public calls."""
    import ctypes
    import torch
    from whispereacp_b200 import synthetic as FE
    from whispereacp_b200 import Decoder, Encoder, EncoderShape, synthetic as S
    run = S.CONFIGS["base_en_b1"]
    shape = run.shape
    eshape = EncoderShape(80, shape.width, shape.heads, shape.layers, shape.feed_forward_width, 3000)
    encoder = Encoder(eshape, device=local)
    encoder.load_weights(FE.synthetic_encoder_tensors(80, shape.width, shape.layers, shape.feed_forward_width, 1500,
                                                      seed=1, scale=0.02))
    encoder.set_filters(FE.synthetic_filters(80))
    decoder = Decoder(shape, windows=1, device=local, storage=run.storage)
    decoder.load_weights(S.normal_weights(shape, seed=0))
    first, later = S.suppression_masks(shape.vocabulary_size)
    decoder.set_generation(run.prompt, first, later, maximum_tokens=run.steps, end_of_text=S.END_OF_TEXT,
                           stop_at_end_of_text=False)
    audio = torch.from_numpy(FE.synthetic_audio(480000)).pin_memory()
    rows = torch.empty((1500, shape.width), dtype=torch.float32, device=f"cuda:{local}")
    lib = encoder._lib
    from whispereacp_b200._native import check

    def once():
        t0 = time.perf_counter()
        check(lib.wsp_encoder_encode_samples(encoder._handle, ctypes.c_void_p(audio.data_ptr()), 480000,
                                             ctypes.c_void_p(rows.data_ptr())))
        t1 = time.perf_counter()
        ids = decoder.transcribe(rows.data_ptr())[0]
        t2 = time.perf_counter()
        return (t1 - t0) * 1e3, (t2 - t1) * 1e3, len(ids)

    for _ in range(2):
        once()
    samples = [once() for _ in range(max(3, min(args.steps, 5)))]
    front = statistics.median(x[0] for x in samples)
    decode = statistics.median(x[1] for x in samples)
    encoder.close()
    decoder.close()
    return {"workload": "base.en: 30 s of audio -> log-mel -> encoder -> 224 greedy tokens, 1 window",
            "ms_per_window": front + decode, "frontend_ms": front, "decode_ms": decode,
            "tokens_per_s": samples[0][2] / ((front + decode) * 1e-3),
            "timing": "host clock around the public calls (pinned host samples in, token ids out), median"}


def run_ours(args, run):
    import torch
    from whispereacp_b200 import Decoder, synthetic as S
    from whispereacp_b200.ranks import max_over_ranks, window_range

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))

    shape = run.shape
    tokens_per_window = args.tokens or run.steps
    # The batch's windows split evenly over the ranks (strong scaling): rank
    # r decodes windows window_range(total, r, world) with its own weights.
    mine = window_range(run.windows, rank, world)
    windows = len(mine)
    tensors = S.normal_weights(shape, seed=0)
    encoder = rank_encoder_rows(run, mine)
    first, later = S.suppression_masks(shape.vocabulary_size)

    decoder = Decoder(shape, windows=windows, device=local, storage=run.storage, products=args.products)
    decoder.load_weights(tensors)
    decoder.set_generation(run.prompt, first, later, maximum_tokens=tokens_per_window,
                           end_of_text=S.END_OF_TEXT, stop_at_end_of_text=False)
    stream = torch.cuda.ExternalStream(decoder.stream, device=local)
    device_rows = torch.from_numpy(encoder).to(f"cuda:{local}")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{local}")
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        decoder.enqueue_transcribe(device_rows.data_ptr(), tokens_per_window)
    decoder.synchronize()

    clocks = ClockSampler(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    elapsed_ms, phases = time_transcriptions(decoder, device_rows, tokens_per_window, args.steps, stream, flush)
    torch.cuda.synchronize()
    clock_record = clocks.stop()
    if world > 1:
        torch.distributed.barrier()
    transcript = decoder.read_transcript()
    assert all(len(t) == tokens_per_window for t in transcript)

    # End to end through the public call: pinned host rows in, token ids out.
    pinned = torch.from_numpy(encoder).pin_memory()
    e2e_ms = []
    for i in range(max(2, min(args.steps, 5)) + 1):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        decoder.transcribe(pinned.data_ptr())
        stop.record(stream)
        stop.synchronize()
        if i > 0:
            e2e_ms.append(start.elapsed_time(stop))
    e2e_step_ms = statistics.median(e2e_ms)

    # Per-op times of the single-token step, measured live.
    decoder.enqueue_transcribe(device_rows.data_ptr(), 2)
    per_kernel = decoder.time_kernels(min(64, shape.max_positions - len(run.prompt) - 2, tokens_per_window))
    decoder.synchronize()
    launches = decoder.step_launches()
    decoder.close()

    step_ms = elapsed_ms / args.steps
    # The slowest rank's device-timed step (an all-reduce MAX over NCCL).
    step_ms, e2e_step_ms = max_over_ranks([step_ms, e2e_step_ms], device=f"cuda:{local}")

    peak, peak_kind = peaks()
    extra = batch1_line(args, local, flush, peak) if rank == 0 and not args.no_batch1 else None
    audio = audio_line(args, local) if rank == 0 and not args.no_audio else None
    if world > 1:
        torch.distributed.barrier()
    tokens = run.windows * tokens_per_window
    result = None
    if rank == 0:
        # The dominant kernel: the decode kernel's launch that runs every
        # single-token step of the transcription (the prompt launch and the
        # sequence start are the rest of the step), on this rank's windows.
        later_steps = tokens_per_window - 1
        mean_keys = len(run.prompt) + later_steps / 2
        nbytes = step_bytes(run, windows, mean_keys)
        per_step_bytes = nbytes["weights"] + nbytes["kv"]
        launch_ms = statistics.median(p["steps"] for p in phases)
        algorithmic = later_steps * per_step_bytes
        achieved = algorithmic / (launch_ms * 1e-3) / 1e9 if launch_ms > 0 else 0.0
        traffic_step = committed_traffic("decode_kernel", run.name)
        h2d = encoder.nbytes
        d2h = windows * (shape.max_positions + 1) * 4
        result = {
            "metric": METRIC, "value": tokens / (step_ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f16" if run.storage == "float16" else "bf16",
            "data": "synthetic (random-init weights N(0,0.02), encoder rows N(0,1))",
            "config": {"workload": run.description, "name": run.name, "windows": run.windows,
                       "windows_per_gpu": windows, "tokens_per_window": tokens_per_window,
                       "prompt": list(run.prompt), "cross_positions": shape.cross_positions,
                       "d_model": shape.width, "decoder_layers": shape.layers,
                       "vocabulary": shape.vocabulary_size,
                       "step": "sequence start + prompt step + greedy single-token steps (one persistent launch)",
                       "l2": "flushed (256 MiB write) between timed steps, outside the timed intervals; "
                             "the cross keys and values alone exceed L2",
                       "parallelism": f"dp{world} ({run.windows} windows split evenly across the GPUs)",
                       "products": args.products},
            "e2e": {"value": tokens / (e2e_step_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": traffic_step * later_steps if traffic_step else None,
                         "kernel": "decode_kernel (launch of the single-token steps), rank 0's windows",
                         "peak_source": f"{peak_kind} hbm_gbs (burst)",
                         "algorithmic_bytes_per_launch": algorithmic,
                         "algorithmic_bytes_per_token_step": per_step_bytes,
                         "token_steps_per_launch": later_steps, "launch_ms": launch_ms},
            "phases_ms": {k: statistics.median(p[k] for p in phases) for k in phases[0]},
            "op_classes_us": {k: {"us_per_op": v[0] * 1e3, "ops_per_token_step": v[1]}
                              for k, v in per_kernel.items() if v[1]},
            "clocks": clock_record,
        }
        if extra is not None:
            result["batch1"] = extra
            result["batch1_ms_per_token_step"] = extra["ms_per_token_step"]
        if audio is not None:
            result["audio_to_tokens"] = audio
        if not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            result["cpu_baseline"] = cpu_baseline_port(run, tensors_for_oracle(tensors, run.storage),
                                                       encoder, threads)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return result


def tensors_for_oracle(tensors, storage):
    from tests.helpers import stored_tensors
    return stored_tensors(tensors, storage)


# ---------------------------------------------------------------- reference

def run_reference(args, run):
    """The reference's own CPU decoder (Tests/Decoder/Common.h:360-468, compiled
    from its sources) as a greedy decoder: each generated token is one
    referenceDecode over the prefix, which is how that implementation decodes.
    All host threads decode independent windows at once (ctypes releases the GIL).

    One token of a 24- or 32-layer decoder takes that code minutes, so a step
    is a bounded sample of the same workload: every thread decodes one token
    of a ONE-layer decoder of the configured architecture (the same width,
    heads, feed-forward width, vocabulary and 1500 encoder rows).  A token's
    cost is fixed (embedding, final norm, logits) plus L times a layer's
    (its cross keys and values, its three sublayers): a one-off two-layer
    decode before the warm-up separates the two, and the value is the
    configured L-layer decoder's tokens/s on all threads."""
    from concurrent.futures import ThreadPoolExecutor
    from dataclasses import replace
    from oracle import oracle as O
    from whispereacp_b200 import synthetic as S
    from tests.golden.make_golden import load_reference, ref_decode

    rank, world, _ = dist_env()
    if rank != 0:
        return None
    path = os.path.join(ROOT, "oracle", "_ref", "libref_decoder.so")
    if not os.path.exists(path):
        return {"impl": "reference", "unavailable": "oracle/_ref/libref_decoder.so was not built"}
    ref, _ = load_reference()
    layers = run.shape.layers
    threads = os.cpu_count() or 1
    prefix = [*run.prompt, 50, 51]
    encoder = S.encoder_output(1, run.shape.cross_positions, run.shape.width, seed=1)[0]
    pool = ThreadPoolExecutor(max_workers=threads)

    def decoder_of(count):
        shape = replace(run.shape, layers=count)
        return O.Shape(**shape.__dict__), tensors_for_oracle(S.normal_weights(shape, seed=0), run.storage)

    def all_threads(model):
        shape, tensors = model
        t0 = time.perf_counter()
        list(pool.map(lambda _: ref_decode(ref, shape, tensors, encoder, prefix), range(threads)))
        return time.perf_counter() - t0

    one, two = decoder_of(1), decoder_of(2)
    all_threads(one)
    all_threads(two)
    t_two = all_threads(two)
    for _ in range(args.warmup):
        all_threads(one)
    times = [all_threads(one) for _ in range(args.steps)]
    pool.shutdown()
    t_one = sum(times) / len(times)
    # A layer costs at most the whole one-layer token (the fixed part is not negative).
    per_layer = min(max(t_two - t_one, 0.0), t_one)
    token_s = (t_one - per_layer) + layers * per_layer
    value = threads / token_s
    sample = (f"each step: {threads} concurrent referenceDecode calls (one per host thread) of a 1-layer "
              f"decoder of this architecture over a {len(prefix)}-token prefix and "
              f"{run.shape.cross_positions} encoder rows ({t_one:.2f} s); a 2-layer run ({t_two:.2f} s) "
              f"splits that into a fixed part and a per-layer part, extrapolated to {layers} layers "
              f"({token_s:.1f} s a token on every thread)")
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_one * 1e3, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": {"workload": run.description, "name": run.name,
                                            "windows": run.windows},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse_args()
    from dataclasses import replace
    from whispereacp_b200.synthetic import CONFIGS
    run = CONFIGS[args.config]
    if args.windows:
        run = replace(run, windows=args.windows, description=f"{run.description}, run with {args.windows} windows")
    result = run_reference(args, run) if args.impl == "reference" else run_ours(args, run)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
