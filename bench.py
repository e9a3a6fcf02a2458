#!/usr/bin/env python3
"""Benchmark of the strict speculative verify step.

Workload (one "step"): the random-init Qwen3-0.6B q8_0 decoder, KV cache
prefilled to 2048 positions with synthetic fp16 K/V, one verify step of
k+1 = 8 rows (seed + 7 proposals), LM-head first max and acceptance.  The
proposal is the target's own greedy continuation for floor(7/2) = 3 tokens
followed by wrong tokens, so every step commits 3 accepted + 1 bonus = 4
tokens and rolls the cache back by 4 rows; the step state is restored on the
device before each step so every step sees the same 2048-position cache.

  value  decoded tokens/s with inputs resident in HBM (device-to-device state
         restore + the captured verify-step graph), whole job over N GPUs;
  e2e    the same metric through the public C ABI with host buffers
         (mtb_resume + mtb_spec_step + mtb_read_ids: host->device and
         device->host copies inside the timed region).

Side lines: `recordings` (configs[4] at every N: 64 recordings of 1500 prompt
rows + 768 decoded tokens, round robin over the ranks, each GPU stepping its
share in groups of 8 through the public calls), and at N=1 `config0`
(configs[0] end to end), `prefill`, `multi_stream`, `long_context`,
`f16_recording`.

`--impl reference` times the CPU restatement of the reference path (the
oracle, built for the host's own ISA with -march=native: the reference's own
ggml build cannot be compiled here) on the same workload with all host cores.  Multi-GPU (torchrun): one independent decoder
replica per GPU, no collective on the data path (weak scaling); rank 0 prints.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "moss-transcribe.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

METRIC = "decoded tokens/s/GPU, strict spec-decode, Qwen3-0.6B q8_0; % of HBM roofline"
UNIT = "tokens/s"
KV_LEN = 2048
T_ROWS = 8
KV_SEED = 1234
PREFILL_ROWS = 407  # configs[1]: 375 audio rows + 32 text rows
# Algorithmic bytes of one verify step (q8_0 weights + LM head once, F32 norms,
# fp16 K+V reads of the cached positions, KV append, embedding rows).
WEIGHT_BYTES = 633_233_408
NORM_BYTES = 262_144
KV_BYTES_PER_POS = 114_688
EMBED_BYTES_PER_ROW = 1_088
# configs[4] sample (multi-stream box throughput): recordings of 1500 audio rows
# (the KV cache they leave, synthetic fp16), decoded with the device n-gram
# draft at k = 8, on one GPU.
MS_STREAMS = 8
MS_KV = 1500
MS_STEPS = 48
MS_NEW = 768  # configs[4]: decoded tokens per recording
MS_RECORDINGS = 64  # configs[4]: recordings on the node, round robin over the GPUs
CONFIG0_NEW = 256  # configs[0]: decoded tokens after the 407-row prompt
# configs[3] context length: a 30-minute recording leaves ~27k cached positions.
LC_KV = 27000
LC_STEPS = 50
PREFILL_LONG_ROWS = 22528  # configs[3]: 60 chunks x 375 audio rows + markers
F16_CHUNKS = 5  # configs[2]: 5 chunks x 375 audio rows, a marker token per chunk, 64 prompt tokens
F16_PROMPT_TOKENS = 64
F16_NEW = 1024


# F16 weights: 28 layers x 15,728,640 weights + the 151936 x 1024
# LM head, two bytes each; an embedding row is 1024 fp16 values.
F16_WEIGHT_BYTES = 1_191_968_768
F16_EMBED_BYTES_PER_ROW = 2_048


def step_bytes(kv_len: int, T: int, f16: bool = False) -> int:
    w, e = (F16_WEIGHT_BYTES, F16_EMBED_BYTES_PER_ROW) if f16 else (WEIGHT_BYTES, EMBED_BYTES_PER_ROW)
    return w + NORM_BYTES + kv_len * KV_BYTES_PER_POS + T * KV_BYTES_PER_POS + T * e


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = f"/tmp/mtb_clocks_{os.getpid()}.csv"

    def start(self):
        """Start sampling and wait (up to 5 s) for the first sample, so the
        timed region that follows is covered from its start."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.02)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args=None):
    """One process per GPU (torchrun's RANK / LOCAL_RANK / WORLD_SIZE): NCCL
    over the node's GPUs, used only for the barriers around the timed region
    and the max over ranks of the measured times (replicas: no data-path
    collective).  MTB_DIST_BACKEND=gloo runs the same host logic on CPU ranks
    (the multi-rank tests)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        backend = os.environ.get("MTB_DIST_BACKEND", "nccl")
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)  # rank -> GPU stated, not guessed
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
        return rank, local, world, dist, torch
    return rank, local, world, None, None


def max_over_ranks(x: float, dist, torch, local: int) -> float:
    """The largest x over all ranks (a multi-GPU time is its slowest rank's)."""
    if not dist:
        return x
    dev = f"cuda:{local}" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, dist, torch, local: int) -> float:
    """The sum of x over all ranks."""
    if not dist:
        return x
    dev = f"cuda:{local}" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def job_throughput(world: int, units_per_rank: float, seconds: float) -> float:
    """Whole-job rate: every rank processed units_per_rank in at most `seconds`."""
    return world * units_per_rank / seconds


def greedy_draft(model_path: str, dec, kv_len: int, T: int, seed_tok: int, vocab: int):
    """The target's greedy continuation (floor((T-1)/2) tokens) + wrong tokens."""
    keep = (T - 1) // 2
    dec.resume([seed_tok], kv_len, 64, -1, k_max=0)
    for _ in range(keep + 1):
        dec.spec_step(None)
    ids, _ = dec.read_ids()
    chain = ids[:keep + 2]
    draft = chain[1:1 + keep] + [(chain[1 + keep] + 1 + i) % vocab for i in range(T - 1 - keep)]
    return draft, keep


def cpu_baseline(path: str, steps: int, sample_s: float = 20.0):
    """The CPU restatement (oracle) on the same workload, all host cores."""
    import oracle
    from mtb import fixture
    oracle.use_native()  # -march=native on this host (AVX-512 / VNNI where present)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    om = oracle.OracleModel(path)
    V = om.shape.vocab
    od = oracle.OracleDecoder(om, KV_LEN + 32, kv_fp16=True)
    od.fill_synthetic_kv(KV_LEN, KV_SEED)
    seed_tok = int(fixture.lcg_ids(1, V, seed=99)[0])
    keep = (T_ROWS - 1) // 2
    draft = [(seed_tok + 1 + i) % V for i in range(T_ROWS - 1)]
    times = []
    t_end = time.time() + sample_s
    while len(times) < max(1, steps) and (time.time() < t_end or not times):
        od.rewind(KV_LEN)
        t0 = time.perf_counter()
        # One verify step as the reference computes it: append T rows, then
        # lazy per-row logits for the accepted prefix (keep + 1 rows).
        h = od.run(om.embed([seed_tok] + draft))
        for r in range(keep + 1):
            od.logits(h[r])
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": (keep + 1) / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{len(times)} verify steps of T={T_ROWS} at kv {KV_LEN} (fp16-rounded KV), "
                      f"append + {keep + 1} lazy LM-head rows each, median {t * 1e3:.1f} ms; "
                      f"C restatement built -O3 -march=native ({oracle.host_isa()})",
            "ms_per_step": round(t * 1e3, 2), "isa": oracle.host_isa(),
            "reference_published_xeon_ms": {"prefix_512_T8": 34.292, "prefix_1024_T8": 40.435,
                                            "source": "cpu-lab/causal-context.md:86,89 (16-core Xeon Gold 5416S, "
                                                      "all 8 logit rows)"}}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the prefill / multi_stream / long_context side measurements (profiling runs)")
    ap.add_argument("--f16", action="store_true",
                    help="the same verify-step microbench on the F16-weight decoder of configs[2] "
                         "(no side measurements, no CPU baseline)")
    ap.add_argument("--only", choices=["long_context", "recordings", "config0", "audio"],
                    help="run one side measurement alone and print it as one JSON line (profiling runs)")
    args = ap.parse_args(argv)
    if args.f16:
        args.no_extras = args.no_cpu_baseline = True
    rank, local, world, dist, torch = dist_setup(args)
    if args.impl == "reference" and rank != 0:
        return  # the reference arm runs on rank 0's host cores only
    from mtb import fixture
    path = fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0, dtype="f16" if args.f16 else "q8_0")
    wname = "F16" if args.f16 else "q8_0"
    config = {"workload": "configs[1] verify-step microbench: KV 2048 fp16 synthetic, k+1=8, draft matches 3"
                          + (" (configs[2]'s F16 decoder weights)" if args.f16 else ""),
              "model": f"Qwen3-0.6B decoder (random-init N(0,0.02), {wname})", "kv_len": KV_LEN, "k_plus_1": T_ROWS,
              "tokens_per_step": 4,
              "l2": f"inputs larger than L2 ({'1192' if args.f16 else '633'} MB of weights streamed per step)",
              "parallelism": f"replicas x{world}"}
    metric = METRIC.replace("q8_0", "F16") if args.f16 else METRIC

    if args.impl == "reference":
        cb = cpu_baseline(path, max(args.steps, 1))
        line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "q8_0 x q8_0 -> f32", "data": "synthetic", "config": config,
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                             "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    from mtb import capi
    if args.only == "audio":
        line = audio_front_end(capi, fixture, local, cpu=rank == 0 and world == 1 and not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps({args.only: line}))
        return
    model = capi.Model(path, local)
    if args.only:
        if args.only == "long_context":
            line = long_context(model, capi, int(fixture.lcg_ids(1, model.vocab, seed=99)[0]))
        elif args.only == "recordings":
            line = recordings_line(model, capi, dist, torch, rank, local, world)
        else:
            line = config0(model, capi, fixture)
        if rank == 0:
            print(json.dumps({args.only: line}))
        return
    dec = capi.Decoder(model, KV_LEN + 64, capi.KV_F16, max_new=64)
    dec.fill_synthetic_kv(KV_LEN, KV_SEED)
    V = model.vocab
    seed_tok = int(fixture.lcg_ids(1, V, seed=99)[0])
    draft, keep = greedy_draft(path, dec, KV_LEN, T_ROWS, seed_tok, V)
    tokens_per_step = keep + 1

    # ---- value: device-resident inputs, captured step graph ----------------
    dec.resume([seed_tok], KV_LEN, 64, -1, k_max=15)
    dec.snapshot_save()
    import ctypes as C
    draft_arr = np.asarray(draft, dtype=np.int32)
    # Device copy of the proposal through the library's own upload path.
    dbuf = _device_ids(dec, draft_arr)
    for _ in range(max(3, args.warmup)):
        dec.snapshot_restore_async()
        dec.spec_step_async(dbuf, len(draft))
    dec.sync()
    ids, c = dec.read_ids()
    assert c["accepted"] == keep and len(ids) == keep + 2, (ids, c)
    launches = dec.step_kernel_launches() + 1  # + the proposal upload kernel
    if dist:
        torch.cuda.synchronize()
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    dec.sync()
    dec.event_record(2)
    for _ in range(args.steps):
        dec.snapshot_restore_async()
        dec.spec_step_async(dbuf, len(draft))
    dec.event_record(3)
    ms = dec.event_elapsed_ms(2, 3)
    clk = clocks.stop()
    ids, c = dec.read_ids()
    assert c["accepted"] == keep, c
    ms = max_over_ranks(ms, dist, torch, local)
    ms_step = ms / args.steps
    value = job_throughput(world, args.steps * tokens_per_step, ms / 1e3)

    # ---- e2e: the public C ABI with host buffers ------------------------------
    h0 = dec.transfer_bytes()
    n_e2e = max(10, args.steps // 4)
    for _ in range(3):
        dec.resume([seed_tok], KV_LEN, 64, -1, k_max=15)
        dec.spec_step(draft)
        dec.read_ids()
    h0 = dec.transfer_bytes()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        dec.resume([seed_tok], KV_LEN, 64, -1, k_max=15)
        dec.spec_step(draft)
        got, _ = dec.read_ids()
    e2e_s = time.perf_counter() - t0
    h1 = dec.transfer_bytes()
    e2e_s = max_over_ranks(e2e_s, dist, torch, local)
    e2e = {"value": job_throughput(world, n_e2e * tokens_per_step, e2e_s), "unit": UNIT,
           "h2d_bytes_per_step": (h1[0] - h0[0]) // n_e2e + len(draft) * 4,
           "d2h_bytes_per_step": (h1[1] - h0[1]) // n_e2e,
           "ms_per_step": e2e_s * 1e3 / n_e2e}

    prefill = ms_line = lc_line = f16_line = c0_line = rec_line = audio_line = None
    if not args.no_extras and model.persistent_grid > 0:
        rec_line = recordings_line(model, capi, dist, torch, rank, local, world)
    if not args.no_extras and world == 1:  # per-GPU side measurements: the N=1 run carries them
        # ---- prefill: the prompt rows of configs[1] (375 audio + 32 text rows)
        # through the public run() call, host rows in and hidden rows out; every
        # layer over all rows at once with the projections on tcgen05.
        pf_dec = capi.Decoder(model, PREFILL_ROWS + 64, capi.KV_F16, max_new=16)
        pf_rows = np.random.default_rng(5).standard_normal((PREFILL_ROWS, model.hidden)).astype(np.float32)
        pf_dec.run(pf_rows)
        pf_times = []
        for _ in range(5):
            pf_dec.rewind(0)
            t0 = time.perf_counter()
            pf_dec.run(pf_rows)
            pf_times.append(time.perf_counter() - t0)
        pf_dec.close()
        pf_s = statistics.median(pf_times)
        # configs[3]'s prompt length (one run after a warm-up pass of 512 rows).
        pl_dec = capi.Decoder(model, PREFILL_LONG_ROWS + 64, capi.KV_F16, max_new=16)
        pl_rows = np.random.default_rng(6).standard_normal((PREFILL_LONG_ROWS, model.hidden)).astype(np.float32)
        pl_dec.run(pl_rows[:512])
        pl_dec.rewind(0)
        t0 = time.perf_counter()
        pl_dec.run(pl_rows)
        pl_s = time.perf_counter() - t0
        pl_dec.close()
        ms_line = _side("multi_stream", lambda: multi_stream(model, capi, fixture)) if model.persistent_grid > 0 else None
        c0_line = _side("config0", lambda: config0(model, capi, fixture))
        lc_line = _side("long_context", lambda: long_context(model, capi, seed_tok))
        f16_line = _side("f16_recording", lambda: f16_recording(capi, fixture, local))
        audio_line = _side("audio_front_end", lambda: audio_front_end(capi, fixture, local, cpu=not args.no_cpu_baseline))
        if isinstance(audio_line, dict) and "error" not in audio_line:
            audio_line["config0_from_samples"] = _side("config0_from_samples",
                                                       lambda: config0_from_samples(model, capi, fixture, local))
        prefill = {"rows": PREFILL_ROWS, "ms": round(pf_s * 1e3, 3), "rows_per_s": round(PREFILL_ROWS / pf_s, 1),
                   "long": {"rows": PREFILL_LONG_ROWS, "ms": round(pl_s * 1e3, 1),
                            "rows_per_s": round(PREFILL_LONG_ROWS / pl_s, 1)},
                   "path": "prefill passes over every row (tcgen05 q8_0 projections, register-blocked attention); the first token's LM head from the last pass",
                   "timing": "host wall clock around run(), median of 5, host rows in, hidden rows out"}

    peak, peak_kind = measured_peaks()
    bytes_step = step_bytes(KV_LEN, T_ROWS, args.f16)
    achieved = bytes_step / (ms_step / 1e3) / 1e9
    kernel = ("k_verify_persistent (the whole verify step, one launch)" if model.persistent_grid > 0
              else "verify step (one CUDA graph of kernels)")
    roofline = {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1),
                "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "algorithmic_bytes": bytes_step,
                # DRAM bytes come from an ncu capture only (profiles/); no number is carried over here.
                "traffic": None}
    line = {"metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": ("f16 x f16 -> f32" if args.f16 else "q8_0 x q8_0 -> f32") + " (fp16 KV)",
            "data": "synthetic", "config": config,
            "roofline": roofline, "e2e": e2e, "gpu_launches": launches * args.steps, "clocks": clk,
            "prefill": prefill, "recordings": rec_line, "config0": c0_line, "multi_stream": ms_line,
            "long_context": lc_line, "f16_recording": f16_line, "audio_front_end": audio_line}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(path, 5)
    if rank == 0:
        print(json.dumps(line))
    dec.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def audio_front_end(capi, fixture, device: int, cpu: bool = True) -> dict:
    """Row (f)4: the audio front end (log-mel, the 24-layer Whisper-Medium
    encoder, the adaptor) of a random-init GGUF on one GPU, through the public
    mtb_audio_encode call with host samples in and host rows out: one 30 s
    chunk (375 rows) and configs[2]'s five chunks (1875 rows).  CPU baseline:
    the C restatement on one chunk, all host threads."""
    path = fixture.cached_audio_fixture(fixture.WHISPER_MEDIUM, seed=0)
    enc = capi.AudioEncoder(path, device)
    s = fixture.WHISPER_MEDIUM
    out = {"model": "Whisper-Medium encoder (24 x 1024, 16 heads, ffn 4096) + adaptor -> 1024, random-init q8_0",
           "timing": "host wall clock around mtb_audio_encode (samples host->device, rows device->host), median of 5; "
                     "device_ms from CUDA events around the same call"}
    # Work per chunk: q8_0 linears (int8 ops) and the F32 attention and conv stem (flops).
    T, d = s.enc_frames, s.d_model
    lin = 2 * T * (4 * d * d + 2 * d * s.ffn) * s.n_layers
    att = 2 * 2 * T * T * d * s.n_layers
    conv = 2 * (s.n_frames * d * 3 * s.n_mels + T * d * 3 * d)
    for name, n in (("chunk_30s", s.n_samples), ("configs2_150s", 5 * s.n_samples)):
        x = fixture.synthetic_pcm(n, seed=7)
        enc.encode(x)
        walls, devs = [], []
        for _ in range(5):
            t0 = time.perf_counter()
            rows = enc.encode(x)
            walls.append(time.perf_counter() - t0)
            devs.append(enc.last_ms())
        w = statistics.median(walls)
        chunks = (n + s.n_samples - 1) // s.n_samples
        out[name] = {"samples": n, "rows": int(rows.shape[0]), "ms": round(w * 1e3, 2),
                     "device_ms": round(statistics.median(devs), 2), "realtime_x": round(n / 16000 / w, 1),
                     "rows_per_s": round(rows.shape[0] / w, 1),
                     "tera_ops_per_s": round(chunks * (lin + att + conv) / (statistics.median(devs) / 1e3) / 1e12, 1)}
    out["ops_per_chunk"] = {"int8_linear": lin, "f32_attention": att, "f32_conv": conv}
    enc.close()
    if cpu:
        import oracle
        oracle.use_native()
        cores = os.cpu_count() or 1
        oracle.set_threads(cores)
        oa = oracle.OracleAudio(path)
        x = fixture.synthetic_pcm(s.n_samples, seed=7)
        t0 = time.perf_counter()
        oa.encode(x)
        t = time.perf_counter() - t0
        out["cpu_baseline"] = {"ms_per_chunk": round(t * 1e3, 1), "cores": cores, "kind": "port",
                               "sample": f"one 30 s chunk, C restatement -O3 -march=native ({oracle.host_isa()})"}
    return out


def recordings_line(model, capi, dist, torch, rank: int, local: int, world: int) -> dict:
    """configs[4] at N GPUs: 64 recordings (1500 synthetic N(0, 1) prompt rows +
    768 decoded tokens each, device n-gram draft k = 8), recording i on rank
    i mod N, each rank decoding its share in groups of 8 (one persistent launch
    per group step) through the public calls (mtb_spec_prime,
    mtb_spec_run_group, mtb_read_ids): host rows in, ids out.  The job's time
    is its slowest rank's (wall clock around the rank's share, after a barrier);
    tokens are summed over the ranks."""
    from mtb import recordings
    mine = recordings.partition(MS_RECORDINGS, world, rank)
    recs = [recordings.Recording(np.random.default_rng(700 + i).standard_normal((MS_KV, model.hidden))
                                 .astype(np.float32), MS_NEW) for i in mine]
    recordings.decode_recordings(model, recs[:1] if recs else [], k_max=8)  # warm-up (graphs, first prefill)
    if dist:
        torch.cuda.synchronize()
        dist.barrier()
    t0 = time.perf_counter()
    outs = recordings.decode_recordings(model, recs, k_max=8)
    dt = time.perf_counter() - t0
    toks = sum(len(ids) for ids, _ in outs)
    acc = sum(c["accepted"] for _, c in outs)
    worst = max_over_ranks(dt, dist, torch, local)
    total = sum_over_ranks(float(toks), dist, torch, local)
    return {"workload": f"configs[4]: {MS_RECORDINGS} recordings x ({MS_KV} prompt rows prefilled + {MS_NEW} tokens, "
                        f"device n-gram draft k=8), round robin over {world} GPU(s), groups of 8 per launch",
            "tokens_per_s": round(total / worst, 1), "tokens_per_s_per_gpu": round(total / worst / world, 1),
            "recordings_per_gpu": len(mine), "tokens": int(total), "s": round(worst, 3), "accepted_rank0": acc,
            "scaling": "weak per recording, strong per job: the 64 recordings are fixed, split over the GPUs",
            "timing": "wall clock around each rank's share (prefill + decode, ids read back), max over ranks"}


def config0(model, capi, fixture) -> dict:
    """configs[0] end to end: the 407-row prompt (375 N(0, 1) audio rows between
    two halves of 32 LCG text ids' embedding rows) prefilled and 256 tokens
    decoded, with the configs' draft (n = 3, k = 8) and with the reference
    policy (k = 4, n-grams 16..2), through mtb_spec_generate: host rows in,
    ids out."""
    import gguf  # the text ids' embedding rows come from the GGUF's token_embd (the fused prompt's input)
    reader = gguf.GGUFReader(fixture.cached_fixture(fixture.QWEN3_0_6B, seed=0))
    embd = next(np.ascontiguousarray(t.data) for t in reader.tensors if t.name == "token_embd.weight")
    prompt = fixture.synthetic_prompt(embd, fixture.read_shape(reader), n_audio=375, n_text=32)
    del reader, embd
    dec = capi.Decoder(model, prompt.shape[0] + CONFIG0_NEW + 64, capi.KV_F32, max_new=CONFIG0_NEW)
    capi.lib().mtb_set_log_level(0)
    out = {}
    try:
        for name, (k, n0, n1) in {"k8_n3": (8, 3, 3), "reference_k4_n2_16": (4, 2, 16)}.items():
            dec.cpu_speculative_generate(prompt, 16, -1, k_max=k, n_min=n0, n_max=n1)  # warm-up
            t0 = time.perf_counter()
            ids, c = dec.cpu_speculative_generate(prompt, CONFIG0_NEW, -1, k_max=k, n_min=n0, n_max=n1)
            dt = time.perf_counter() - t0
            out[name] = {"tokens_per_s": round(len(ids) / dt, 1), "s": round(dt, 4), "tokens": len(ids),
                         "target_calls": c["target_calls"], "accepted": c["accepted"]}
    finally:
        capi.lib().mtb_set_log_level(1)
        dec.close()
    return {"workload": "configs[0]: 407 prompt rows (375 audio + 32 text) prefilled + 256 tokens, F32 KV",
            **out, "timing": "host wall clock around mtb_spec_generate (prefill + decode), ids read back"}


def config0_from_samples(model, capi, fixture, device: int) -> dict:
    """configs[0]'s prompt made from 30 s of samples on the device instead of
    N(0, 1) rows: mtb_audio_encode (log-mel, Whisper-Medium encoder, adaptor:
    375 rows), then mtb_spec_generate_ids (32 LCG text ids around the 375 audio
    positions, fused and prefilled on the device, 256 tokens decoded with n = 3,
    k = 8): transcribe_pcm16k's device chain without the tokenizer."""
    audio = capi.AudioEncoder(fixture.cached_audio_fixture(fixture.WHISPER_MEDIUM, seed=0), device)
    samples = fixture.synthetic_pcm(480000, seed=7)
    audio_id = fixture.QWEN3_0_6B.audio_token_id
    text = fixture.lcg_ids(32, model.vocab).tolist()
    n_rows = audio.tokens(len(samples))
    ids = text[:16] + [audio_id] * n_rows + text[16:]
    dec = capi.Decoder(model, len(ids) + CONFIG0_NEW + 64, capi.KV_F32, max_new=CONFIG0_NEW)
    capi.lib().mtb_set_log_level(0)
    try:
        rows = audio.encode(samples)
        dec.spec_generate_ids(ids, rows, audio_id, 16, -1, k_max=8, n_min=3, n_max=3)  # warm-up
        t0 = time.perf_counter()
        rows = audio.encode(samples)
        t1 = time.perf_counter()
        out, c = dec.spec_generate_ids(ids, rows, audio_id, CONFIG0_NEW, -1, k_max=8, n_min=3, n_max=3)
        t2 = time.perf_counter()
    finally:
        capi.lib().mtb_set_log_level(1)
        dec.close()
        audio.close()
    return {"workload": "30 s of samples -> 375 audio rows -> 407-row prompt (ids + rows fused on the device) "
                        "prefilled + 256 tokens, F32 KV, n = 3, k = 8",
            "s": round(t2 - t0, 4), "audio_ms": round((t1 - t0) * 1e3, 2), "prefill_decode_s": round(t2 - t1, 4),
            "tokens": len(out), "tokens_per_s": round(len(out) / (t2 - t0), 1),
            "realtime_x": round(30.0 / (t2 - t0), 1), "target_calls": c["target_calls"], "accepted": c["accepted"],
            "timing": "host wall clock: mtb_audio_encode (samples in, rows out) + mtb_spec_generate_ids (ids out)"}


def _side(name: str, fn):
    """A side measurement: its failure is reported in the line instead of
    losing the headline numbers measured before it."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001
        print(f"side measurement {name} failed: {e!r}", file=sys.stderr)
        return {"error": repr(e)}


def long_context(model, capi, seed_tok) -> dict:
    """configs[3]'s context length: the configs[1] verify step (k+1 = 8, a
    draft whose first floor(7/2) tokens are the target's own continuation)
    against a 27,000-position fp16 cache; device-timed like `value` (state
    restored on the device before each step)."""
    dec = capi.Decoder(model, LC_KV + 64, capi.KV_F16, max_new=64)
    dec.fill_synthetic_kv(LC_KV, KV_SEED)
    draft, keep = greedy_draft(None, dec, LC_KV, T_ROWS, seed_tok, model.vocab)
    dec.resume([seed_tok], LC_KV, 64, -1, k_max=15)
    dec.snapshot_save()
    dbuf = _device_ids(dec, np.asarray(draft, dtype=np.int32))
    for _ in range(5):
        dec.snapshot_restore_async()
        dec.spec_step_async(dbuf, len(draft))
    dec.sync()
    dec.event_record(2)
    for _ in range(LC_STEPS):
        dec.snapshot_restore_async()
        dec.spec_step_async(dbuf, len(draft))
    dec.event_record(3)
    ms = dec.event_elapsed_ms(2, 3) / LC_STEPS
    _, c = dec.read_ids()
    dec.close()
    assert c["accepted"] == keep, c
    peak, _ = measured_peaks()
    b = step_bytes(LC_KV, T_ROWS)
    return {"workload": f"configs[3] context: KV {LC_KV} fp16 synthetic, k+1=8, draft matches {keep}",
            "ms_per_step": round(ms, 4), "tokens_per_s": round((c["accepted"] + 1) / (ms / 1e3), 1),
            "accepted_per_step": c["accepted"], "algorithmic_bytes": b,
            "achieved_gbs": round(b / (ms / 1e3) / 1e9, 1), "frac": round(b / (ms / 1e3) / 1e9 / peak, 4)}


def multi_stream(model, capi, fixture) -> dict:
    """configs[4] on one GPU, a bounded sample: MS_STREAMS recordings decoded
    MS_STEPS verify steps each, (a) one recording at a time (one persistent
    launch per recording per step) and (b) as one group (one launch per step for
    all of them: cross-stream batching; the rows beyond 16 are cut in stream
    order).  Host wall clock around the public calls (mtb_spec_run_group), ids
    read back; the accepted ids of (a) and (b) are identical by construction
    and checked here."""
    V = model.vocab
    ds = []
    for i in range(MS_STREAMS):
        d = capi.Decoder(model, MS_KV + 512, capi.KV_F16, max_new=512)
        d.fill_synthetic_kv(MS_KV, 2000 + i)
        ds.append(d)
    hist = [fixture.lcg_ids(32, V, seed=300 + i).tolist() for i in range(MS_STREAMS)]

    def start():
        for d, h in zip(ds, hist):
            d.resume(h, MS_KV, 512, -1, k_max=8, n_min=3, n_max=3)

    def run(groups):
        start()
        t0 = time.perf_counter()
        for g in groups:
            capi.spec_run_group(g, MS_STEPS)
        dt = time.perf_counter() - t0
        out = [d.read_ids() for d in ds]
        toks = sum(len(ids) - len(h) for (ids, _), h in zip(out, hist))
        rows = sum(c["target_input_tokens"] for _, c in out)
        acc = sum(c["accepted"] for _, c in out)
        return dt, toks, rows, acc, [ids for ids, _ in out]

    run([[d] for d in ds])  # warm-up
    s_dt, s_toks, s_rows, s_acc, s_ids = run([[d] for d in ds])
    run([ds])
    g_dt, g_toks, g_rows, g_acc, g_ids = run([ds])
    for d in ds:
        d.close()
    assert g_ids == s_ids, "group decode differs from single-stream decode"

    return {"workload": f"configs[4] sample: {MS_STREAMS} recordings, KV {MS_KV} fp16 synthetic each, "
                        f"{MS_STEPS} verify steps each, device n-gram draft k=8",
            "single_stream": {"tokens_per_s": round(s_toks / s_dt, 1), "ms_per_launch": round(s_dt * 1e3 / (MS_STREAMS * MS_STEPS), 3),
                              "tokens": s_toks, "rows": s_rows, "accepted": s_acc},
            "grouped": {"tokens_per_s": round(g_toks / g_dt, 1), "ms_per_launch": round(g_dt * 1e3 / MS_STEPS, 3),
                        "tokens": g_toks, "rows": g_rows, "accepted": g_acc},
            "speedup": round((g_toks / g_dt) / (s_toks / s_dt), 3),
            "timing": "host wall clock around mtb_spec_run_group, ids read back; same ids in both modes"}


def f16_recording(capi, fixture, device: int) -> dict:
    """configs[2] end to end on one GPU: the F16-weight decoder (random-init
    N(0, 0.02) like configs[1], stored F16), a 132 s recording's prompt (64
    prompt tokens, then per chunk a time-marker token and 375 audio rows N(0, 1))
    fused on the device, prefilled, and 1024 tokens decoded with the device
    n-gram draft (k = 8) into an fp16 KV cache, all through the public
    mtb_spec_generate_ids call: host ids and audio rows in, ids out."""
    shape = fixture.QWEN3_0_6B
    path = fixture.cached_fixture(shape, seed=0, dtype="f16")
    model = capi.Model(path, device)
    rng = np.random.default_rng(132)
    ids = list(fixture.lcg_ids(F16_PROMPT_TOKENS, shape.vocab, seed=77))
    markers = fixture.lcg_ids(F16_CHUNKS, shape.vocab, seed=78)
    for c in range(F16_CHUNKS):
        ids.append(int(markers[c]))
        ids.extend([shape.audio_token_id] * 375)
    ids = np.asarray(ids, dtype=np.int32)
    audio = rng.standard_normal((F16_CHUNKS * 375, shape.hidden)).astype(np.float32)
    dec = capi.Decoder(model, len(ids) + F16_NEW + 64, capi.KV_F16, max_new=F16_NEW)
    dec.spec_generate_ids(ids, audio, shape.audio_token_id, 64, -1, k_max=8)  # warm-up (graphs)
    dec.rewind(0)
    t0 = time.perf_counter()
    out, c = dec.spec_generate_ids(ids, audio, shape.audio_token_id, F16_NEW, -1, k_max=8)
    dt = time.perf_counter() - t0
    dec.close()
    model.close()
    return {"workload": f"configs[2]: F16 weights, fp16 KV, {len(ids)} prompt rows ({F16_CHUNKS * 375} audio), "
                        f"{F16_NEW} tokens, device n-gram draft k=8, one recording",
            "tokens_per_s": round(len(out) / dt, 1), "s": round(dt, 3), "tokens": len(out),
            "target_calls": c["target_calls"], "accepted": c["accepted"],
            "path": "F16 GEMV kernels (multi-kernel verify step); the persistent kernel and tcgen05 prefill are q8_0",
            "timing": "host wall clock around mtb_spec_generate_ids (fuse + prefill + decode), ids read back"}


def _device_ids(dec, arr: np.ndarray) -> int:
    """Device buffer holding `arr` (int32), allocated with torch (plumbing)."""
    import torch
    t = torch.from_numpy(arr.copy()).to(f"cuda:{dec.model.device}")
    torch.cuda.synchronize()
    _KEEP.append(t)
    return t.data_ptr()


_KEEP = []

if __name__ == "__main__":
    main()
