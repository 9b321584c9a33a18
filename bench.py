#!/usr/bin/env python
"""Throughput of the B200 batch-transcription compute layer: audio-seconds per second.

Workload: 512 synthetic utterances with lengths U[1, 13] s rescaled to
3600 s in total, the 40-layer int8 model (random init, reference shapes), whole-utterance windows
(every utterance is <= 2000 frames, src/stream.rs:159-161).  Utterances are sharded across the N
GPUs with a length-balanced LPT assignment, one process per GPU, no collective on the data path
(units are independent); the whole 3600 s is split over the ranks ("strong" scaling).

One step = one pass of the hot path over the rank's whole shard (conv frontend, 40 layers,
output layer + argmax) with features already resident in HBM -> `value`.  `e2e` is the same metric
through the public C-ABI call a user makes (wasr_transcribe) with pinned host features in and host
ids out, copies inside the timed region.  The CPU baseline is the oracle port of the reference CPU
path on this host's cores over a bounded sample.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "wechat-asr-gpu_b200")
METRIC = "audio-sec/sec 40-layer int8 ASR @1/2/4/8 B200; int8 GEMM TOPS vs peak"
WORKLOAD = ("config4: 512 utterances U[1,13] s rescaled to 3600 s total; 40-layer int8 model "
            "(D=512, 8 heads, FF=2048, vocab 10502); whole-utterance windows; LPT-sharded by utterance")


def load_pkg():
    name = "wechat_asr_gpu_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    """The CPU restatement of the reference CPU path: only the cpu_baseline / reference leg."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402
    if not os.path.exists(oracle.LIB):
        oracle.build()
    return oracle


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------- workload
def make_workload(pkg, shard, lengths):
    """Synthetic audio of this rank's utterances -> product fbank features.  Also returns the
    wall time of the host fbank calls alone (the shell's stage, reported as its own line)."""
    feats, sils, secs, fb_s, pcms = [], [], 0.0, 0.0, []
    for i in shard:
        pcm = pkg.synth.make_audio(100000 + i, lengths[i])
        t0 = time.perf_counter()
        f, s = pkg.fbank(pcm)
        fb_s += time.perf_counter() - t0
        feats.append(f)
        sils.append(s)
        pcms.append(pcm)
        secs += pcm.size / 16000.0
    return feats, sils, secs, fb_s, pcms


def gpu_fbank_line(pkg, pcms, feats, local, stream, reps=5):
    """The batched GPU fbank (wasr_fbank_device) over this rank's whole PCM, resident in HBM,
    timed with CUDA events on the launching stream; plus its agreement with the host fbank."""
    import torch
    L = pkg.abi.load()
    dev = f"cuda:{local}"
    soff = np.concatenate([[0], np.cumsum([p.size for p in pcms])]).astype(np.int64)
    nfr = [f.shape[0] for f in feats]
    foff = np.concatenate([[0], np.cumsum(nfr)]).astype(np.int64)
    frames, n = int(foff[-1]), len(pcms)
    pcm_d = torch.from_numpy(np.concatenate(pcms).astype(np.int16)).to(dev)
    soff_d, foff_d = torch.from_numpy(soff).to(dev), torch.from_numpy(foff).to(dev)
    raw = torch.empty((max(frames, 1), 40), dtype=torch.float64, device=dev)
    out = torch.empty((max(frames, 1), 40), dtype=torch.float32, device=dev)
    sil = torch.empty((n, 40), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    def run():
        return L.wasr_fbank_device(pcm_d.data_ptr(), soff_d.data_ptr(), foff_d.data_ptr(), n, frames, raw.data_ptr(),
                                   out.data_ptr(), sil.data_ptr(), stream.cuda_stream)
    for _ in range(2):
        rc = run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        rc = run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    ref = np.concatenate(feats, 0).view(np.int32)
    got = out[:frames].cpu().numpy().view(np.int32)
    same = float(np.mean(got == ref)) if frames else 1.0
    secs = float(sum(p.size for p in pcms)) / 16000.0
    return {"value": round(secs / (ms / 1e3), 1), "unit": "audio-s/s", "rc": int(rc), "ms": round(ms, 3),
            "frames": frames, "identical_to_host": same, "impl": "wasr_fbank_device (f64 FFT512 per frame block)"}


def algorithmic_work(t1_list, n_layers=40, vocab=10502):
    """Per-class algorithmic work of one forward (unpadded shapes).  int8 ops count 2 per MAC;
    bytes for the memory-bound classes are the minimum reads + writes of each kernel."""
    rows = float(sum(t1_list))
    sq = float(sum(t * t for t in t1_list))
    D, FF, FLAT = 512, 2048, 3840
    ops = {
        "gemm_lin": 2 * rows * FLAT * D,
        "gemm_qkv": n_layers * 2 * rows * D * 3 * D,
        "gemm_o": n_layers * 2 * rows * D * D,
        "gemm_f1": n_layers * 2 * rows * D * FF,
        "gemm_f2": n_layers * 2 * rows * FF * D,
        "gemm_out_argmax": 2 * rows * D * vocab,
    }
    # bytes: attention reads q,k,v (fp32) once and writes the output; LN reads h, writes int8 + scale;
    # conv2 reads y1 rows once and writes y2; conv3 (with its quantisation fused) reads y2 and
    # writes int8 rows + scales; GELU + quant reads the FF1 output and writes int8 + scale (the
    # two-kernel path; the engine fuses it into the f1 GEMM where the shapes allow); quant
    # (attention output, final h) reads fp32 rows and writes int8
    byts = {
        "attention": n_layers * rows * (3 * D * 4 + D * 4),
        "layernorm": 2 * n_layers * rows * (D * 4 + D + 4),
        "conv2": rows * (5 * 32 * 40 * 4 + 64 * 41 * 4),
        "conv3": rows * (64 * 41 * 4 + FLAT + 4),
        "conv1": rows * 5 * (40 * 4 + 32 * 40 * 4),
        "gelu_quant": n_layers * rows * (FF * 4 + FF + 4),
        "quant": rows * ((n_layers * D + D) * 5),
    }
    flops = {"attention": n_layers * 4.0 * sq * D}
    # exactly rounded fp32 multiply-adds (one FMUL + one FADD each on the CUDA-core pipe): the
    # bound of the kernels that must reproduce the CPU's sequential float sums
    macs = {
        "attention": n_layers * sq * 8 * 64 * 2,      # QK^T and PV, 8 heads of 64
        "conv2": rows * 64 * 40 * 32 * 49,
    }
    # fused multiply-adds (one fp32 lane-op each): conv3 sums its products in any order and
    # certifies the quantised result against the reference order
    fmas = {"conv3": rows * 192 * 20 * 64 * 9}
    return ops, byts, flops, rows, macs, fmas


# ---------------------------------------------------------------- int8 GEMM probe
def gemm_probe(pkg, local, stream, peak_tops, M=16384, N=2048, K=2048, reps=20):
    """The tcgen05 int8 GEMM alone on a compute-bound shape (int32 accumulators out, through
    wp_gemm_i32), timed with CUDA events on the launching stream: the "int8 GEMM TOPS vs
    peak" half of the metric.  A 256-row slice is checked against an int64 matmul."""
    import torch
    L = pkg.abi.load()
    rng = np.random.default_rng(7)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    blob = np.ascontiguousarray(w).view(np.uint8).reshape(-1).copy()
    ctx = L.wp_create(blob.ctypes.data, blob.size)
    if not ctx:
        return {"error": "wp_create failed"}
    try:
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=f"cuda:{local}")
        out = torch.empty((M, N), dtype=torch.int32, device=f"cuda:{local}")
        torch.cuda.synchronize()  # the operands were made on the default stream
        L.wp_set_stream(ctx, stream.cuda_stream)
        for _ in range(3):
            L.wp_gemm_i32(ctx, a.data_ptr(), M, K, 0, N, stream.cuda_stream, out.data_ptr())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            rc = L.wp_gemm_i32(ctx, a.data_ptr(), M, K, 0, N, stream.cuda_stream, out.data_ptr())
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        ref = a[:256].cpu().numpy().astype(np.int64) @ w.astype(np.int64).T
        exact = bool(np.array_equal(out[:256].cpu().numpy(), ref.astype(np.int32)))
        tops = 2.0 * M * N * K / (ms / 1e3) / 1e12
        return {"M": M, "N": N, "K": K, "epilogue": "int32 accumulators", "rc": int(rc), "ms": round(ms, 4),
                "tops": round(tops, 1), "peak": round(peak_tops, 1), "frac": round(tops / peak_tops, 4),
                "exact_slice": exact, "unit": "TOPS"}
    finally:
        L.wp_destroy(ctx)


def int8_peak(pkg, local, stream, iters=2048, reps=5):
    """Dense int8 tensor-core rate of this GPU, measured: wasr_i8_mma_peak issues back-to-back
    tcgen05.mma kind::i8 (M 128, N 256, K 32) from shared memory on every SM with no loads;
    CUDA events on the launching stream around `reps` launches after a warm-up."""
    import torch
    L = pkg.abi.load()
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    err = torch.zeros(1, dtype=torch.int32, device=f"cuda:{local}")
    torch.cuda.synchronize()
    rc = L.wasr_i8_mma_peak(iters, sms, err.data_ptr(), stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        rc |= L.wasr_i8_mma_peak(iters, sms, err.data_ptr(), stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    ops = float(sms) * iters * 4 * 2 * 128 * 256 * 32
    return {"tops": round(ops / (ms / 1e3) / 1e12, 1), "ms": round(ms, 4), "rc": int(rc), "wait_error": int(err.item()),
            "how": f"{sms} CTAs x {iters} x 4 tcgen05.mma kind::i8 M128 N256 K32 from shared memory, no loads"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev = dev
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out = ""
        rows = []
        for ln in out.splitlines():
            f = [x.strip() for x in ln.split(",")]
            if len(f) >= 8:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        pw = [num(r[2]) for r in rows if num(r[2]) is not None]
        load = [num(r[0]) for r in rows if num(r[2]) is not None and num(r[2]) > 0.5 * max(pw or [0])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(load or sm)) if (load or sm) else None,
                "sm_max_mhz": num(rows[0][1]), "power_w_max": max(pw) if pw else None,
                "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_baseline(orc, pkg, lengths, budget_s: float):
    """Oracle transcription of config-4 utterances in order until `budget_s` of CPU time spent in
    the transcription calls (audio synthesis and fbank excluded); returns (audio-s/s, sample, cores)."""
    blob, plan = pkg.synth.make_model(seed=1, n_layers=40)
    cores = os.cpu_count() or 1
    orc.set_threads(cores)
    done_s, n, spent, ids = 0.0, 0, 0.0, []
    while spent < budget_s and n < len(lengths):
        pcm = pkg.synth.make_audio(100000 + n, lengths[n])
        f, s = orc.fbank(pcm)
        ts = time.perf_counter()
        ref, _ = orc.transcribe(blob, plan, f, s, blk=1600)
        spent += time.perf_counter() - ts
        ids.append(ref)
        done_s += pcm.size / 16000.0
        n += 1
    return (done_s / spent, f"first {n} config-4 utterances ({done_s:.1f} s of audio), {spent:.1f} s CPU wall", cores,
            ids)


def run_reference(args, rank):
    """--impl reference: the reference CPU path (oracle port, no Rust toolchain here) on this
    host's cores, same metric; rank 0 only."""
    if rank != 0:
        return
    pkg = load_pkg()
    orc = load_oracle()
    lengths = pkg.synth.config_lengths(4)
    blob, plan = pkg.synth.make_model(seed=1, n_layers=40)
    cores = os.cpu_count() or 1
    orc.set_threads(cores)
    # each step transcribes the same bounded sample with config 4's length distribution: the
    # utterances at 12 evenly spaced quantiles of the length (about 84 s of audio)
    order = sorted(range(len(lengths)), key=lambda i: lengths[i])
    sample = sorted({order[int((k + 0.5) * len(order) / 12)] for k in range(12)})
    data = []
    for i in sample:
        pcm = pkg.synth.make_audio(100000 + i, lengths[i])
        f, s = orc.fbank(pcm)
        data.append((f, s, pcm.size / 16000.0))
    audio = sum(d[2] for d in data)

    def step():
        t = time.perf_counter()
        for f, s, _ in data:
            orc.transcribe(blob, plan, f, s, blk=1600)
        return time.perf_counter() - t
    for _ in range(args.warmup):
        step()
    ts = [step() for _ in range(args.steps)]
    sec = float(np.mean(ts))
    val = audio / sec
    line = {"metric": METRIC, "value": round(val, 3), "unit": "audio-s/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD,
                       "sample": f"{len(sample)} utterances at evenly spaced length quantiles, {audio:.2f} s of audio per step"},
            "cpu_baseline": {"value": round(val, 3), "unit": "audio-s/s", "cores": cores, "kind": "port",
                             "sample": f"oracle restatement of src/kernels.rs + src/model.rs CPU path, "
                                       f"{len(sample)} utterances / {audio:.2f} s audio per step"},
            "e2e": {"value": round(val, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def stream_line(pkg, eng, utts=3, seconds=20.0, chunk_s=0.1, partial_every=5):
    """The streaming path (src/stream.rs) on the GPU engine: each utterance is fed in chunk_s
    pieces as audio would arrive, partial() every partial_every pushes (a UI refresh), finish()
    at the end; one window per decode through the 40-layer model, graphs off as Stream::new sets
    them below 20000 frames.  Host wall-clock per call (fbank, copy in, forward, copy out, text):
    the latency a user sees.  Also the host text output (Model::text + tidy) of the e2e ids."""
    st = pkg.stream
    vocab = ["<blank>"] + [f"t{i}" for i in range(1, 10502)]
    chunk = int(round(chunk_s * 16000))
    part, commit, fin = [], [], []
    windows, busy, audio = 0, 0.0, 0.0
    for u in range(utts + 1):  # the first utterance warms up and is not counted
        pcm = pkg.synth.make_audio(1000 + u, seconds)
        s = st.Stream(eng, vocab)
        t_u = time.perf_counter()
        for k, a in enumerate(range(0, pcm.size, chunk)):
            s0 = s.s
            t0 = time.perf_counter()
            s.push(pcm[a:a + chunk])
            if s.s != s0 and u:
                commit.append(time.perf_counter() - t0)
            if k % partial_every == partial_every - 1:
                t0 = time.perf_counter()
                s.partial()
                if u:
                    part.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        s.finish()
        if u:
            fin.append(time.perf_counter() - t0)
            busy += time.perf_counter() - t_u
            audio += pcm.size / 16000.0
            windows += s.n_windows
        s.fb.close()
    eng.set_graphs(True)
    ms = lambda v, q: round(float(np.quantile(np.asarray(v), q)) * 1e3, 3) if v else None  # noqa: E731
    return {"partial_ms_p50": ms(part, 0.5), "partial_ms_p99": ms(part, 0.99), "commit_ms_p50": ms(commit, 0.5),
            "finish_ms_p50": ms(fin, 0.5), "windows": windows, "partials": len(part),
            "rtf": round(busy / audio, 5) if audio else None, "utterances": utts, "seconds_each": seconds,
            "chunk_s": chunk_s, "partial_every_s": round(chunk_s * partial_every, 3),
            "cfg": "prev 200 / blk 400 / post 100 frames + 50 silence, 40 layers, one stream"}


def text_line(pkg, ids_list):
    """Host text output (Model::text + tidy) of every utterance's ids, placeholder vocabulary."""
    st = pkg.stream
    vocab = ["<blank>"] + [f"t{i}" for i in range(1, 10502)]
    t0 = time.perf_counter()
    n_chars = sum(len(st.tidy(st.text(ids, vocab))) for ids in ids_list)
    dt = time.perf_counter() - t0
    return {"utterances": len(ids_list), "ms": round(dt * 1e3, 3), "chars": n_chars,
            "impl": "Python restatement of Model::text + tidy (src/model.rs:620-642, src/stream.rs:203-210)"}


def gather_and_check(pkg, eng, blob, plan, lengths, shard, local_ids, rank, world, local):
    """After the timed steps: each rank hands its shard's ids (from the e2e run) to the node
    driver, which gathers every utterance on rank 0 through the rendezvous store, re-queueing
    the shard of a rank that does not deliver.  Rank 0 then transcribes all utterances on its
    one GPU and counts the utterances whose gathered ids are identical."""
    import torch.distributed as dist
    store = dist.distributed_c10d._get_default_store()

    def features(idx):
        fs = [pkg.fbank(pkg.synth.make_audio(100000 + i, lengths[i])) for i in idx]
        return [f for f, _ in fs], [x for _, x in fs]

    def transcribe(idx):  # this rank's own shard comes from the e2e run; a re-queued one is redone
        if all(i in local_ids for i in idx):
            return [local_ids[i] for i in idx]
        f, x = features(idx)
        return eng.transcribe(f, x, blk=1600)

    t0 = time.perf_counter()
    allids = pkg.dist.run_sharded(transcribe, lengths, rank, world, store, timeout_s=120.0, tag="bench_gather")
    gather_ms = (time.perf_counter() - t0) * 1e3
    if rank != 0:
        return None
    f, x = features(range(len(lengths)))
    rows = sum((a.shape[0] - 5) // 5 + 1 for a in f if a.shape[0] >= 5)
    one = pkg.Engine(blob, plan, device=local, max_rows=max(rows, 1024))
    try:
        ref = one.transcribe(f, x, blk=1600)
    finally:
        one.close()
    same = sum(bool(np.array_equal(a, b)) for a, b in zip(allids, ref))
    return {"utterances": len(ref), "ids_identical_to_one_gpu": int(same), "gather_ms": round(gather_ms, 3),
            "failed_ranks": list(pkg.dist.run_sharded.last_failed),
            "how": "dist.run_sharded: per-rank ids through the rendezvous store to rank 0; "
                   "reference = all utterances transcribed on rank 0's GPU alone"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--max-rows", type=int, default=0,
                    help="rows per engine chunk (0 = this rank's whole shard in one chunk)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gemm-probe", action="store_true")
    ap.add_argument("--no-stream", action="store_true")
    ap.add_argument("--utts", type=int, default=0,
                    help="profiling aid: only the first N config-4 utterances (0 = all 512)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "b200" else args.warmup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import datetime

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dist_on = world > 1
    if dist_on:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    pkg = load_pkg()
    lengths = pkg.synth.config_lengths(4)
    if args.utts:
        lengths = lengths[:args.utts]
    shards = pkg.synth.lpt_shards(lengths, world)
    shard = shards[rank]
    feats, sils, my_audio, fbank_s, pcms = make_workload(pkg, shard, lengths)
    total_audio = float(sum(lengths))
    blob, plan = pkg.synth.make_model(seed=1, n_layers=40)
    t = np.array([f.shape[0] for f in feats], np.int32)
    t1 = [(x - 5) // 5 + 1 if x >= 5 else 0 for x in t]
    # one chunk holds the whole shard by default (the activations of 72K rows take ~5 GB): every
    # launch then has its full width and no short last chunk
    args.max_rows = args.max_rows if args.max_rows > 0 else max(int(sum(t1)), 1024)
    eng = pkg.Engine(blob, plan, device=local, max_rows=args.max_rows)
    stream = torch.cuda.Stream(device=local)
    eng.set_stream(stream.cuda_stream)

    cat = np.ascontiguousarray(np.concatenate(feats, 0), np.float32)
    feats_dev = torch.from_numpy(cat).to(f"cuda:{local}")
    ids_dev = torch.empty(max(sum(t1), 1), dtype=torch.int32, device=f"cuda:{local}")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=f"cuda:{local}")
    eng.set_profile(False)  # timed steps run the plain graphs; the per-kernel split comes after

    def fwd():
        eng.forward_device(feats_dev.data_ptr(), t, ids_dev.data_ptr(), sync=False)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            fwd()
        torch.cuda.synchronize()
        if dist_on:
            dist.barrier()
        torch.cuda.synchronize()
        clk = ClockSampler(local)
        clk.start()
        launches0 = eng.kernel_launches()
        evs = []
        for _ in range(args.steps):
            flush.zero_()                       # L2 flush (256 MiB write) outside the timed events
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fwd()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        launches = eng.kernel_launches() - launches0
        clocks = clk.stop()
        ms = sum(a.elapsed_time(b) for a, b in evs)
        if dist_on:
            dist.barrier()
        # per-kernel split: the same forward with an event recorded around every kernel (graphs
        # recaptured with the event nodes; the second run is a replay), after the timed steps
        eng.set_profile(True)
        for _ in range(2):
            flush.zero_()
            fwd()
        torch.cuda.synchronize()
    err = eng.error()
    prof_ms, prof_n = eng.profile()
    eng.set_profile(False)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{local}")
    if dist_on:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    ms_per_step = ms_max / args.steps
    value = total_audio / (ms_per_step / 1e3)

    # ---- e2e through the public call with host buffers (pinned), copies inside the timing
    e2e, e2e_ids = None, None
    if not args.no_e2e:
        pinned = torch.from_numpy(cat).pin_memory()
        cat_pinned = pinned.numpy()
        eng.set_stream(None)  # the engine's own stream; wasr_transcribe synchronises it
        eng.transcribe(feats, sils, blk=1600, feats_cat=cat_pinned)  # warm (captures the graphs)
        torch.cuda.synchronize()
        if dist_on:
            dist.barrier()
        e_ts = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            out = eng.transcribe(feats, sils, blk=1600, feats_cat=cat_pinned)
            e_ts.append(time.perf_counter() - t0)
        e_t = torch.tensor([float(np.mean(e_ts))], dtype=torch.float64, device=f"cuda:{local}")
        if dist_on:
            dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
        ids_bytes = 4 * sum(len(o) for o in out)
        local_ids = dict(zip(shard, out))
        e2e_ids = out if world == 1 else None  # rank 0 of one rank holds every utterance, in order
        e2e = {"value": round(total_audio / float(e_t.item()), 3), "unit": "audio-s/s",
               "h2d_bytes_per_step": int(cat.nbytes), "d2h_bytes_per_step": int(ids_bytes),
               "api": "wasr_transcribe (pinned host features in, host ids out)"}

    # ---- N > 1: every rank's ids gathered on rank 0 through the rendezvous store (the node
    # driver dist.run_sharded, src/bin/wasr.rs:147-169 collects per file), checked against one GPU
    gather = None
    if dist_on and e2e is not None:
        gather = gather_and_check(pkg, eng, blob, plan, lengths, shard, local_ids, rank, world, local)

    # ---- roofline of the dominant kernel class (last timed step, CUDA events on its stream)
    hbm, bf16, src = peaks()
    i8 = int8_peak(pkg, local, stream)
    i8_peak = i8["tops"] if i8["rc"] == 0 and i8["wait_error"] == 0 else 2 * bf16
    names = pkg.abi.KERNEL_CLASSES
    ops, byts, flops, rows, macs, fmas = algorithmic_work(t1, plan.n_layers)
    dom = max(range(len(names)), key=lambda i: prof_ms[i])
    dname = names[dom]
    dms = prof_ms[dom]
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic_per_row.json")
    if os.path.exists(tf):
        tr = json.load(open(tf)).get(dname)
        # units of the class per step: rows (frontend, lin), rows x layers, or 2 LayerNorms per layer
        per_layer = 2 * plan.n_layers if dname == "layernorm" else (
            1 if dname in ("conv1", "conv2", "conv3", "gemm_lin", "gemm_out_argmax") else plan.n_layers)
        if tr and prof_n[dom]:
            traffic = round(tr * rows * per_layer / prof_n[dom])
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    peak_mac = sms * 128 * mhz * 1e6 / 2 / 1e12
    mac_basis = (f"{sms} SMs x 128 fp32 lanes x {mhz:.0f} MHz / 2 ops per exactly rounded MAC (packed and "
                 f"scalar fp32 ops both measured at 127 lane-ops/clk/SM)")
    if dname in ops:
        ach = ops[dname] / prof_n[dom] / (dms / prof_n[dom] / 1e3) / 1e12
        roof = {"kernel": dname, "bound": "tensor", "achieved": round(ach, 2), "peak": round(i8_peak, 1),
                "unit": "TOPS", "frac": round(ach / i8_peak, 4), "traffic": traffic,
                "peak_source": "measured int8 dense (int8_peak)",
                "launches": int(prof_n[dom]), "avg_launch_us": round(dms / prof_n[dom] * 1e3, 2)}
    elif dname in macs and prof_n[dom]:
        # the exact-arithmetic kernels (attention, conv2, conv3) are bound by the CUDA-core fp32
        # pipe: every MAC is a rounded multiply then a rounded add, in the CPU's order
        ach_mac = macs[dname] / (dms / 1e3) / 1e12
        b = byts.get(dname, 0.0)
        roof = {"kernel": dname, "bound": "fp32", "achieved": round(ach_mac, 3), "peak": round(peak_mac, 2),
                "unit": "TMAC/s", "frac": round(ach_mac / peak_mac, 4), "traffic": traffic,
                "peak_source": mac_basis, "launches": int(prof_n[dom]),
                "avg_launch_us": round(dms / prof_n[dom] * 1e3, 2),
                "hbm": {"achieved": round(b / (dms / 1e3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(b / (dms / 1e3) / 1e9 / hbm, 4), "peak_source": f"{src} hbm_gbs"}}
    else:
        b = byts.get(dname, 0.0)
        ach = b / prof_n[dom] / (dms / prof_n[dom] / 1e3) / 1e9 if prof_n[dom] else 0.0
        roof = {"kernel": dname, "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(ach / hbm, 4), "traffic": traffic, "peak_source": f"{src} hbm_gbs",
                "launches": int(prof_n[dom]), "avg_launch_us": round(dms / prof_n[dom] * 1e3, 2)}
    gemm_ops = sum(ops.values())
    gemm_ms = sum(prof_ms[names.index(k)] for k in ops)
    roof["all_gemms_tops"] = round(gemm_ops / (gemm_ms / 1e3) / 1e12, 2) if gemm_ms else None
    # every int8 GEMM of the model at its real shape (M = this rank's rows) and epilogue, against
    # the measured int8 peak (BASELINE's target: >= 60 % of dense int8 peak at M >= 1600)
    roof["int8_peak"] = i8
    roof["gemms"] = {k: {"tops": round(ops[k] / (prof_ms[names.index(k)] / 1e3) / 1e12, 1),
                         "frac": round(ops[k] / (prof_ms[names.index(k)] / 1e3) / 1e12 / i8_peak, 4),
                         "ms": round(prof_ms[names.index(k)], 3), "M": int(rows)}
                     for k in ops if prof_ms[names.index(k)] > 0}
    if prof_n[names.index("gelu_quant")] == 0 and prof_ms[names.index("gemm_f1")] > 0:
        # the engine's fused f1 kernel (f1 + GELU + row quantisation, two MMA passes per row
        # block): its ops count the GEMM once, its time includes the GELU and the quantisation
        roof["gemms"]["gemm_f1"]["fused"] = "gelu + row quant (gemm_i8_gelu_q)"
    roof["exact_fp32"] = {k: {"tmac_s": round(macs[k] / (prof_ms[names.index(k)] / 1e3) / 1e12, 3),
                              "frac": round(macs[k] / (prof_ms[names.index(k)] / 1e3) / 1e12 / peak_mac, 4),
                              "ms": round(prof_ms[names.index(k)], 3)}
                          for k in macs if prof_ms[names.index(k)] > 0}
    peak_fma = 2 * peak_mac  # one lane-op per fused multiply-add
    roof["fma_fp32"] = {k: {"tfma_s": round(fmas[k] / (prof_ms[names.index(k)] / 1e3) / 1e12, 3),
                            "frac": round(fmas[k] / (prof_ms[names.index(k)] / 1e3) / 1e12 / peak_fma, 4),
                            "peak": round(peak_fma, 2), "ms": round(prof_ms[names.index(k)], 3)}
                        for k in fmas if prof_ms[names.index(k)] > 0}
    roof["hbm_classes"] = {k: {"gbs": round(byts[k] / (prof_ms[names.index(k)] / 1e3) / 1e9, 1),
                               "frac": round(byts[k] / (prof_ms[names.index(k)] / 1e3) / 1e9 / hbm, 4),
                               "ms": round(prof_ms[names.index(k)], 3)}
                           for k in ("gelu_quant", "layernorm", "quant") if k in byts and prof_ms[names.index(k)] > 0}
    roof["kernel_ms_last_step"] = {names[i]: round(prof_ms[i], 3) for i in range(len(names)) if prof_n[i]}

    gprobe = gemm_probe(pkg, local, stream, i8_peak) if (rank == 0 and not args.no_gemm_probe) else None
    fbg = gpu_fbank_line(pkg, pcms, feats, local, stream) if (rank == 0 and not args.no_gemm_probe) else None

    # single-stream latency does not depend on N: measured at N = 1 only
    strm = stream_line(pkg, eng) if (world == 1 and not args.no_stream) else None
    txt = text_line(pkg, e2e_ids) if (world == 1 and e2e_ids is not None and not args.no_stream) else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        orc = load_oracle()
        v, sample, cores, ref_ids = cpu_baseline(orc, pkg, lengths, args.cpu_budget)
        cpu = {"value": round(v, 3), "unit": "audio-s/s", "cores": cores, "kind": "port", "sample": sample}
        if e2e_ids is not None:
            # the oracle's per-frame ids of the sample against the GPU's from the e2e run
            same = [np.array_equal(np.asarray(g, np.uint32), np.asarray(r, np.uint32))
                    for g, r in zip(e2e_ids, ref_ids)]
            cpu["parity"] = {"utterances": len(same), "ids_identical": int(sum(same))}

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic",
                "config": {"workload": WORKLOAD, "total_audio_s": round(total_audio, 3), "utterances": len(lengths),
                           "rows_rank0": int(sum(t1)), "n_layers": plan.n_layers, "max_rows_per_chunk": args.max_rows,
                           "l2": "flushed (256 MiB write) before every timed step",
                           "parallelism": f"utterance-sharded LPT over {world} GPU(s), no collective"},
                "roofline": roof, "gemm_probe": gprobe, "cpu_baseline": cpu, "e2e": e2e, "gather": gather,
                "fbank_host": {"value": round(my_audio / fbank_s, 1) if fbank_s > 0 else None, "unit": "audio-s/s",
                               "threads": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())),
                               "scope": "rank 0's utterances, one call per utterance",
                               "impl": "host C++ f64 FFT512 + CMS (src/fbank.rs), OpenMP over frames"},
                "fbank_gpu": fbg,
                "stream": strm, "text_host": txt,
                "gpu_launches": int(launches),
                "clocks": clocks, "device_error": err}
        print(json.dumps(line), flush=True)
    eng.close()
    if dist_on:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
