#!/usr/bin/env python3
"""Frame-decode benchmark: the navi-tts per-frame hot path on B200.

One step = one 12.5 Hz frame at batch 1: the 28-layer talker decode step at KV length L
(configs[1]) + codebook-0 sampling + the 15-step code predictor with top-k 50 / top-p 0.9
/ temperature 0.9 on the Philox stream + the next step embedding, i.e. one
launch of the persistent frame kernel.  The metric is box frames/s (1000 / ms per frame
per GPU, summed over GPUs); every GPU decodes its own independent stream (request-parallel
replicas, no inter-GPU traffic), so scaling is weak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--kv L] [--impl ours|reference]

`value`  device time of K back-to-back frames (CUDA events on the engine stream; weights and
         KV already in HBM; per-frame working set ~1.1 GB, larger than the 126 MB L2).
`e2e`    the same frames through the public C ABI, synchronous per frame, with the trailing
         text row copied host->device from pinned memory and the 16 codes read back each frame.
`--impl reference` times the CPU oracle (PyTorch fp32 restatement of the reference's math,
         oracle/model.py) on a bounded sample of the same workload on the host's cores: the
         reference's own engine is HIP-only (RDNA3) and cannot run here.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "navi-tts_b200"))
sys.path.insert(0, ROOT)

METRIC = "frames/s, batch-1 frame decode (talker step + 15-step code predictor + sampling)"
BENCH_NAVI = os.environ.get("NAVI_BENCH_NAVI", "/tmp/navi_bench_full.navi")


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def algorithmic_bytes(p, L: int) -> int:
    """HBM bytes one frame must read at KV length L, 15 code-predictor weight passes:
    talker layers + final norm + codec_head, the KV cache rows 0..L of every layer,
    15 x (code-predictor layers + final norm) + 15 lm_heads (one per codebook)."""
    def layers(t):
        H, Q, K, F, D = t.hidden, t.n_head * t.head_dim, t.n_kv_head * t.head_dim, t.ff, t.head_dim
        per = 2 * (Q * H + 2 * K * H + H * Q + 3 * F * H) + 4 * (2 * H + 2 * D)
        return t.n_layer * per
    tl, cp = p.talker, p.cp
    talker = layers(tl) + 4 * tl.hidden + 2 * tl.vocab * tl.hidden
    kv = tl.n_layer * 2 * (L + 1) * tl.n_kv_head * tl.head_dim * 2
    cpb = 15 * (layers(cp) + 4 * cp.hidden) + 15 * 2 * cp.vocab * cp.hidden
    return talker + kv + cpb


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, max clock, throttle reasons)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[0] == str(self.gpu):
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit())
        mx = max(float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.rows), "power_w_max": max(float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit())}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(L: int):
    """dram bytes per frame-kernel launch from the committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "frame_kernel_traffic.json")) as f:
            j = json.load(f)
        return j.get(str(L)) or j.get("default")
    except Exception:
        return None


def ensure_weights(rank: int, world: int):
    from navi_b200 import model_spec
    if rank == 0 and not os.path.exists(BENCH_NAVI):
        model_spec.write_synthetic(BENCH_NAVI, model_spec.full_config(1024))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline(L: int, n_frames: int = 3):
    """The oracle (PyTorch fp32 on the host cores) on a bounded sample of the same frame."""
    import numpy as np
    import torch
    from oracle import model as om
    torch.set_num_threads(os.cpu_count() or 1)
    W = om.Weights.from_navi(BENCH_NAVI)
    tl = W.tl
    kvd = tl.n_kv_head * tl.head_dim
    g = torch.Generator().manual_seed(L)
    kv = [(torch.randn(L + 1, kvd, generator=g).half().float(), torch.randn(L + 1, kvd, generator=g).half().float())
          for _ in range(tl.n_layer)]
    step = torch.randn(tl.hidden, generator=g)
    trailing = torch.randn(tl.hidden, generator=g)
    s = om.Sampling(top_p=0.9, cp_top_p=0.9, rng=1)
    seen = np.zeros(tl.vocab, np.uint8)
    om.frame(W, step_in=step, kv=kv, n_past=L, trailing=trailing, s=s, seed=1, frame_index=0, seen=seen)   # warm-up
    t0 = time.perf_counter()
    for i in range(n_frames):
        out = om.frame(W, step_in=step, kv=kv, n_past=L, trailing=trailing, s=s, seed=1, frame_index=i + 1, seen=seen)
        step = out.step_out
    dt = time.perf_counter() - t0
    return {"value": n_frames / dt, "unit": "frames/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n_frames} full frames (28-layer talker step at KV {L} + 15-step code predictor + sampling), "
                      f"PyTorch fp32 oracle, {torch.get_num_threads()} threads, after 1 warm-up frame"}


LAYER_NAVI = os.environ.get("NAVI_LAYER_NAVI", "/tmp/navi_bench_layer.navi")


def layer_bytes(t, L: int) -> int:
    """HBM bytes of one talker decoder layer step at KV length L: f16 q/k/v/o/gate/up/down
    weights, f32 norm weights (input, post-attention, q, k), and the cached K/V rows
    0..L-1 plus the new row L, f16."""
    H, Q, K, F, D = t.hidden, t.n_head * t.head_dim, t.n_kv_head * t.head_dim, t.ff, t.head_dim
    return 2 * (Q * H + 2 * K * H + H * Q + 3 * F * H) + 4 * (2 * H + 2 * D) + 2 * (L + 1) * K * 2


def layer_bench(dev_ordinal: int, reps: int, warm: int, L: int = 256):
    """one talker decoder layer, one decode step at batch 1, KV length 256, seed-0
    weights, input hidden N(0, 1), cache N(0, 1) f16. Each timed launch follows a 256 MB
    write that flushes L2 (the layer's 32.5 MB would otherwise stay resident); the time is
    the launch's CUDA-event device time (Frame::run_layer), median over `reps`."""
    import numpy as np
    import torch
    from navi_b200 import engine, model_spec
    if not os.path.exists(LAYER_NAVI):
        model_spec.write_synthetic(LAYER_NAVI, model_spec.layer_config(), seed_offset=model_spec.LAYER_SEED_OFFSET)
    dev = engine.Device(dev_ordinal)
    w = engine.Weights(dev, LAYER_NAVI)
    fr = engine.Frame(dev, w)
    t = w.params.talker
    kvd = t.n_kv_head * t.head_dim
    cuda = f"cuda:{dev_ordinal}"
    g = torch.Generator(device=cuda).manual_seed(0)
    k = [torch.randn(L + 8, kvd, generator=g, device=cuda).half()]
    v = [torch.randn(L + 8, kvd, generator=g, device=cuda).half()]
    kv = engine.KvCache.wrap([k[0].data_ptr()], [v[0].data_ptr()], L + 8, kvd, keepalive=(k, v))
    x = torch.randn(t.hidden, generator=g, device=cuda)
    y = torch.empty_like(x)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.ExternalStream(dev.stream, device=cuda)
    us = []
    for i in range(warm + reps):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
        r = fr.run_layer(0, x.data_ptr(), kv, L, y.data_ptr())
        assert r.ok, r.error
        if i >= warm:
            us.append(r.us)
    us_med = float(np.median(us))
    ab = layer_bytes(t, L)
    peak, kind = measured_peak()
    achieved = ab / (us_med * 1e-6) / 1e9
    fr.close()
    w.close()
    dev.close()
    return {"workload": f"configs[0]: one talker decoder layer (hidden {t.hidden}, {t.n_head}/{t.n_kv_head} heads x "
                        f"{t.head_dim}, SwiGLU {t.ff}), KV {L}, batch 1, seed-0 weights",
            "us_per_step": round(us_med, 3), "us_p10": round(float(np.percentile(us, 10)), 3),
            "us_p90": round(float(np.percentile(us, 90)), 3), "launches": reps,
            "l2": "flushed before every launch (256 MB write)",
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "algorithmic_bytes": ab, "peak_kind": kind,
                         "bound_us": round(ab / (peak * 1e9) * 1e6, 3)}}


def batch_bench(frame, p, local: int, steps: int, warm: int, L: int = 512):
    """Batched decode (Frame::enqueue_batch): nb = 1, 2 and 4 streams per launch, each at KV
    length L in its own cache, decoding one frame each per launch; device time of `steps`
    launches back to back (CUDA events on the engine stream), frames/s = nb * launches / time."""
    import torch
    from navi_b200 import engine
    tl = p.talker
    kvd = tl.n_kv_head * tl.head_dim
    cuda = f"cuda:{local}"
    g = torch.Generator(device=cuda).manual_seed(77)
    kvs = []
    for _ in range(4):
        k = [torch.randn(L + 8, kvd, generator=g, device=cuda).half() for _ in range(tl.n_layer)]
        v = [torch.randn(L + 8, kvd, generator=g, device=cuda).half() for _ in range(tl.n_layer)]
        kvs.append(engine.KvCache.wrap([t.data_ptr() for t in k], [t.data_ptr() for t in v], L + 8, kvd, keepalive=(k, v)))
    tr = [torch.randn(tl.hidden, generator=g, device=cuda) for _ in range(4)]
    s = engine.Sampling(temperature=0.9, top_k=50, top_p=0.9, repetition_penalty=1.05, cp_temperature=0.9, cp_top_k=50,
                        cp_top_p=0.9, min_frames=2, rng=1)
    stream = torch.cuda.ExternalStream(frame.dev.stream, device=cuda)
    out = {}
    for nb in (1, 2, 4):
        slots = list(range(nb))
        args = lambda f: (slots, kvs[:nb], [L] * nb, [t.data_ptr() for t in tr[:nb]], s, [101 + i for i in range(nb)], [f] * nb)
        for i in range(nb):
            frame.reset_slot(i)
            frame.set_step_in_slot(i, tr[i].data_ptr())
        for f in range(warm):
            frame.enqueue_batch(*args(f))
        assert all(r.ok for r in frame.collect_batch(nb))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(local)
        e0.record(stream)
        for f in range(steps):
            frame.enqueue_batch(*args(warm + f))
        e1.record(stream)
        res = frame.collect_batch(nb)
        torch.cuda.synchronize(local)
        assert all(r.ok for r in res), res[0].error
        ms = e0.elapsed_time(e1) / steps
        out[str(nb)] = {"ms_per_launch": round(ms, 4), "frames_per_s": round(nb * 1000.0 / ms, 1)}
    return {"workload": f"configs[1]+[2] frames of nb independent streams per launch at KV {L} each (one weight pass)",
            "per_gpu": out}


def vocoder_flops_per_frame(p) -> float:
    """2 x multiply-adds of every GEMM / conv of the decoder per frame (vocoder.hip:261-343)."""
    v = p.vocoder
    L, VH, HD, FF, CD, DD = p.vq_latent, v.hidden, v.n_head * v.head_dim, v.ff, p.vq_codebook_dim, p.decoder_dim
    macs = CD * CD + 3 * CD * L + L * VH + VH * L                       # rvq projection, pre_conv, in / out projection
    macs += v.n_layer * (VH * 3 * HD + HD * VH + VH * 2 * FF + FF * VH)  # pre-transformer
    rows = 1
    for r in p.upsampling_ratios[:2]:
        macs += rows * r * L * L                                         # transposed conv k = s
        rows *= r
        macs += rows * (L * 4 * L * 2)                                   # ConvNeXt pointwise pair
    macs += rows * 7 * L * DD                                            # decoder.0
    w = DD
    for r in p.upsample_rates[:4]:
        ow = w // 2
        macs += rows * r * 2 * w * ow                                    # transposed conv k = 2s
        rows *= r
        macs += rows * 3 * (7 * ow * ow + ow * ow)                       # 3 residual units
        w = ow
    macs += rows * 7 * w                                                 # output conv
    return 2.0 * macs


def vocoder_weight_bytes(w) -> int:
    """f16 bytes of the decoder's GEMM / conv weights (codebooks excluded: rows are gathered)."""
    from navi_b200 import model_spec
    total = 0
    for name, shape in model_spec.tensor_table(model_spec.full_config(w.params.decoder_dim)):
        if name.startswith("codec.decoder.") and len(shape) >= 2 and "_codebook" not in name:
            n = 1
            for d in shape:
                n *= d
            total += 2 * n
    return total


def vocoder_bench(dev, w, reps: int = 20, chunks=(4, 16), warm: int = 3):
    """decode of 4- and 16-frame chunks of uniform random codes (device time of
    Vocoder::decode including the codes / PCM copies, median of reps, after `warm` decodes)."""
    import numpy as np
    from navi_b200 import engine
    p = w.params
    flops = vocoder_flops_per_frame(p)
    wb = vocoder_weight_bytes(w)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tpeak, hpeak = float(peaks.get("bf16_tflops", 1590.0)), float(peaks.get("hbm_gbs", 6650.0))
    rng = np.random.default_rng(3)
    out = {}
    for chunk in chunks:
        voc = engine.Vocoder(dev, w, max_chunk_frames=chunk)
        codes = rng.integers(0, p.vq_codebook_size, (chunk, p.vq_n_q)).astype(np.int32)
        for _ in range(warm):
            voc.decode(codes)
        dev_ms, wall_ms = [], []
        for _ in range(reps):
            t0 = time.perf_counter()
            voc.decode(codes)
            wall_ms.append((time.perf_counter() - t0) * 1000.0)
            dev_ms.append(voc.last_ms)
        ms = float(np.median(dev_ms))
        bound_ms = max(chunk * flops / (tpeak * 1e12), wb / (hpeak * 1e9)) * 1e3
        out[str(chunk)] = {"ms_per_chunk": round(ms, 4), "us_per_frame": round(ms * 1000.0 / chunk, 2),
                           "e2e_ms_per_chunk": round(float(np.median(wall_ms)), 4),
                           "tflops": round(chunk * flops / (ms * 1e-3) / 1e12, 2),
                           "roofline_ms": round(bound_ms, 4), "roofline_frac": round(bound_ms / ms, 4)}
        voc.close()
    return {"workload": "configs[3]: codes [T][16] -> PCM [T*1920], decoder_dim %d, chunks of 4 and 16 frames" % p.decoder_dim,
            "flops_per_frame": flops, "weight_bytes": wb, "chunks": out,
            "roofline_note": "bound = max(FLOPs / measured bf16 peak, weight bytes / measured HBM); the tensor-core "
                             "passes run f16 hi + lo activation halves, so issued MMA work is twice the FLOPs"}


def serving_bench(dev, w, rank: int, world: int, dist, streams: int = 64, frames: int = 400, n_text: int = 200, group: int = 4):
    """configs[4], request-parallel: `streams` synthetic utterances (a 200-id text prompt of
    uniform ids, prefill, `frames` frames, their PCM streamed through the vocoder 4 frames
    first, then 16 at a time) dealt round-robin to the ranks. Each rank runs its streams in
    groups of `group` through the public API (host ids in, host PCM out): Graph::synth_batch,
    whose streams decode their frames together in batched launches (group 1: Graph::synth,
    graph.cpp:52-111, one stream after another). Aggregate frames/s = all frames / the slowest
    rank's wall time; time to first audio is SynthStats::ttfa_ms of every stream, counted from
    the start of its group's call."""
    import numpy as np
    import torch
    from navi_b200 import engine, model_spec
    p = w.params
    cfg = model_spec.full_config(p.decoder_dim)
    g = engine.Graph(dev, w, max_prompt_tokens=1024, max_frames=frames + 8, vocoder_chunk=16, max_streams=group)
    s = engine.Sampling(temperature=0.9, top_k=50, top_p=0.9, repetition_penalty=1.05, cp_temperature=0.9, cp_top_k=50,
                        cp_top_p=0.9, min_frames=frames, rng=1)
    spk = np.random.default_rng(4).standard_normal(p.talker.hidden).astype(np.float32)

    def ids_of(j):
        r = np.random.default_rng(1000 + j)
        return ([cfg.im_start_id, cfg.assistant_id, 198] + r.integers(0, cfg.text_vocab, n_text).tolist()
                + [cfg.im_end_id, 198, cfg.im_start_id, cfg.assistant_id, 198])

    # warm-up: one group of short utterances
    g.synth_batch([(ids_of(-1 - j), spk, 5 + j, 24) for j in range(group)], "english", s, first_batch=4, vocoder_batch=16)
    mine = [j for j in range(streams) if j % world == rank]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    ttfa, rtf, pre, voc_ms, n_frames, pcm_samples = [], [], [], 0.0, 0, 0
    for k in range(0, len(mine), group):
        js = mine[k:k + group]
        for (codes, pcm, st) in g.synth_batch([(ids_of(j), spk, 77 + j, frames) for j in js], "english", s, first_batch=4,
                                              vocoder_batch=16):
            assert st.n_frames == frames and pcm.size == frames * p.codec_upsample
            ttfa.append(st.ttfa_ms)
            rtf.append(st.rtf)
            pre.append(st.prefill_ms)
            voc_ms += st.vocoder_ms
            n_frames += st.n_frames
            pcm_samples += pcm.size
    elapsed = time.perf_counter() - t0
    g.close()
    stats = {"elapsed": elapsed, "frames": n_frames, "ttfa": ttfa, "rtf": rtf, "pre": pre, "voc_ms": voc_ms}
    if dist:
        out = [None] * world
        dist.all_gather_object(out, stats)
    else:
        out = [stats]
    slowest = max(o["elapsed"] for o in out)
    total = sum(o["frames"] for o in out)
    allt = [t for o in out for t in o["ttfa"]]
    return {"workload": f"configs[4]: {streams} streams x ({n_text}-id prompt, prefill, {frames} frames, PCM in batches "
                        f"of 4 then 16), round-robin over {world} GPU(s), on a GPU in groups of {group} decoded together "
                        f"(batched frames)",
            "frames_per_s": round(total / slowest, 2), "ttfa_ms_p50": round(float(np.median(allt)), 3),
            "ttfa_ms_max": round(float(max(allt)), 3),
            "prefill_ms_p50": round(float(np.median([t for o in out for t in o["pre"]])), 3),
            "rtf_p50": round(float(np.median([t for o in out for t in o["rtf"]])), 5),
            "vocoder_ms_per_frame": round(sum(o["voc_ms"] for o in out) / total, 4),
            "streams": streams, "frames_per_stream": frames, "wall_s": round(slowest, 3),
            "timing": "wall clock around Graph::synth calls (host ids in, host PCM out), max over ranks"}


def vocoder_cpu_baseline(n_frames: int = 4):
    """The vocoder oracle (PyTorch fp32 on the host cores) on one chunk of configs[3]."""
    import numpy as np
    import torch
    from oracle import model as om
    from oracle import vocoder as ov
    torch.set_num_threads(os.cpu_count() or 1)
    W = om.Weights.from_navi(BENCH_NAVI)
    codes = np.random.default_rng(3).integers(0, W.cfg.vq_codebook_size, (n_frames, W.cfg.vq_n_q))
    v = ov.Vocoder(W)
    v.decode_chunk(codes)                    # warm-up
    t0 = time.perf_counter()
    v.decode_chunk(codes)
    dt = time.perf_counter() - t0
    return {"value": round(dt * 1000.0 / n_frames, 3), "unit": "ms/frame", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"one {n_frames}-frame chunk, PyTorch fp32 vocoder oracle, after 1 warm-up chunk"}


def run_reference(args):
    rank, local, world = dist_env()
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
    if rank != 0:
        return
    ensure_weights(0, 1)
    n = max(1, min(args.steps, 60))          # about 7 s of CPU time at ~9 frames/s
    cb = cpu_baseline(args.kv, n_frames=n)
    line = {"metric": METRIC, "value": cb["value"], "unit": "frames/s", "n_gpus": args.gpus, "steps": n,
            "steps_requested": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights, random KV)",
            "config": {"workload": f"configs[1]+[2] frame at KV {args.kv}", "kv_len": args.kv, "batch": 1},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def combine_ranks(ms: float, e2e_ms: float, world: int, dist, device: str):
    """Whole-job numbers of N request-parallel replicas: every rank decodes the same number
    of frames, so the job takes as long as its slowest rank (max over ranks of the per-frame
    times) and processes world frames per step. Returns (ms, e2e_ms, frames/s, e2e frames/s)."""
    import torch
    t = torch.tensor([ms, e2e_ms], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    return ms, e2e_ms, world * 1000.0 / ms, world * 1000.0 / e2e_ms


def run_vocoder_only(args):
    """`--vocoder-only`: the configs[3] measurement alone (one GPU), one JSON line."""
    import torch
    rank, local, world = dist_env()
    if world > 1 and rank != 0:
        return
    torch.cuda.set_device(local)
    ensure_weights(0, 1)
    from navi_b200 import engine
    dev = engine.Device(local)
    w = engine.Weights(dev, BENCH_NAVI)
    chunks = tuple(int(c) for c in args.voc_chunks.split(","))
    v = vocoder_bench(dev, w, reps=args.steps, chunks=chunks, warm=args.warmup)
    line = {"metric": "vocoder ms per frame (configs[3])", "impl": "ours", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "dtype": "f16 weights / f32 activations (f16 hi+lo on the tensor cores)",
            "data": "synthetic (seeded random-init weights N(0,0.02), uniform random codes)", "vocoder": v}
    if args.cpu_baseline:
        line["vocoder"]["cpu_baseline"] = vocoder_cpu_baseline()
    emit(line)


def run_prefill_only(args):
    """`--prefill-only`: the talker prefill of configs[4]'s prompt (200 uniform text ids in the
    reference's template, 208 prefill rows) alone on one GPU: prompt rows then the 28-layer
    prefill (Talker::build_prompt + Talker::prefill, talker.hip:283-399), device time per call
    (Talker::last_ms, the prefill kernels only) and wall time of both calls, medians of
    `--steps` after `--warmup`. One JSON line."""
    import numpy as np
    import torch
    rank, local, world = dist_env()
    if world > 1 and rank != 0:
        return
    torch.cuda.set_device(local)
    ensure_weights(0, 1)
    from navi_b200 import engine, model_spec
    dev = engine.Device(local)
    w = engine.Weights(dev, BENCH_NAVI)
    cfg = model_spec.full_config(w.params.decoder_dim)
    tal = engine.Talker(dev, w, max_prompt_tokens=1024, max_positions=4096)
    r = np.random.default_rng(1000)
    ids = [cfg.im_start_id, cfg.assistant_id, 198] + r.integers(0, cfg.text_vocab, 200).tolist() + \
        [cfg.im_end_id, 198, cfg.im_start_id, cfg.assistant_id, 198]
    spk = np.random.default_rng(4).standard_normal(w.params.talker.hidden).astype(np.float32)
    dev_ms, wall_ms, rows = [], [], 0
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        pr = tal.build_prompt(ids, "english", spk)
        tal.prefill(pr)
        torch.cuda.synchronize()
        if i >= args.warmup:
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            dev_ms.append(tal.last_ms())
        rows = pr.n_prefill
    emit({"metric": "talker prefill ms (configs[4] prompt)", "impl": "ours", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
          "higher_is_better": False, "dtype": "f16 weights / f32 activations (f16 hi+lo on the tensor cores)",
          "data": "synthetic (seeded random-init weights N(0,0.02), uniform random text ids)",
          "config": {"workload": "configs[4] prompt: 200 text ids, prefill rows", "prefill_rows": rows},
          "prefill_ms": float(np.median(dev_ms)), "prompt_and_prefill_wall_ms": float(np.median(wall_ms))})


def run_phase_trace(args):
    """`--phase-trace`: per-phase device time of the configs[1]+[2] frame at --kv on one GPU.
    After --warmup frames, --steps traced frames stamp every phase on every CTA
    (Frame.set_profile(True, -1)); a phase ends when its last CTA stamps its end. Prints the
    per-phase medians over the traced frames and their sums by part of the frame."""
    import numpy as np
    import torch
    from navi_b200 import engine
    ensure_weights(0, 1)
    dev = engine.Device(0)
    w = engine.Weights(dev, BENCH_NAVI)
    frame = engine.Frame(dev, w)
    tl = w.params.talker
    kvd = tl.n_kv_head * tl.head_dim
    max_pos = max(2048, args.kv) + 1
    g = torch.Generator(device="cuda:0").manual_seed(1000)
    k = [torch.randn(max_pos, kvd, generator=g, device="cuda:0").half() for _ in range(tl.n_layer)]
    v = [torch.randn(max_pos, kvd, generator=g, device="cuda:0").half() for _ in range(tl.n_layer)]
    kv = engine.KvCache.wrap([t.data_ptr() for t in k], [t.data_ptr() for t in v], max_pos, kvd, keepalive=(k, v))
    step0 = torch.randn(tl.hidden, generator=g, device="cuda:0")
    trailing = torch.randn(tl.hidden, generator=g, device="cuda:0")
    s = engine.Sampling(temperature=0.9, top_k=50, top_p=0.9, repetition_penalty=1.05, cp_temperature=0.9, cp_top_k=50,
                        cp_top_p=0.9, min_frames=2, rng=1)
    frame.set_step_in(step0.data_ptr())
    frame.reset()
    for i in range(args.warmup):
        assert frame.run(kv, args.kv, trailing.data_ptr(), s, 7, i).ok
    frame.set_profile(True, -1)
    durs = []
    for i in range(args.steps):
        assert frame.run(kv, args.kv, trailing.data_ptr(), s, 7, args.warmup + i).ok
        t0, st = frame.profile_all()                        # [G], [G, phases, 4] ns
        ends = np.concatenate([[t0.min()], st[:, :, 3].max(axis=0)])
        durs.append(np.diff(ends) / 1000.0)
    frame.set_profile(False)
    d = np.median(np.array(durs), axis=0)
    # program order: talker layers (5 phases each), codec head, code-predictor positions 0 + 1
    # as one pass of 26 phases (its first phase stages the codebook-0 draw), 14 passes of 26
    # (each first phase stages the previous draw), FINAL
    L = tl.n_layer * 5
    cp = d[L + 1:L + 27]
    passes = d[L + 27:-1]
    emit({"metric": "k_frame per-phase device time (us)", "impl": "ours", "n_gpus": 1, "kv_len": args.kv, "traced_frames": args.steps,
          "total_us": round(float(d.sum()), 1), "n_phases": int(len(d)),
          "talker": {"us": round(float(d[:L].sum()), 1),
                     "median_by_kind_qkv_attn_o_gu_down": [round(float(x), 2) for x in np.median(d[:L].reshape(-1, 5), axis=0)]},
          "codec_head_us": round(float(d[L]), 2), "codebook0_draw_phase_us": round(float(d[L + 1]), 2),
          "cp_positions_0_1_us": round(float(cp.sum()), 1),
          "cp_positions_2_15_us": round(float(passes.sum()), 1),
          "cp_pass_us_median": round(float(np.median(passes.reshape(-1, 26).sum(axis=1))), 1) if len(passes) % 26 == 0 else None,
          "cp_draw_phase_us_median": round(float(np.median(passes.reshape(-1, 26)[:, 0])), 2) if len(passes) % 26 == 0 else None,
          "final_us": round(float(d[-1]), 2),
          "phases_us": [round(float(x), 2) for x in d]})


def run_ours(args):
    import numpy as np
    import torch
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=900))
    ensure_weights(rank, world)
    from navi_b200 import engine

    dev = engine.Device(local)
    w = engine.Weights(dev, BENCH_NAVI)
    frame = engine.Frame(dev, w)
    p = w.params
    tl = p.talker
    kvd = tl.n_kv_head * tl.head_dim
    max_pos = max(2048, args.kv) + 1
    g = torch.Generator(device=f"cuda:{local}").manual_seed(1000 + rank)
    k = [torch.randn(max_pos, kvd, generator=g, device=f"cuda:{local}").half() for _ in range(tl.n_layer)]
    v = [torch.randn(max_pos, kvd, generator=g, device=f"cuda:{local}").half() for _ in range(tl.n_layer)]
    kv = engine.KvCache.wrap([t.data_ptr() for t in k], [t.data_ptr() for t in v], max_pos, kvd, keepalive=(k, v))
    step0 = torch.randn(tl.hidden, generator=g, device=f"cuda:{local}")
    trailing = torch.randn(tl.hidden, generator=g, device=f"cuda:{local}")
    s = engine.Sampling(temperature=0.9, top_k=50, top_p=0.9, repetition_penalty=1.05, cp_temperature=0.9, cp_top_k=50,
                        cp_top_p=0.9, min_frames=2, rng=1)
    stream = torch.cuda.ExternalStream(dev.stream, device=f"cuda:{local}")
    seed = 20260 + rank

    def frames(n, L, start):
        for i in range(n):
            frame.enqueue(kv, L, trailing.data_ptr(), s, seed, start + i)

    def device_time(n, L):
        frame.set_step_in(step0.data_ptr())
        frame.reset()
        frames(args.warmup, L, 0)
        r = frame.collect()
        assert r.ok, r.error
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(local)
        if dist:
            dist.barrier()
        e0.record(stream)
        frames(n, L, args.warmup)
        e1.record(stream)
        r = frame.collect()
        torch.cuda.synchronize(local)
        assert r.ok, r.error
        return e0.elapsed_time(e1) / n   # ms per frame

    L = args.kv
    with ClockSampler(local) as clk:
        ms = device_time(args.steps, L)
    # e2e: public C ABI, synchronous per frame, host trailing row in, codes out
    h_trailing = torch.empty(tl.hidden, dtype=torch.float32, pin_memory=True)
    h_trailing.copy_(trailing.cpu())
    d_trailing = torch.empty_like(trailing)
    frame.set_step_in(step0.data_ptr())
    frame.reset()
    for i in range(args.warmup):
        frame.run(kv, L, trailing.data_ptr(), s, seed, i)
    torch.cuda.synchronize(local)
    if dist:
        dist.barrier()
    prev_stream = torch.cuda.current_stream(local)
    torch.cuda.set_stream(stream)   # the H2D copies go on the frame's stream, in order with the frames
    t0 = time.perf_counter()
    for i in range(args.steps):
        d_trailing.copy_(h_trailing, non_blocking=True)
        r = frame.run(kv, L, d_trailing.data_ptr(), s, seed, args.warmup + i)
        assert r.ok, r.error
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    torch.cuda.set_stream(prev_stream)
    # the KV-length sweep of configs[1] (device time, fewer frames)
    sweep = {}
    for Ls in (64, 512, 2048):
        sweep[str(Ls)] = round(device_time(max(10, args.steps // 4), Ls), 4)
    # per-phase profile of one frame (CTA 0), for the record
    frame.set_profile(True)
    frame.run(kv, L, trailing.data_ptr(), s, seed, 10_000)
    prof = frame.profile()
    frame.set_profile(False)

    ms, e2e_ms, value, e2e_value = combine_ranks(ms, e2e_ms, world, dist, f"cuda:{local}")
    serving = serving_bench(dev, w, rank, world, dist, streams=args.streams, group=args.group) if args.streams > 0 else None
    if rank == 0:
        ab = algorithmic_bytes(p, L)
        peak, kind = measured_peak()
        achieved = ab / (ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 weights / f32 math", "data": "synthetic (seeded random-init weights N(0,0.02), random f16 KV)",
            "config": {"workload": f"configs[1]+[2]: 28-layer talker step at KV {L} + 15-step code predictor, "
                                   f"top-k 50 / top-p 0.9 / T 0.9, Philox", "kv_len": L, "batch": 1,
                       "parallelism": f"request-parallel replicas x{world}",
                       "l2": "per-frame working set ~1.1 GB > 126 MB L2 (no flush needed)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": ncu_traffic(L), "peak_kind": kind,
                         "algorithmic_bytes": ab},
            "e2e": {"value": e2e_value, "unit": "frames/s", "h2d_bytes_per_step": 4 * tl.hidden,
                    "d2h_bytes_per_step": 16 * 4 + 16},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "kv_sweep_ms_per_frame": sweep,
            "phase_profile_us": {"total": round(float(prof.sum()), 1), "n_phases": int(len(prof)),
                                 "median": round(float(np.median(prof)), 2), "max": round(float(prof.max()), 2)},
        }
        if serving:
            line["serving"] = serving
        line["batched_decode"] = batch_bench(frame, p, local, steps=max(10, min(args.steps, 100)), warm=args.warmup)
        if args.layer:
            line["layer"] = layer_bench(local, reps=max(20, min(args.steps, 200)), warm=args.warmup)
        if args.vocoder:
            line["vocoder"] = vocoder_bench(dev, w)
        if args.cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(L)
            if args.vocoder:
                line["vocoder"]["cpu_baseline"] = vocoder_cpu_baseline()
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


_JSON_FD = None


def emit(line: dict) -> None:
    """Writes the result line to the process's real standard output (libraries' banners,
    such as NCCL's version line, go to standard error; see main)."""
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _JSON_FD
    # everything written to fd 1 by this process or its libraries goes to standard error; the
    # one JSON line goes to the original standard output
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--kv", type=int, default=512)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-vocoder", dest="vocoder", action="store_false", help="skip the configs[3] vocoder line")
    ap.add_argument("--vocoder-only", action="store_true", help="run only the configs[3] vocoder measurement")
    ap.add_argument("--prefill-only", action="store_true", help="run only the talker prefill of the configs[4] prompt")
    ap.add_argument("--phase-trace", action="store_true", help="per-phase device time of one frame (traced, not a bench value)")
    ap.add_argument("--voc-chunks", default="4,16", help="vocoder chunk lengths (frames), comma separated")
    ap.add_argument("--no-layer", dest="layer", action="store_false", help="skip the configs[0] single-layer line")
    ap.add_argument("--streams", type=int, default=64, help="configs[4] utterances over all GPUs (64 = the full config; 0 = skip)")
    ap.add_argument("--group", type=int, default=4, choices=[1, 2, 3, 4], help="configs[4] streams decoded together per GPU")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.vocoder_only:
        run_vocoder_only(args)
    elif args.prefill_only:
        run_prefill_only(args)
    elif args.phase_trace:
        run_phase_trace(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
