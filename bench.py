#!/usr/bin/env python3
"""Benchmark: Q8_0 SigLIP2-so400m vision tower, images/s, on a 512-image NaFlex batch.

One step = one batch of 512 NaFlex images (patch count uniform in [256, 1024]
on a random grid, patches uniform in [-1, 1], PROBE pooling) through the full
27-layer Q8_0 tower with synthetic N(0, 0.02) weights, followed by the NCCL
gather of the 1152-d pooled embeddings to rank 0.  With N GPUs the 512 images
are sharded across ranks (length-balanced), so total work is fixed: strong
scaling.  Inputs (1.2 GB of patches) and activations are far larger than L2,
so no separate L2 flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

`value` is device-timed (CUDA events, max over ranks) with patches resident in
HBM; `e2e` is the same metric through the public host-buffer entry points,
pinned host patches in and host embeddings out every step: on one GPU the
pipelined b2q_vision_submit_host (each step's upload overlaps the previous
step's encode), on several the same with b2q_vision_wait_submitted, each
step's embeddings gathered on a side stream while the next step encodes.  `roofline` is the dominant kernel, the fc1 Q8_0 GEMM, timed with CUDA
events at the batch's shape.  `cpu_baseline` times the CPU restatement of the
same tower on this host's cores on a bounded sample (the reference's ggml CPU
path cannot be built here: its ggml submodule is empty).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "hbd-siglip2.cpp_b200"))

METRIC = "Q8_0 vision images/s at 1/2/4/8 B200; MMQ GEMM int8 TOPS vs peak"
N_IMAGES = 512
CPU_SIDE = 25        # CPU samples: one 25x25-patch image, nearest square to the batch's mean patch count
PATCH_DIM = 768
# DRAM bytes per token of one fc1 launch: dram__bytes_read + dram__bytes_write
# = 171.99 + 551.98 MB from one ncu capture (one pass) of
# `bench.py --profile-gemm 65536` (192-column tiles), scaled to the batch's
# token count (the traffic grows in proportion to M).
FC1_DRAM_BYTES_PER_TOKEN = (171.99e6 + 551.98e6) / 65536


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def int8_peak_tops():
    """Dense int8 tensor-core reference measured here: cuBLASLt int8 x int8 ->
    int32 GEMM (torch._int_mm) at 8192^3, best of 10 after warm-up (a library
    GEMM used as the yardstick, not part of the measured path)."""
    import torch
    try:
        n = 8192
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except RuntimeError as exc:      # no int8 GEMM in this torch build
        log(f"int8 reference GEMM unavailable: {exc}")
        return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops", 1590.0)), float(d.get("hbm_gbs", 6650.0)), "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"b2q_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if not self.proc or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                if int(f[0]) not in self.gpus:
                    continue
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        try:
            self.path.unlink()
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons)}


def cpu_tower_sample(threads=None):
    """Time the CPU restatement of the tower on one 25x25-patch image (625
    tokens), PROBE pooling, all host threads."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from b2q import synth
    O.build()
    n = threads or os.cpu_count() or 1
    O.set_threads(n)
    ck = synth.vision_checkpoint(synth.TowerConfig(), seed=0)
    x = synth.patches(CPU_SIDE * CPU_SIDE, PATCH_DIM, seed=1)
    O.vision_encode(ck, x[:16], 4, 4, pooling=1)   # warm the library and threads
    return O, ck, x, n


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    O, ck, x, cores = cpu_tower_sample()
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.vision_encode(ck, x, CPU_SIDE, CPU_SIDE, pooling=1)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = args.steps / total
    sample = (f"1 image of {CPU_SIDE}x{CPU_SIDE} = {CPU_SIDE * CPU_SIDE} patches per step (the 512-image "
              "NaFlex batch averages 613 patches per image), PROBE pooling")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": {"workload": "512-image NaFlex batch through the 27-layer Q8_0 SigLIP2-so400m vision tower "
                               "(CPU sample)", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def fc1_gemm(M, weights=None, reps=5, gelu=True):
    """Time the fc1 Q8_0 GEMM (N=4304, K=1152) with the GELU->q8_1 epilogue
    (or, gelu=False, the bias epilogue with fp32 output) at M tokens; CUDA
    events on the launching stream.  -> (ms per launch, TOPS)"""
    import torch
    import b2q
    from b2q import synth
    cfg = synth.TowerConfig()
    if weights is None:
        rng = np.random.default_rng(0)
        weights = synth.quantize_q8_0((rng.standard_normal((cfg.ffn, cfg.hidden)) * 0.02).astype(np.float32))
    W = b2q.Weight(weights, cfg.ffn, cfg.hidden)
    act = b2q.act_empty(M, cfg.hidden)
    act_o = b2q.act_empty(M, cfg.ffn)
    b2q.quantize_q8_1(torch.randn((M, cfg.hidden), device="cuda"), act, M, cfg.hidden)
    bias = torch.zeros(cfg.ffn, device="cuda")
    stream = torch.cuda.current_stream()
    y = None if gelu else torch.empty((M, cfg.ffn), dtype=torch.float32, device="cuda")

    def launch():
        if gelu:
            b2q.mul_mat(W, act, M, None, kind=b2q.EPI_BIAS_GELU_Q8, bias=bias, act_out=act_o)
        else:
            b2q.mul_mat(W, act, M, y, kind=b2q.EPI_BIAS, bias=bias)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    W.release()
    return ms, 2.0 * M * cfg.ffn * cfg.hidden / (ms * 1e-3) / 1e12


def profile_gemm(tokens, epilogue="gelu", ctas=0):
    import b2q
    b2q.init(0)
    b2q.tune(b2q.TUNE_GEMM_CTAS, ctas)
    ms, tops = fc1_gemm(tokens, reps=2, gelu=epilogue == "gelu")
    b2q.check_device()
    print(json.dumps({"kernel": "gemm_q8_kernel fc1", "epilogue": epilogue, "ctas_per_sm": ctas or "auto",
                      "tokens": tokens, "ms": ms, "tops": tops}), flush=True)
    return 0


def profile_rowops(tokens):
    """Time the two HBM-bound row kernels at `tokens` rows of 1152 (one CUDA
    event pair over 5 launches each, after warm-up) and report GB/s on their
    algorithmic bytes: LayerNorm->q8_1 reads 4*H and writes the q8_1 planes
    (H value carriers + 4*H/32 scales); quantize reads 4*K and writes the same
    planes.  The planes' value carriers are 1 byte (int8 operand mode) or 2
    bytes (fp16 carriers, the default)."""
    import torch
    import b2q
    b2q.init(0)
    H = 1152
    _, es, _, _ = b2q.act_layout(tokens, H)
    x = torch.randn((tokens, H), device="cuda")
    w = torch.ones(H, device="cuda")
    b = torch.zeros(H, device="cuda")
    act = b2q.act_empty(tokens, H)
    plane_bytes = H * es + 4 * H // 32
    _, hbm, src = peaks()
    res = {"kernel": "rowops", "tokens": tokens, "carrier_bytes": es, "hbm_peak_gbs": hbm, "peak_source": src}
    for name, fn in (("ln_quant_kernel", lambda: b2q.ln_quantize(x, w, b, 1e-6, tokens, H, act)),
                     ("quantize_rows_kernel", lambda: b2q.quantize_q8_1(x, act, tokens, H))):
        ms = min(_events_ms(fn, 5) for _ in range(3))
        gbs = tokens * (4 * H + plane_bytes) / (ms * 1e-3) / 1e9
        res[name] = {"ms": ms, "bytes_per_token": 4 * H + plane_bytes, "gbs": gbs, "frac_hbm": gbs / hbm}
    b2q.check_device()
    print(json.dumps(res), flush=True)
    return 0


def profile_attention(n_images):
    """Time one layer's attention over a packed batch of n_images NaFlex images
    (the bench's seeded grids, random fp16 [Q|K|V] rows) with each tensor-core
    kernel; CUDA events.  Algorithmic work 4*L^2*72 flops per head."""
    import torch
    import b2q
    from b2q import synth
    b2q.init(0)
    cfg = synth.TowerConfig()
    H, nh = cfg.hidden, cfg.n_head
    grids = synth.naflex_grids(n_images, seed=0)
    lens = [int(h) * int(w) for h, w in grids]
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    T = int(sum(lens))
    qkv = torch.randn((T, 3 * H), device="cuda", dtype=torch.float16)
    out = torch.empty((T, H), device="cuda", dtype=torch.float32)
    flops = sum(4.0 * L * L * (H // nh) * nh for L in lens)

    def run():
        b2q.attention(qkv, 3 * H, qkv[:, H:], 3 * H, qkv[:, 2 * H:], 3 * H, offs, lens, offs, lens, offs, nh, out, H)

    res = {"kernel": "attention", "images": n_images, "tokens": T}
    for name, k in (("tcgen05", 0), ("mma_sync", 1)):
        b2q.tune(b2q.TUNE_ATTN_KERNEL, k)
        ms = min(_events_ms(run, 1) for _ in range(5))
        res[name] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}
    b2q.tune(b2q.TUNE_ATTN_KERNEL, 0)
    b2q.check_device()
    print(json.dumps(res), flush=True)
    return 0


def _events_ms(fn, reps, warm=2):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def suite(args):
    """The other workloads on one GPU, one JSON line each: batch-1 vision at 27x27
    patches, the isolated GEMM sweep, the 5x64 text batch and zero-shot scoring
    (the NaFlex batch is the default bench line).  CPU counterparts: the CPU restatement (oracle/)
    on all host threads, on the samples named in each line."""
    import math
    import torch
    import b2q
    from b2q import synth
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    O.build()
    cores = os.cpu_count() or 1
    O.set_threads(cores)
    b2q.init(0)
    out = []

    def emit(d):
        print(json.dumps(d), flush=True)
        out.append(d)

    i8 = int8_peak_tops()
    cfg = synth.TowerConfig()
    rng = np.random.default_rng(0)

    # ---- GEMM sweep (ggml_mul_mat = quantize + GEMM, and GEMM alone)
    for (N, K) in [(1152, 1152), (3456, 1152), (4304, 1152), (1152, 4304)]:
        Kp = (K + 31) // 32 * 32
        wq = synth.quantize_q8_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32), Kp)
        W = b2q.Weight(wq, N, Kp)
        xs = rng.standard_normal((64, K)).astype(np.float32)
        t = time.perf_counter()
        qs, d = O.quantize_q8_1(xs, Kp)
        O.gemm_q8(wq, N, Kp, qs, d)
        cpu_gops = 2.0 * 64 * N * K / (time.perf_counter() - t) / 1e9
        for M in (729, 4096, 65536):
            x = torch.randn((M, K), device="cuda")
            act = b2q.act_empty(M, Kp)
            scratch = b2q.act_empty(M, Kp)
            y = torch.empty((M, N), device="cuda")
            b2q.quantize_q8_1(x, act, M, K)
            ms_gemm = _events_ms(lambda: b2q.mul_mat(W, act, M, y), 10)
            ms_full = _events_ms(lambda: b2q.mul_mat_f32(W, x, M, K, y, scratch), 10)
            tops = 2.0 * M * N * K / (ms_gemm * 1e-3) / 1e12
            emit({"config": "GEMM sweep", "M": M, "N": N, "K": K, "gemm_ms": ms_gemm, "gemm_tops": tops,
                  "mul_mat_ms": ms_full, "mul_mat_tops": 2.0 * M * N * K / (ms_full * 1e-3) / 1e12,
                  "frac_int8": tops / i8 if i8 else None, "int8_peak_measured": i8,
                  "cpu_gops": cpu_gops, "cpu_sample": f"M=64 rows, {cores} threads"})
            del x, act, scratch, y
        W.release()
    b2q.check_device()

    # ---- vision tower, batch 1, 27 x 27 patches
    vck = synth.vision_checkpoint(cfg, seed=0)
    vt = b2q.VisionTower(cfg)
    vt.load(vck)
    p1 = synth.patches(729, cfg.patch_dim, seed=1)
    pd = torch.from_numpy(p1).cuda()
    emb = torch.empty((1, cfg.hidden), device="cuda")
    ms1 = _events_ms(lambda: vt.encode(pd, [(27, 27)], b2q.POOL_PROBE, out=emb), 20, warm=3)
    t = time.perf_counter()
    O.vision_encode(vck, p1, 27, 27, pooling=1)
    cpu1 = 1.0 / (time.perf_counter() - t)
    emit({"config": "vision batch 1, 729 patches", "ms_per_image": ms1, "images_per_s": 1e3 / ms1,
          "int8_tops": 604.5e9 / (ms1 * 1e-3) / 1e12, "cpu_images_per_s": cpu1, "cpu_cores": cores})

    # ---- text tower, 5 prompts x 64
    tck = synth.text_checkpoint(cfg, seed=0)
    tt = b2q.TextTower(cfg)
    tt.load(tck)
    ids = synth.token_ids(5, cfg.n_pos, cfg.vocab, seed=1)
    idd = torch.from_numpy(ids).cuda()
    temb = torch.empty((5, cfg.hidden), device="cuda")
    ms3 = _events_ms(lambda: tt.encode(idd, out=temb), 20, warm=3)
    t = time.perf_counter()
    O.text_encode(tck, ids)
    cpu3 = 5.0 / (time.perf_counter() - t)
    emit({"config": "text 5 x 64", "ms_per_batch": ms3, "prompts_per_s": 5e3 / ms3,
          "cpu_prompts_per_s": cpu3, "cpu_cores": cores})

    # ---- zero-shot, 2048 images x 729 patches vs 1000 prompts, one GPU
    n_img, n_txt, chunk = 2048, 1000, 512
    pchunk = torch.from_numpy(np.concatenate([synth.patches(729, cfg.patch_dim, seed=10 + i)
                                              for i in range(chunk)])).cuda()
    img = torch.empty((n_img, cfg.hidden), device="cuda")
    ids5 = torch.from_numpy(synth.token_ids(n_txt, cfg.n_pos, cfg.vocab, seed=2)).cuda()
    txt = torch.empty((n_txt, cfg.hidden), device="cuda")
    vt.reserve(chunk * 729, chunk)
    tt.reserve(n_txt)

    def zero_shot():
        for c in range(0, n_img, chunk):
            vt.encode(pchunk, [(27, 27)] * chunk, b2q.POOL_PROBE, out=img[c:c + chunk])
        tt.encode(ids5, out=txt)
        return b2q.score(img, txt, math.log(10.0), -10.0, logits=False)

    ms5 = _events_ms(zero_shot, 2, warm=1)
    b2q.check_device()
    emit({"config": "zero-shot 2048 images x 1000 prompts (1 GPU)", "ms": ms5,
          "images_per_s": n_img * 1e3 / ms5, "note": "patches of the 512-image chunk reused for all 4 chunks"})
    if args.out:
        Path(args.out).write_text("".join(json.dumps(d) + "\n" for d in out))
    return 0


INT8_DATASHEET_TOPS = 4500.0
INT8_DATASHEET_SOURCE = ("NVIDIA HGX B200 specifications: INT8 Tensor Core 72 POPS for 8 GPUs with sparsity, "
                         "i.e. 4.5 POPS dense per GPU")


def roofline_line(gemm_ms, gemm_tops, M, i8_peak):
    """The fc1 GEMM against the int8 tensor-core roofline: the int8 dense
    reference measured in this run (cuBLASLt int8 GEMM at 8192^3) when the
    torch build has one, else the datasheet figure; both fractions and the
    bf16 one are reported."""
    bf16_peak, _, peak_src = peaks()
    peak = i8_peak if i8_peak else INT8_DATASHEET_TOPS
    traffic = (FC1_DRAM_BYTES_PER_TOKEN * M) if FC1_DRAM_BYTES_PER_TOKEN else None
    return {"kernel": "gemm_q8_kernel (fc1, N=4304, K=1152, GELU->q8_1 epilogue)",
            "bound": "tensor", "achieved": gemm_tops, "peak": peak, "unit": "TFLOP/s",
            "op_kind": "int8 multiply-adds counted as 2 ops (TOPS)",
            "frac": gemm_tops / peak,
            "peak_source": ("int8 dense, measured in this run: cuBLASLt int8 x int8 -> int32 GEMM "
                            "(torch._int_mm) at 8192^3, best of 10" if i8_peak else INT8_DATASHEET_SOURCE),
            "int8_peak_measured": i8_peak,
            "int8_peak_datasheet": INT8_DATASHEET_TOPS, "int8_datasheet_source": INT8_DATASHEET_SOURCE,
            "frac_datasheet": gemm_tops / INT8_DATASHEET_TOPS,
            "bf16_peak_measured": bf16_peak, "frac_bf16": gemm_tops / bf16_peak,
            "bf16_peak_source": f"MEASURED_PEAKS.json bf16 burst ({peak_src})",
            "launch_ms": gemm_ms, "M": M, "traffic": traffic}


def timed(fn, steps, stream, world):
    """Device time of `steps` calls of fn (CUDA events on `stream`, barrier
    and synchronize on both sides) -> (max over ranks, this rank's) in ms."""
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    mine = e0.elapsed_time(e1)
    ms = torch.tensor([mine], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item()), mine


def per_rank(values, world):
    """All-gather a small list of floats from every rank -> list per rank."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    if world == 1:
        return [values]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="naflex", choices=["naflex", "zeroshot"],
                    help="naflex: the 512-image NaFlex vision batch (default); zeroshot: 2048 images x 1000 "
                         "prompts scored with both towers, images and prompts sharded over the ranks")
    ap.add_argument("--images", type=int, default=N_IMAGES)
    ap.add_argument("--exact-attention", action="store_true",
                    help="attention in the fixed fp32 order that makes the tower bit-identical to the CPU "
                         "restatement (the parity-clean configuration)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-gemm", type=int, default=0, metavar="TOKENS",
                    help="only run the fc1 GEMM (GELU->q8_1 epilogue) at this token count, for ncu captures")
    ap.add_argument("--profile-epilogue", default="gelu", choices=["gelu", "f32"],
                    help="--profile-gemm: GELU->q8_1 epilogue (default) or bias + fp32 output")
    ap.add_argument("--profile-ctas", type=int, default=0, choices=[0, 1, 2],
                    help="--profile-gemm: GEMM CTAs per SM (0 = the library's choice)")
    ap.add_argument("--profile-rowops", type=int, default=0, metavar="TOKENS",
                    help="only time the LayerNorm->q8_1 and quantize kernels at this token count (GB/s)")
    ap.add_argument("--profile-attention", type=int, default=0, metavar="IMAGES",
                    help="only time one layer's attention over this many NaFlex images, both tensor-core kernels")
    ap.add_argument("--suite", action="store_true",
                    help="the other workloads on one GPU (batch-1 vision, GEMM sweep, text, zero-shot), JSON lines")
    ap.add_argument("--out", default="", help="--suite: also write the JSON lines to this file")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.profile_gemm:
        return profile_gemm(args.profile_gemm, args.profile_epilogue, args.profile_ctas)
    if args.profile_rowops:
        return profile_rowops(args.profile_rowops)
    if args.profile_attention:
        return profile_attention(args.profile_attention)
    if args.suite:
        return suite(args)

    import torch
    import torch.distributed as dist
    import b2q

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    b2q.init(local)
    if args.exact_attention:
        b2q.tune(b2q.TUNE_ATTN_EXACT, 1)
    try:
        if args.workload == "zeroshot":
            run_zeroshot(args, world, rank)
        else:
            run_naflex(args, world, rank)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    return 0


def run_naflex(args, world, rank):
    import torch
    import b2q
    from b2q import synth
    from b2q.shard import gather_in_order, per_rank_capacity, shard_images

    cfg = synth.TowerConfig()
    t0 = time.time()
    ck = synth.vision_checkpoint(cfg, seed=0)
    tower = b2q.VisionTower(cfg)
    tower.load(ck)
    log(f"[rank {rank}] weights ready in {time.time() - t0:.1f}s")

    grids = synth.naflex_grids(args.images, seed=0)
    mine = shard_images(grids, rank, world)
    my_grids = [grids[i] for i in mine]
    my_tokens = sum(h * w for h, w in my_grids)
    total_tokens = sum(h * w for h, w in grids)
    host = torch.empty((my_tokens, PATCH_DIM), dtype=torch.float32, pin_memory=True)
    off = 0
    for i in mine:
        n = grids[i][0] * grids[i][1]
        host[off:off + n] = torch.from_numpy(synth.patches(n, PATCH_DIM, seed=i))
        off += n
    dev = host.cuda()
    tower.reserve(my_tokens, len(my_grids))
    per_cap = per_rank_capacity(args.images, world)
    emb = torch.zeros((per_cap, cfg.hidden), dtype=torch.float32, device="cuda")
    mine_dev = torch.tensor(mine, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()
    gather_events = []

    def gather(record=False):
        # pooled embeddings of all images, in the batch's order, on every rank
        if world == 1:
            return emb[:len(mine)]
        if record:
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
        out = gather_in_order(emb[:len(mine)], mine_dev, args.images)
        if record:
            g1.record(stream)
            gather_events.append((g0, g1))
        return out

    def step_device(record=False):
        tower.encode(dev, my_grids, b2q.POOL_PROBE, out=emb)
        gather(record)

    gathered_host = torch.empty((args.images, cfg.hidden), dtype=torch.float32, pin_memory=True)

    out_pinned = torch.empty((len(my_grids), cfg.hidden), dtype=torch.float32, pin_memory=True)

    def step_e2e():
        # public host-buffer entry point, one rank: pinned patches in,
        # embeddings out, pipelined (this step's upload overlaps the previous
        # step's encode; the timed region ends after the last download).
        # Several ranks: e2e_pipelined below.
        import ctypes as C
        g = np.asarray(my_grids, np.int32).reshape(-1)
        b2q.check(b2q.lib().b2q_vision_submit_host(tower.handle, host.data_ptr(), g.ctypes.data_as(b2q.I32P),
                                                   len(my_grids), b2q.POOL_PROBE, out_pinned.data_ptr(),
                                                   C.c_void_p(stream.cuda_stream)))

    # Several ranks: each step's embeddings feed the gather, so the step is
    # pipelined across the host-buffer entry points: submit batch i (its
    # upload runs under batch i - 1's encode), wait for batch i - 1's
    # download, gather it on a side stream while batch i encodes.  Every
    # step's upload, download and gather falls inside the timed region
    # (events on `stream`, which waits for the side stream at the end).
    out_pin = [torch.empty((len(my_grids), cfg.hidden), dtype=torch.float32, pin_memory=True) for _ in range(2)]
    side = torch.cuda.Stream() if world > 1 else None

    def submit(i):
        import ctypes as C
        g = np.asarray(my_grids, np.int32).reshape(-1)
        b2q.check(b2q.lib().b2q_vision_submit_host(tower.handle, host.data_ptr(), g.ctypes.data_as(b2q.I32P),
                                                   len(my_grids), b2q.POOL_PROBE, out_pin[i % 2].data_ptr(),
                                                   C.c_void_p(stream.cuda_stream)))

    def consume(i):
        with torch.cuda.stream(side):
            # a blocking copy: the pinned buffer is free again when it returns
            emb[:len(my_grids)].copy_(out_pin[i % 2], non_blocking=False)
            allemb = gather_in_order(emb[:len(mine)], mine_dev, args.images)
            if rank == 0:
                gathered_host.copy_(allemb, non_blocking=True)

    def e2e_pipelined(steps):
        import torch.distributed as dist
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            submit(i)
            if i > 0:
                tower.wait_submitted(1)
                consume(i - 1)
        tower.wait_submitted(0)
        consume(steps - 1)
        stream.wait_stream(side)
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize()
    b2q.check_device()

    n0 = b2q.launch_count()
    gpus_used = list(range(args.gpus)) if rank == 0 else []
    with ClockSampler(gpus_used) as clk:
        ms, my_ms = timed(lambda: step_device(True), args.steps, stream, world)
    launches = b2q.launch_count() - n0
    clocks = clk.summary()
    b2q.check_device()
    gather_ms = (sum(a.elapsed_time(b) for a, b in gather_events) / len(gather_events)) if gather_events else 0.0

    # end to end through the host-buffer entry points
    if world == 1:
        step_e2e()
        ms_e2e, _ = timed(step_e2e, args.steps, stream, world)
    else:
        e2e_pipelined(2)
        ms_e2e = e2e_pipelined(args.steps)

    # roofline of the dominant kernel: fc1 GEMM (N=4304, K=1152) with the
    # GELU->q8_1 epilogue at this rank's token count, CUDA events on the stream
    M = my_tokens
    gemm_ms, gemm_tops = fc1_gemm(M, weights=ck.tensors["v.blk.0.ffn_up.weight"])
    i8_peak = int8_peak_tops() if rank == 0 else None
    ranks = per_rank([float(rank), float(my_tokens), float(len(mine)), my_ms / args.steps, gather_ms], world)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            O, ck_cpu, x, cores = cpu_tower_sample()
            t = time.perf_counter()
            O.vision_encode(ck_cpu, x, CPU_SIDE, CPU_SIDE, pooling=1)
            dt = time.perf_counter() - t
            cpu = {"value": 1.0 / dt, "unit": "images/s", "cores": cores, "kind": "port",
                   "sample": f"1 image of {CPU_SIDE}x{CPU_SIDE} patches (the batch averages 613), PROBE pooling, "
                             "CPU restatement (oracle/), AVX512-VNNI block dots where the host has them, "
                             "OpenMP over all host threads"}
        images = args.images * args.steps
        line = {
            "metric": METRIC, "value": images / (ms * 1e-3), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": "512 NaFlex images (256-1024 patches, random grids) through the "
                                   "27-layer Q8_0 SigLIP2-so400m vision tower, PROBE pooling",
                       "arithmetic": "Q8_0 x q8_1 int8 block dots, fp32 scales and accumulation",
                       "attention": ("exact: fixed fp32 order, tower bit-identical to the CPU restatement"
                                     if args.exact_attention else "tcgen05 tensor cores, fp16 Q/K/V"),
                       "global_batch": args.images, "tokens_per_step": total_tokens,
                       "parallelism": f"image-sharded replicas x{world} + NCCL all-gather",
                       "l2": "inputs and activations larger than L2 (no flush)"},
            "e2e": {"value": images / (ms_e2e * 1e-3), "unit": "images/s",
                    "h2d_bytes_per_step": int(total_tokens * PATCH_DIM * 4),
                    "d2h_bytes_per_step": int(args.images * cfg.hidden * 4)},
            "roofline": roofline_line(gemm_ms, gemm_tops, M, i8_peak),
            "gemm_tops": gemm_tops,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "ranks": [{"rank": int(r[0]), "tokens": int(r[1]), "images": int(r[2]), "ms_per_step": r[3],
                       "gather_ms": r[4]} for r in ranks],
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def run_zeroshot(args, world, rank):
    """Zero-shot scoring of 2048 images (27x27 patches, PROBE pooling) against
    1000 prompts (64 random token ids, EOS last) with logit scale exp(log 10)
    and bias -10: images and prompts split over the ranks, prompt embeddings
    all-gathered, each rank scoring its images, score rows gathered in image
    order (b2q.zeroshot).  One step is the whole job; value = images/s."""
    import math
    import torch
    import b2q
    from b2q import synth
    from b2q.shard import shard_rows
    from b2q.zeroshot import zero_shot

    n_img, n_txt, side, chunk = 2048, 1000, 27, 512
    ntok = side * side
    cfg = synth.TowerConfig()
    vt = b2q.VisionTower(cfg)
    vt.load(synth.vision_checkpoint(cfg, seed=0))
    tt = b2q.TextTower(cfg)
    tt.load(synth.text_checkpoint(cfg, seed=0))
    img_rows, txt_rows = shard_rows(n_img, rank, world), shard_rows(n_txt, rank, world)
    n_mine = len(img_rows)
    host = torch.empty((n_mine * ntok, PATCH_DIM), dtype=torch.float32, pin_memory=True)
    for j, i in enumerate(img_rows):
        host[j * ntok:(j + 1) * ntok] = torch.from_numpy(synth.patches(ntok, PATCH_DIM, seed=1000 + i))
    ids_all = synth.token_ids(n_txt, cfg.n_pos, cfg.vocab, seed=2)
    ids_host = torch.from_numpy(np.ascontiguousarray(ids_all[txt_rows.start:txt_rows.stop])).pin_memory()
    dev_p = host.cuda()
    ids_dev = ids_host.cuda()
    vt.reserve(min(chunk, n_mine) * ntok, min(chunk, n_mine))
    tt.reserve(max(1, len(txt_rows)))
    img_emb = torch.empty((n_mine, cfg.hidden), device="cuda")
    txt_emb = torch.empty((len(txt_rows), cfg.hidden), device="cuda")
    probs_host = torch.empty((n_img, n_txt), dtype=torch.float32, pin_memory=True)
    stream = torch.cuda.current_stream()

    def enc_img(rows):
        for c in range(0, n_mine, chunk):
            k = min(chunk, n_mine - c)
            vt.encode(dev_p[c * ntok:(c + k) * ntok], [(side, side)] * k, b2q.POOL_PROBE, out=img_emb[c:c + k])
        return img_emb

    def enc_txt(rows):
        if len(rows):
            tt.encode(ids_dev, out=txt_emb)
        return txt_emb

    def score(img, txt):
        _, probs = b2q.score(img, txt, math.log(10.0), -10.0, logits=False)
        return probs

    events = {}

    def step(record=False):
        return zero_shot(enc_img, enc_txt, score, n_img, n_txt, rank, world, timings=events if record else None)

    def step_e2e():
        dev_p.copy_(host, non_blocking=True)
        ids_dev.copy_(ids_host, non_blocking=True)
        out = step()
        if rank == 0:
            probs_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    b2q.check_device()
    n0 = b2q.launch_count()
    with ClockSampler(list(range(args.gpus)) if rank == 0 else []) as clk:
        ms, my_ms = timed(lambda: step(True), args.steps, stream, world)
    launches = b2q.launch_count() - n0
    clocks = clk.summary()
    b2q.check_device()

    def phase(a, b):
        return sum(x.elapsed_time(y) for x, y in zip(events[a], events[b])) / len(events[a])

    phases = [phase("start", "encoded"), phase("encoded", "text_gathered"), phase("text_gathered", "scored"),
              phase("scored", "done")]
    ms_e2e, _ = timed(step_e2e, args.steps, stream, world)
    ranks = per_rank([float(rank), float(n_mine), float(len(txt_rows)), my_ms / args.steps] + phases, world)
    if rank == 0:
        line = {
            "metric": "zero-shot images/s, 2048 images x 1000 prompts (both Q8_0 towers + sigmoid scoring)",
            "value": n_img * args.steps / (ms * 1e-3), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": "zero-shot: 2048 images of 27x27 patches (PROBE pooling) x 1000 prompts of 64 "
                                   "token ids, L2-normalised, sigmoid(10 * dot - 10)",
                       "parallelism": f"images and prompts sharded x{world}, prompt embeddings and score rows "
                                      "all-gathered (NCCL)",
                       "attention": ("exact" if args.exact_attention else "tcgen05 tensor cores (vision), "
                                     "exact (text)"),
                       "l2": "inputs and activations larger than L2 (no flush)"},
            "e2e": {"value": n_img * args.steps / (ms_e2e * 1e-3), "unit": "images/s",
                    "h2d_bytes_per_step": int(n_img * ntok * PATCH_DIM * 4 + n_txt * cfg.n_pos * 4),
                    "d2h_bytes_per_step": int(n_img * n_txt * 4)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "ranks": [{"rank": int(r[0]), "images": int(r[1]), "prompts": int(r[2]), "ms_per_step": r[3],
                       "encode_ms": r[4], "gather_text_ms": r[5], "score_ms": r[6], "gather_scores_ms": r[7]}
                      for r in ranks],
        }
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    sys.exit(main())
