"""Benchmark of the SAM 3 ViT vision trunk on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--format f16|q8_0] [--images 64]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's CPU trunk

Workload (ours): the seeded SAM 3 trunk (random-init weights of the real
architecture, GGUF in the requested format) on a batch of 64 synthetic
1008x1008 images sharded by image across the N GPUs (64/N each), outputs
gathered to rank 0 over NCCL.  One step = the whole batch through the trunk
(+ the gather).  `value` = images/s of the whole job with inputs resident in
HBM; `e2e` = the same through the public API with pinned host buffers
(host->device images and device->host feature maps inside the timed region).
Inputs (780 MB of images, 0.9 GB of weights, ~8 GB of activations per step)
are far larger than the 126 MB L2, so no explicit flush is done.

After the timed regions, one eager pass of the same trunk records a CUDA
event after every launch (s3t_trunk_profile): the roofline of the GEMM family,
the attention and LayerNorm figures and `trunk_profile_ms` come from the
trunk's own kernels at the bench's shape.

Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ViT-trunk images/s @1008^2"
FLOP_PER_IMAGE = 5.3986e12          # GEMMs 4609.6 GF + attention 782.8 GF + patch 6.24 GF
GEMM_FLOP_PER_IMAGE_LAYER = 144.05e9  # 2*T*C*(3C + C + 2F), T=5184, C=1024, F=4736
LAUNCHES_PER_TRUNK = 3 + 32 * 6 + 31  # im2col, patch GEMM, stem LN; 6 per block; 31 inter-block LNs
GATHER_CHUNKS = 4                     # N > 1: pieces of a rank's shard whose gather overlaps the next piece
MIN_PIECE = 8                         # ... each of at least this many images
# DRAM bytes (read + write) of the four GEMM launches of one block, per image:
# one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of the four
# GEMM launches of block 0 of a 16-image trunk, whose fp32 residual (340 MB)
# is beyond the L2 (QKV 643 + proj 796 + fc1 916 + fc2 1752 MB;
# profiles/gemm_pair_16img.md), scaled by the images a launch processes.
GEMM_DRAM_BYTES_PER_IMAGE_LAYER = 4107e6 / 16


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
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
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


# --------------------------------------------------------------- ours ---

def run_ours(a):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup(a.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    # A real (non-default) stream: the trunk, torch's events and the gather
    # all run on it.
    with torch.cuda.stream(torch.cuda.Stream(dev)):
        _run_ours(a, torch, dist, world, rank, local, dev)


def _run_ours(a, torch, dist, world, rank, local, dev):

    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as syn

    if a.images % world:
        raise SystemExit("--images must be divisible by --gpus")
    per = a.images // world

    # model files: rank 0 writes them (cached), the others wait
    if rank == 0:
        path = syn.synthetic_gguf(a.format)
        if a.format == "f16" and not a.no_extras:
            syn.synthetic_gguf("q8_0")
    if world > 1:
        dist.barrier()
    path = syn.synthetic_gguf(a.format)
    t_load = time.perf_counter()
    model = s3t.GgufModel(path, device=local)
    load_s = time.perf_counter() - t_load   # GGUF read + upload + fp16 conversion, once per context
    trunk = s3t.VisionTrunk(model)

    imgs_host = torch.from_numpy(syn.synthetic_images(per, start=rank * per)).pin_memory()
    imgs = imgs_host.to(dev)
    out = torch.empty((per, 1024, 72, 72), dtype=torch.float32, device=dev)
    gathered = torch.empty((world, per, 1024, 72, 72), device=dev) if (rank == 0 and world > 1) else None
    stream = torch.cuda.current_stream(dev)
    # N > 1: the shard runs in GATHER_CHUNKS pieces, and each piece's features
    # go to rank 0 (NCCL point-to-point) while the next piece computes.
    chunks = shard_pieces(per, world)
    img_elems, out_elems = 3 * 1008 * 1008, 1024 * 72 * 72

    def gather_piece(i0, i1):
        return gather_piece_to_rank0(rank, world, out, gathered, i0, i1)

    def step(gather=True):
        reqs = []
        for i0, i1 in chunks:
            trunk.run_device(imgs.data_ptr() + i0 * img_elems * 4, i1 - i0, out.data_ptr() + i0 * out_elems * 4,
                             stream.cuda_stream)
            if world > 1 and gather:
                reqs += gather_piece(i0, i1)
        for r in reqs:
            r.wait()
        if world > 1 and gather and rank == 0:
            gathered[0].copy_(out, non_blocking=True)

    def gather_only():
        reqs = []
        for i0, i1 in chunks:
            reqs += gather_piece(i0, i1)
        for r in reqs:
            r.wait()

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    for _ in range(a.warmup):
        step()
    trunk.sync(stream.cuda_stream)
    with ClockSampler(local) as clk:
        total_ms = timed(step, a.steps)
    trunk.sync(stream.cuda_stream)
    ms_step = total_ms / a.steps
    value = a.images * a.steps / (total_ms / 1e3)
    # the same step's parts on their own (not overlapped): trunk only, gather only
    parts = {}
    if world > 1:
        k = max(1, min(a.steps, 5))
        parts["trunk_only_ms_per_step"] = round(timed(lambda: step(gather=False), k) / k, 3)
        parts["gather_only_ms_per_step"] = round(timed(gather_only, k) / k, 3)

    # e2e: public API with pinned host buffers (H2D + trunk + D2H per step)
    out_host = torch.empty((per, 1024, 72, 72), dtype=torch.float32).pin_memory()

    def e2e_step():
        trunk.run_device(imgs_host.data_ptr(), per, out_host.data_ptr(), stream.cuda_stream,
                         images_on_device=False, output_on_device=False)

    for _ in range(max(1, a.warmup // 2)):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_ms = timed(e2e_step, a.steps)
    e2e_wall = time.perf_counter() - t0
    e2e_value = a.images * a.steps / (e2e_ms / 1e3)

    # per-kernel device time of the trunk's own launches at this shape: one
    # eager pass with a CUDA event after every launch, right after the timed region
    prof = trunk.profile(imgs.data_ptr(), per, out.data_ptr(), stream.cuda_stream)

    # Q8_0 weights, same sharding and gather, fewer steps
    q8 = {}
    if a.format == "f16" and not a.no_extras:
        qmodel = s3t.GgufModel(syn.synthetic_gguf("q8_0"), device=local)
        trunk_f16, trunk = trunk, s3t.VisionTrunk(qmodel)
        k = max(1, min(a.steps, 5))
        step()
        q8_ms = timed(step, k) / k
        trunk.sync(stream.cuda_stream)
        trunk = trunk_f16
        q8 = {"q8_0": {"value": round(a.images / (q8_ms / 1e3), 3), "unit": "images/s", "ms_per_step": round(q8_ms, 3),
                       "steps": k}}
        qmodel.close()

    extras = {}
    if rank == 0 and world == 1 and not a.no_extras:
        extras = config_extras(torch, dev, stream, trunk, syn, s3t)

    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    bf16_peak, bf16_sus, hbm_peak, peak_kind = measured_peaks()
    layers = prof["qkv"][1]
    per_gemm = {k: prof[k][0] / max(prof[k][1], 1) for k in ("qkv", "proj", "fc1", "fc2")}
    gemm_ms = sum(per_gemm.values())                     # one block's four GEMM launches
    gemm_flop = GEMM_FLOP_PER_IMAGE_LAYER * per
    achieved = gemm_flop / (gemm_ms / 1e3) / 1e12
    attn = {}
    for kind, key, n_groups, L in (("windowed", "attn_windowed", 9 * per, 576), ("global", "attn_global", per, 5184)):
        ms, n = prof[key]
        if n:
            flop = 4.0 * n_groups * 16 * L * L * 64
            attn[kind] = {"ms": round(ms / n, 4), "tflops": round(flop / (ms / n / 1e3) / 1e12, 1), "launches": n}
    ln_ms, ln_n = prof["layernorm"]
    ln_bytes = per * 5184 * 1024 * 6                     # read fp32 residual, write fp16 operand
    norm = {"ms": round(ln_ms / max(ln_n, 1), 4), "launches": ln_n,
            "gbs": round(ln_bytes / (ln_ms / max(ln_n, 1) / 1e3) / 1e9, 1)}
    norm["frac_of_hbm"] = round(norm["gbs"] / hbm_peak, 4)
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "images/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms_step, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16" if a.format != "q8_0" else "q8_0->f16",
        "data": "synthetic (seeded random-init SAM 3 trunk weights, uniform[-1,1] images)",
        "config": {
            "workload": f"SAM 3 ViT trunk, {a.format.upper()} GGUF, {a.images} images 3x1008x1008 sharded by image "
                        f"({per}/GPU), outputs gathered to rank 0",
            "format": a.format, "global_batch": a.images, "per_gpu_batch": per, "tokens_per_image": 5184,
            "layers": 32, "parallelism": f"image-sharded x{world}",
            "l2_policy": "inputs and activations far larger than the 126 MB L2; no flush",
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "gemm_pair_kernel: the trunk's QKV+RoPE, proj+residual, fc1+GELU, fc2+residual "
                      "launches of one block (M=%d), per-launch CUDA events, averaged over %d blocks"
                      % (per * 5184, layers),
            "achieved": round(achieved, 1), "peak": bf16_peak, "unit": "TFLOP/s",
            "frac": round(achieved / bf16_peak, 4), "peak_kind": f"{peak_kind} bf16 burst",
            "frac_of_sustained": round(achieved / bf16_sus, 4) if bf16_sus else None,
            "traffic": GEMM_DRAM_BYTES_PER_IMAGE_LAYER * per,
            "traffic_note": "DRAM bytes of one block's four GEMM launches: ncu capture at 16 images "
                            "(profiles/gemm_pair_16img.md) scaled by images",
            "per_gemm_ms": {k: round(v, 4) for k, v in per_gemm.items()},
            "trunk_tensor_frac": round(FLOP_PER_IMAGE * value / world / 1e12 / bf16_peak, 4),
        },
        "e2e": {"value": round(e2e_value, 3), "unit": "images/s",
                "h2d_bytes_per_step": int(imgs_host.numel() * 4 * world),
                "d2h_bytes_per_step": int(out_host.numel() * 4 * world),
                "wall_s": round(e2e_wall, 3)},
        "clocks": (clocks := clk.summary()),
        # step time x median SM clock: comparable across runs whose power-capped clocks differ
        "ms_per_step_x_sm_ghz": round(ms_step * clocks["sm_mhz"] / 1e3, 3) if clocks["sm_mhz"] else None,
        "gpu_launches": LAUNCHES_PER_TRUNK * len(chunks) * a.steps * world,
        **parts,
        **q8,
        "attention": attn,
        "layernorm": norm,
        "trunk_profile_ms": {k: round(v[0], 3) for k, v in prof.items()},
        "model_load_s": round(load_s, 3),
        **extras,
    }
    if world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a.format)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _event_ms(torch, dev, stream, fn, warm, reps):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / reps


def attention_microbench(torch, dev, stream, images=32):
    """Attention-only microbenchmark in bf16 with axial RoPE on Q and K:
    windowed (images x 9 windows x 576 tokens x 16 heads x d64) and global
    (images x 5184 tokens x 16 heads x d64), Q/K/V ~ N(0, 1) from seed 5."""
    import ctypes as C
    from sam3cpp_b200 import lib, check
    L = lib()
    peak = measured_peaks()[0]
    g = torch.Generator(device=dev).manual_seed(5)
    res = {}
    for kind, (groups, Lk, win) in {"windowed": (9 * images, 576, 1), "global": (images, 5184, 0)}.items():
        q, k, v = (torch.randn((groups * 16, Lk, 64), generator=g, device=dev, dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty((images * 5184, 1024), device=dev, dtype=torch.bfloat16)
        sp = C.c_void_p(stream.cuda_stream)

        def rope():
            check(L.s3t_rope(dev.index, C.c_void_p(q.data_ptr()), groups, Lk, win, 1, sp))
            check(L.s3t_rope(dev.index, C.c_void_p(k.data_ptr()), groups, Lk, win, 1, sp))

        def attn():
            check(L.s3t_attention(dev.index, C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                  C.c_void_p(v.data_ptr()), groups, Lk, win, 1, C.c_void_p(o.data_ptr()), sp))

        ms_attn = _event_ms(torch, dev, stream, attn, 3, 10)
        ms_both = _event_ms(torch, dev, stream, lambda: (rope(), attn()), 2, 5)
        flop = 4.0 * groups * 16 * Lk * Lk * 64
        res[kind] = {"shape": f"{groups}x16x{Lk}x64", "attention_ms": round(ms_attn, 4),
                     "tflops": round(flop / (ms_attn / 1e3) / 1e12, 1),
                     "frac_of_bf16_peak": round(flop / (ms_attn / 1e3) / 1e12 / peak, 4),
                     "with_rope_ms": round(ms_both, 4)}
        del q, k, v, o
    check(L.s3t_device_status(dev.index))
    return res


def encoder_attention_extras(torch, dev, stream, s3t, images=4):
    """The encoder fusion's and decoder's attention (s3t_mha_d32: 8 heads of
    32): encoder self attention over the 72x72 image tokens of `images` images
    (one batched launch, no mask; and one launch per image, the reference's
    batch of 1), image-to-prompt cross attention (5184 queries, 33 prompt keys
    of which 9 are masked), and the decoder's self attention (201 queries) and
    image cross attention (201 x 5184 with a full box bias).  fp16 q/k/v ~
    N(0, 1.5^2), bias ~ N(0, 2^2), seed 6."""
    peak = measured_peaks()[0]
    g = torch.Generator(device=dev).manual_seed(6)
    T = 5184
    q, k, v = ((torch.randn((images, T, 256), generator=g, device=dev) * 1.5).half() for _ in range(3))
    o = torch.empty((images, T, 256), device=dev)
    kp, vp = ((torch.randn((33, 256), generator=g, device=dev) * 1.5).half() for _ in range(2))
    mask = torch.zeros(33, device=dev)
    mask[24:] = float("-inf")
    op = torch.empty((T, 256), device=dev)
    sp = stream.cuda_stream

    def self_attn():
        s3t.mha_d32(dev.index, q.data_ptr(), k.data_ptr(), v.data_ptr(), images, T, T, None, o.data_ptr(), 0, sp)

    def self_attn_per_image():
        for i in range(images):
            s3t.mha_d32(dev.index, q[i].data_ptr(), k[i].data_ptr(), v[i].data_ptr(), 1, T, T, None,
                        o[i].data_ptr(), 0, sp)

    def cross_attn():
        s3t.mha_d32(dev.index, q[0].data_ptr(), kp.data_ptr(), vp.data_ptr(), 1, T, 33, mask.data_ptr(),
                    op.data_ptr(), 0, sp)

    # The decoder's 201 queries: self attention, and the image cross attention
    # against the 5184 tokens with a full [8][201][5184] box bias (S3T_MHA_BIAS).
    NQ = 201
    dq = (torch.randn((NQ, 256), generator=g, device=dev) * 1.5).half()
    bias = torch.randn((8, NQ, T), generator=g, device=dev) * 2.0

    def dec_self():
        s3t.mha_d32(dev.index, dq.data_ptr(), dq.data_ptr(), dq.data_ptr(), 1, NQ, NQ, None, op.data_ptr(), 0, sp)

    def dec_image():
        s3t.mha_d32(dev.index, dq.data_ptr(), k[0].data_ptr(), v[0].data_ptr(), 1, NQ, T, bias.data_ptr(),
                    op.data_ptr(), s3t.MHA_BIAS, sp)

    ms_self = _event_ms(torch, dev, stream, self_attn, 3, 10)
    ms_one = _event_ms(torch, dev, stream, self_attn_per_image, 3, 10)
    ms_cross = _event_ms(torch, dev, stream, cross_attn, 3, 20)
    ms_dec_self = _event_ms(torch, dev, stream, dec_self, 3, 20)
    ms_dec_image = _event_ms(torch, dev, stream, dec_image, 3, 20)
    check_status = s3t.lib().s3t_device_status(dev.index)
    flop = 4.0 * images * T * T * 32 * 8
    tf = flop / (ms_self / 1e3) / 1e12
    return {"self_shape": f"{images}x{T}x{T}x8x32", "self_ms": round(ms_self, 4), "self_tflops": round(tf, 1),
            "self_frac_of_bf16_peak": round(tf / peak, 4),
            "self_one_launch_per_image_tflops": round(flop / (ms_one / 1e3) / 1e12, 1),
            "cross_shape": f"{T}x33(9 masked)x8x32", "cross_ms": round(ms_cross, 4),
            "decoder_self_shape": f"{NQ}x{NQ}x8x32", "decoder_self_ms": round(ms_dec_self, 4),
            "decoder_image_shape": f"{NQ}x{T}x8x32 + bias", "decoder_image_ms": round(ms_dec_image, 4),
            "decoder_image_tflops": round(4.0 * NQ * T * 32 * 8 / (ms_dec_image / 1e3) / 1e12, 1),
            "status": check_status}


def config_extras(torch, dev, stream, trunk, syn, s3t):
    """Single-GPU extras: b=1 F16 p50 latency (device in -> device out, and
    host in -> host out by wall clock: the host call returns once the features
    are in host memory), Q8_0 batch-8 throughput and the bf16 attention
    microbenchmark."""
    img = torch.from_numpy(syn.synthetic_images(1)).to(dev)
    out = torch.empty((1, 1024, 72, 72), device=dev)
    lat = []
    for i in range(110):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        trunk.run_device(img.data_ptr(), 1, out.data_ptr(), stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if i >= 10:
            lat.append(e0.elapsed_time(e1))
    res = {"latency_b1_p50_ms": round(statistics.median(lat), 3),
           "latency_b1_p90_ms": round(sorted(lat)[int(0.9 * len(lat))], 3)}
    # the same from pinned host image to pinned host features (H2D 12.2 MB, D2H 21.2 MB)
    img_h = img.cpu().pin_memory()
    out_h = torch.empty((1, 1024, 72, 72)).pin_memory()
    lat_h = []
    for i in range(60):
        t0 = time.perf_counter()
        trunk.run_device(img_h.data_ptr(), 1, out_h.data_ptr(), stream.cuda_stream, images_on_device=False,
                         output_on_device=False)
        if i >= 10:
            lat_h.append((time.perf_counter() - t0) * 1e3)
    res["latency_b1_host_p50_ms"] = round(statistics.median(lat_h), 3)
    try:
        qm = s3t.GgufModel(syn.synthetic_gguf("q8_0"), device=dev.index)
        qt = s3t.VisionTrunk(qm)
        imgs = torch.from_numpy(syn.synthetic_images(8)).to(dev)
        o8 = torch.empty((8, 1024, 72, 72), device=dev)
        fn = lambda: qt.run_device(imgs.data_ptr(), 8, o8.data_ptr(), stream.cuda_stream)
        ms = _event_ms(torch, dev, stream, fn, 3, 10)
        qt.sync(stream.cuda_stream)
        res["q8_0_b8_images_per_s"] = round(8 / (ms / 1e3), 2)
        qm.close()
    except Exception as e:  # reported, not fatal for the headline line
        res["q8_0_b8_error"] = str(e)
    res["attention_microbench_bf16"] = attention_microbench(torch, dev, stream)
    try:
        res["encoder_attention_fp16"] = encoder_attention_extras(torch, dev, stream, s3t)
    except Exception as e:  # reported, not fatal for the headline line
        res["encoder_attention_error"] = str(e)
    res["rgb8"] = rgb8_extras(torch, dev, stream, trunk, s3t)
    try:
        res["neck_first"] = neck_extras(torch, dev, stream, syn, s3t)
    except Exception as e:  # reported, not fatal for the headline line
        res["neck_first_error"] = str(e)
    return res


def neck_extras(torch, dev, stream, syn, s3t, batch=8):
    """The hand-off to the vision neck (s3t_neck_first): each level's first
    operation on an 8-image trunk output left on the device (seeded F16 file
    with the neck; 2 trunk layers, which do not change the neck's work)."""
    model = s3t.GgufModel(syn.synthetic_gguf("f16", seed=0, layers=2, perturb=True, neck=True), device=dev.index)
    trunk = s3t.VisionTrunk(model)
    imgs = torch.from_numpy(syn.synthetic_images(batch)).to(dev)
    feats = torch.empty((batch, 1024, 72, 72), device=dev)
    trunk.run_device(imgs.data_ptr(), batch, feats.data_ptr(), stream.cuda_stream)
    res = {"batch": batch}
    for level in range(4):
        shape = trunk.neck_first_shape(level)
        out = torch.empty((batch,) + tuple(shape[1:]), device=dev)
        fn = lambda: trunk.neck_first_device(level, feats.data_ptr(), batch, out.data_ptr(), stream.cuda_stream)
        ms = _event_ms(torch, dev, stream, fn, 3, 20)
        oc, side = shape[1], shape[2]
        rows = oc * (4 if level < 2 else 1)
        positions = (36 * 36 if level == 3 else 5184) * batch
        flop = 2.0 * positions * 1024 * rows
        res[f"level{level}"] = {"out": f"{batch}x{oc}x{side}x{side}", "ms": round(ms, 4),
                                "tflops": round(flop / (ms / 1e3) / 1e12, 1)}
    trunk.sync(stream.cuda_stream)
    model.close()
    return res


def rgb8_extras(torch, dev, stream, trunk, s3t, batch=8, height=1080, width=1920):
    """Decoded 8-bit frames (1920x1080, seeded uniform bytes) through the
    reference's load_image_rgb preprocessing on the device: the preprocess
    kernel alone (device in/out) and the whole uint8-in -> features-out run."""
    import numpy as np
    rgb_host = torch.from_numpy(np.random.default_rng(3).integers(0, 256, (batch, height, width, 3),
                                                                  dtype=np.uint8)).pin_memory()
    rgb = rgb_host.to(dev)
    img = torch.empty((batch, 3, 1008, 1008), device=dev)
    out = torch.empty((batch, 1024, 72, 72), device=dev)
    pre = lambda: s3t.preprocess_rgb8(dev.index, rgb.data_ptr(), width, height, batch, img.data_ptr(),
                                      stream.cuda_stream)
    ms_pre = _event_ms(torch, dev, stream, pre, 3, 20)
    run = lambda: trunk.run_rgb8_device(rgb.data_ptr(), width, height, batch, out.data_ptr(), stream.cuda_stream)
    ms_run = _event_ms(torch, dev, stream, run, 2, 5)
    trunk.sync(stream.cuda_stream)
    written = batch * 3 * 1008 * 1008 * 4
    return {"frame": f"{width}x{height} uint8 RGB", "batch": batch,
            "preprocess_ms": round(ms_pre, 4), "preprocess_gbs": round(written / (ms_pre / 1e3) / 1e9, 1),
            "trunk_from_rgb8_images_per_s": round(batch / (ms_run / 1e3), 2)}


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_build():
    """The reference's CPU trunk as its CMake builds it by default
    (GGML_NATIVE: -march=native; oracle/_ref/libsam3ref_native.so) when this
    host has the build host's ISA extensions, else the AVX-512 / AVX2 build;
    and the host's physical core count, the thread count it runs with."""
    from oracle.pyoracle import Reference, physical_cores, reference_path
    return Reference(reference_path(prefer_native=True)), physical_cores()


def cpu_baseline(fmt):
    """The reference's own CPU trunk (oracle/_ref: ggml CPU backend compiled
    from the reference sources) on one image, one thread per physical core,
    and at its as-shipped 4 threads."""
    try:
        from sam3cpp_b200 import synthetic as syn
        ref, threads = reference_build()
        path, img = syn.synthetic_gguf(fmt), syn.synthetic_image(0)
        _, sec = ref.trunk(path, img, threads)
        # also at the reference's as-shipped thread count (GGML_DEFAULT_N_THREADS = 4)
        _, sec4 = ref.trunk(path, img, 4)
        return {"value": round(1.0 / sec, 5), "unit": "images/s", "cores": threads, "kind": "reference",
                "sample": f"1 image, sam3::VisionTrunk::run ({fmt.upper()} GGUF), {sec:.1f} s, "
                          f"{ref.path.name}, {threads} threads = physical cores "
                          f"({os.cpu_count()} logical CPUs)",
                "cpu_model": _cpu_model(),
                "as_shipped_4_threads": {"value": round(1.0 / sec4, 5), "seconds": round(sec4, 2)}}
    except Exception as e:
        return {"value": None, "unit": "images/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"unavailable: {e}"}


# ------------------------------------------------------------ reference ---

def run_reference(a):
    world, rank, _ = dist_setup(a.gpus)
    if rank != 0:
        return
    from sam3cpp_b200 import synthetic as syn
    ref, threads = reference_build()
    path = str(syn.synthetic_gguf(a.format))
    img = syn.synthetic_image(0)
    import ctypes as C
    h = ref.lib.ref_model_load(path.encode(), threads)
    if not h:
        print(json.dumps({"impl": "reference", "unavailable": ref.lib.ref_last_error().decode()}))
        return
    out = np.empty((1, 1024, 72, 72), np.float32)
    sec = C.c_double()

    def one():
        rc = ref.lib.ref_model_run(h, img.ctypes.data, out.ctypes.data, C.byref(sec))
        if rc != 0:
            raise RuntimeError(ref.lib.ref_last_error().decode())
        return sec.value

    # One reference step is one image through sam3::VisionTrunk::run (tens of
    # seconds on the host cores), so warm-up is capped at 1 and the timed
    # steps at what fits ~150 s.
    warm = min(a.warmup, 1)
    t_first = None
    for _ in range(warm):
        t_first = one()
    if t_first is None:
        t_first = one()
    k = max(1, min(a.steps, int(150.0 / max(t_first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(k):
        one()
    total = time.perf_counter() - t0
    ref.lib.ref_model_free(h)
    value = k / total
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "images/s", "n_gpus": a.gpus,
        "steps": k, "steps_requested": a.steps, "warmup": warm, "ms_per_step": round(total / k * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (ggml CPU)",
        "data": "synthetic (seeded random-init SAM 3 trunk weights, uniform[-1,1] images)",
        "config": {"workload": f"SAM 3 ViT trunk, {a.format.upper()} GGUF, 1 image per step (sample of the "
                               f"{a.images}-image batch), ggml CPU backend ({ref.path.name}), {threads} threads "
                               f"= physical cores", "format": a.format},
        "cpu_baseline": {"value": round(value, 5), "unit": "images/s", "cores": threads, "kind": "reference",
                         "sample": f"{k} image(s) through sam3::VisionTrunk::run ({ref.path.name})"},
        "e2e": {"value": round(value, 5), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def shard_pieces(per: int, world: int, pieces: int = GATHER_CHUNKS) -> list[tuple[int, int]]:
    """The [i0, i1) image ranges of one rank's shard of `per` images: one range
    at N = 1, else up to `pieces` ranges of at least MIN_PIECE images whose
    gathers overlap the next range's compute.  Smaller pieces cost more trunk
    time (2 images: 6.8 ms per image, 4: 6.45, 64: 6.0) than the exposed
    gather of the last piece (21 MB per image over NVLink) saves."""
    if world <= 1:
        return [(0, per)]
    pieces = max(1, min(pieces, per // MIN_PIECE))
    ranges = [(i * per // pieces, (i + 1) * per // pieces) for i in range(pieces)]
    return [r for r in ranges if r[1] > r[0]]


def gather_piece_to_rank0(rank: int, world: int, out, gathered, i0: int, i1: int):
    """Images [i0, i1) of every rank's `out` [per, ...] into rank 0's
    `gathered` [world, per, ...] (row r from rank r) by point-to-point sends;
    returns the requests.  Rank 0's own rows are copied by the caller."""
    import torch.distributed as dist

    if rank == 0:
        ops = [dist.P2POp(dist.irecv, gathered[r, i0:i1], r) for r in range(1, world)]
    else:
        ops = [dist.P2POp(dist.isend, out[i0:i1], 0)]
    return dist.batch_isend_irecv(ops)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--format", default="f16", choices=["f16", "q8_0", "f32"])
    ap.add_argument("--images", type=int, default=64)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--encoder-attention-only", action="store_true",
                    help="time only the encoder-fusion attention (s3t_mha_d32) and print its numbers")
    a = ap.parse_args()
    if a.encoder_attention_only:
        import torch
        import sam3cpp_b200 as s3t
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            print(json.dumps({"encoder_attention_fp16": encoder_attention_extras(torch, dev, stream, s3t,
                                                                                 images=a.images)}))
        return
    if a.warmup < 3 and a.impl == "ours":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
