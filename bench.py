#!/usr/bin/env python
"""Benchmark of the quantfun2 DiT attention hot path on B200.

Workload (one "step"): one Sage-style attention call on Flux-shaped heads --
B=2 sequences x 24 heads x 4608 tokens (4096 image + 512 text) x head_dim 128,
bf16 inputs resident in HBM; Q, V ~ N(0,1), K ~ N(0,1) + per-channel N(0, 3^2)
offset.  The call quantizes Q/K to INT8 (per 64-token block, K smoothed by its
token mean) and V to FP8, then runs the tcgen05 attention kernel (INT8 QK^T,
FP8 PV, fp32 accumulation).  Metric: attention TFLOPS = 4*B*H*S^2*D / time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The JSON line also carries
  "flux_step":   ms per Flux-dev-shaped denoise step (19 double + 38 single blocks,
                 FP8 linears + Sage attention) at 4608 and 16,896 tokens, split over the
                 N ranks with Ulysses head-parallel attention when N > 1;
  "lumina_step": ms per Lumina-Image-2.0-2B-shaped step (INT8 weight-only linears),
                 one sample per rank (batch-parallel), and the 8-sample batch on one GPU;
  "blocksparse": the top-k block-sparse attention workload (S=16384, keep 12.5 %), N=1.

N > 1 is launched by torchrun, one rank per GPU; each rank runs its own B=2
problem (independent sequences, no collective on the data path: weak scaling).
Rank 0 prints one JSON line.  `--impl reference` times the reference's CPU path
(its torch-eager SDPA branch, fp32) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, H, S, D = 2, 24, 4608, 128
WORKLOAD = f"sage attention, B={B} H={H} S={S} (4096 img + 512 txt) D={D}, bf16 io, INT8 QK^T / FP8 PV"
METRIC = "attention TFLOPS (Flux-shaped 4608 tok, Sage INT8 QK / FP8 PV)"
# dram bytes (read + write) of one sage_attn_kernel launch at this workload, from an ncu
# capture of this kernel at this shape (85.074 MB read + 24.418 MB written)
NCU_ATTN_TRAFFIC_BYTES = 109_491_712


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-flux", action="store_true")
    p.add_argument("--no-lumina", action="store_true")
    p.add_argument("--no-blocksparse", action="store_true")
    p.add_argument("--no-bandwidth", action="store_true", help="skip the bandwidth-kernel measurements")
    p.add_argument("--no-cpu-baselines", action="store_true", help="skip the CPU baselines of configs 1, 3, 4, 5")
    p.add_argument("--flux-sides", default="64,128",
                   help="image-token grid sides of the Flux step (64 -> 4608 tokens, 128 -> 16,896)")
    p.add_argument("--profile-kernel", default=None,
                   help="run one kernel's case three times and exit (single-kernel ncu captures)")
    p.add_argument("--profile", action="store_true",
                   help="for ncu runs: no clock soak, no cuBLAS peak, no CPU baseline, no 8-sample Lumina batch")
    return p.parse_args()


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while work runs."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.rows: list[tuple[float, list[str]]] = []
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            ident = str(device_index)
        self.cmd = ["nvidia-smi", f"--id={ident}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "100"]

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float) -> dict:
        rows = [r for (t, r) in self.rows if t0 <= t <= t1 + 0.15]
        window = "timed"
        if len(rows) < 3:  # very short timed region: include the load just before it
            rows = [r for (t, r) in self.rows if t0 - 2.0 <= t <= t1 + 0.15]
            window = "timed+preceding 2 s of the same work"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "window": window}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def fp8_gemm_peak_tflops(dev) -> float | None:
    """cuBLAS e4m3 GEMM throughput (8192^3, best of 10): the dense FP8/INT8 tensor peak
    this pool's B200 reaches through the vendor library, measured in this run."""
    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3)
        del a, b
        return 2.0 * n ** 3 / best / 1e12
    except Exception:
        return None


# --------------------------------------------------------------- reference --
def run_reference(args, rank: int, world: int):
    """The reference's CPU path for this workload: its torch-eager SDPA branch
    (src/models/flux/attn.py:42-43), fp32, on the full B x H x S x D problem each step,
    on all host cores.  Rank 0 alone runs it; the other ranks exit."""
    if rank != 0:
        return
    from oracle.baseline import sdpa_cpu

    for _ in range(max(args.warmup, 0)):
        sdpa_cpu(B, H, S, D)
    tot_t, tot_f, threads = 0.0, 0.0, 1
    for _ in range(args.steps):
        dt, fl, threads = sdpa_cpu(B, H, S, D)
        tot_t += dt
        tot_f += fl
    tflops = tot_f / tot_t / 1e12
    sample = (f"the full workload each step: B={B} x {H} heads x {S} tokens x D={D}, fp32 torch SDPA "
              f"on the host (src/models/flux/attn.py:42-43)")
    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOPS", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": tot_t / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "same_config": True},
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_cpu_baselines() -> dict:
    """CPU baselines of the other benchmark configurations (torch fp32 restatements of the
    reference's eager paths on all host cores; oracle/baseline.py)."""
    from oracle import baseline as cb
    from quantfun2_b200.dit import flux_step_flops
    from quantfun2_b200.lumina import lumina_step_flops

    out = {}
    dt, fl, thr = cb.joint_attention_cpu()
    out["config1_joint_attention_block"] = {
        "ms": dt * 1e3, "tflops": fl / dt / 1e12, "cores": thr, "kind": "port",
        "what": "JointAttention fp32, B=1, S=1024, dim 3072 (24 x 128), RMSNorm q/k, 2-D RoPE, SDPA, best of 3"}
    dt, fl, thr = cb.blocktopk_cpu()
    out["config3_block_topk"] = {
        "ms": dt * 1e3, "tflops": fl / dt / 1e12, "cores": thr, "kind": "port",
        "what": "block top-k, B=1 H=24 S=16384 D=128, keep 16/128 blocks, fp32 (pool, scores, top-k, "
                "softmax over kept blocks)"}
    dt, fl, thr = cb.lumina_block_cpu()
    step = lumina_step_flops(1)
    out["config4_lumina_step"] = {
        "ms": dt * step / fl * 1e3, "block_ms": dt * 1e3, "cores": thr, "kind": "port",
        "what": "one Lumina 2B JointTransformerBlock fp32 at 4352 tokens timed, step extrapolated by FLOPs "
                f"({step:.3e} / {fl:.3e})"}
    td, ts, thr = cb.flux_blocks_cpu()
    out["config5_flux_step_4608"] = {
        "ms": (19 * td + 38 * ts) * 1e3, "double_block_ms": td * 1e3, "single_block_ms": ts * 1e3,
        "tflops": flux_step_flops(4608) / (19 * td + 38 * ts) / 1e12, "cores": thr, "kind": "port",
        "what": "one double and one single Flux block fp32 at 4608 tokens timed, step = 19 x double + 38 x single "
                "(extrapolation)"}
    return out


def _bw_time(fn, iters: int = 10) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / iters


def run_bandwidth_kernels(dev, hbm_gbs: float, prep_s: float) -> dict:
    """Achieved HBM bandwidth of each bandwidth-bound kernel: algorithmic bytes (each input
    read once, each output written once) / CUDA-event time, on inputs of 0.2-1.2 GB (above
    the 126 MB L2) in the DiT steps' row shapes."""
    from quantfun2_b200 import kernels as K
    from quantfun2_b200 import quant as Q
    from quantfun2_b200.attention import block_topk_select
    from quantfun2_b200.dit import flux_position_ids, rope_freqs

    res = {}

    def add(name, kernel, t, nbytes, shape):
        res[name] = {"kernel": kernel, "ms": t * 1e3, "bytes": nbytes, "gbs": nbytes / t / 1e9,
                     "frac_hbm": nbytes / t / 1e9 / hbm_gbs, "shape": shape}

    g = torch.Generator(device=dev).manual_seed(5)
    bf = torch.bfloat16
    add("sage_quantization", "sage_prep_kernel (+ 32-byte memset)", prep_s, 3 * B * H * S * D * 3,
        f"B={B} H={H} S={S} D={D}: q, k, v read once (2 B/elem), codes written (1 B/elem); timed in the main loop")
    # RoPE in place on q and k [8, 4608, 24, 128]
    Bq, L = 8, 4608
    q = torch.randn(Bq, L, 24, 128, device=dev, generator=g).to(bf)
    k = torch.randn(Bq, L, 24, 128, device=dev, generator=g).to(bf)
    fr = rope_freqs(flux_position_ids(Bq, 512, 64, 64, dev), (16, 56, 56))
    t = _bw_time(lambda: K.rope_apply_(q, k, fr, fp16_trig=False))
    add("rope", "rope_kernel", t, 4 * q.numel() * 2 + fr.numel() * 8, "q, k [8, 4608, 24, 128] bf16, in place")
    # fused q/k RMSNorm + RoPE on the QKV projection [4, 4608, 3 x 3072]
    qkv = torch.randn(4, L, 3 * 3072, device=dev, generator=g).to(bf)
    qo = torch.empty(4, L, 24, 128, device=dev, dtype=bf)
    ko, vo = torch.empty_like(qo), torch.empty_like(qo)
    w1 = torch.ones(128, device=dev, dtype=bf)
    t = _bw_time(lambda: K.qkv_norm_rope(qkv, 24, w1, w1, fr[:4], qo, ko, vo))
    add("qkv_norm_rope", "qkv_norm_rope_kernel", t, 2 * qkv.numel() * 2 + fr[:4].numel() * 8,
        "qkv [4, 4608, 9216] bf16 -> q, k, v")
    del q, k, qkv, qo, ko, vo
    # RMSNorm over rows of 2304 (eager and fused rounding)
    x = torch.randn(131072, 2304, device=dev, generator=g).to(bf)
    w = torch.ones(2304, device=dev, dtype=bf)
    t = _bw_time(lambda: K.rmsnorm_apply(x, w, 1e-5))
    add("rmsnorm_eager", "rmsnorm kernel (eager rounding)", t, 2 * x.numel() * 2, "x [131072, 2304] bf16")
    t = _bw_time(lambda: K.rmsnorm_apply(x, w, 1e-5, fused=True))
    add("rmsnorm_fused", "rmsnorm kernel (fused rounding)", t, 2 * x.numel() * 2, "x [131072, 2304] bf16")
    # Lumina gated residual + next norm-modulate: reads y, x; writes x, h
    M = 65536
    xr, yr, hr = (torch.randn(M, 2304, device=dev, generator=g).to(bf) for _ in range(3))
    gate = torch.randn(1, 2304, device=dev, generator=g).to(bf)
    t = _bw_time(lambda: K.rms_gate_residual(xr, yr, hr, M, w, 1e-5, gate, True, w, 1e-5, gate))
    add("rms_gate_residual", "gate_residual_kernel", t, 4 * xr.numel() * 2, "x, y, h [65536, 2304] bf16")
    del x, xr, yr, hr
    # softmax rows of 16384
    sm = torch.randn(16384, 16384, device=dev, generator=g).to(bf)
    t = _bw_time(lambda: K.inplace_softmax(sm))
    add("softmax", "softmax_rows_kernel", t, 2 * sm.numel() * 2, "x [16384, 16384] bf16, in place")
    del sm
    # adaLN LayerNorm + modulate (+ e4m3 quantizer), activation quantizer, code expansion
    xa = torch.randn(36864, 3072, device=dev, generator=g).to(bf)
    mod = torch.randn(1, 6 * 3072, device=dev, generator=g).to(bf)
    sh, sc = mod[:, :3072], mod[:, 3072:6144]
    t = _bw_time(lambda: Q.ln_modulate(xa, sh, sc, 36864, "bf16"))
    add("ln_modulate_bf16", "ln_modulate_warp_kernel", t, 2 * xa.numel() * 2, "x [36864, 3072] bf16 -> bf16")
    t = _bw_time(lambda: Q.ln_modulate(xa, sh, sc, 36864, "e4m3"))
    add("ln_modulate_e4m3", "ln_modulate_warp_kernel (e4m3 out)", t, xa.numel() * 3 + 36864 * 4,
        "x [36864, 3072] bf16 -> e4m3 codes + row scales")
    t = _bw_time(lambda: Q.quantize_rows(xa, "e4m3"))
    add("quantize_rows_e4m3", "quantize_rows_vec_kernel", t, xa.numel() * 3 + 36864 * 4,
        "x [36864, 3072] bf16 -> e4m3 codes + row scales")
    codes, _ = Q.quantize_rows(xa, "int8")
    t = _bw_time(lambda: Q.codes_to_bf16(codes, "int8"))
    add("codes_to_bf16", "codes_to_bf16_vec_kernel", t, codes.numel() * 3, "int8 [36864, 3072] -> bf16")
    # chunk permutation copy (the Ulysses layout change): [P=8, 3, 1, L, 3 heads x 128] bf16
    src = torch.randn(8 * 3 * 4 * 4608 * 3 * 128, device=dev, generator=g).to(bf)
    dst = torch.empty_like(src)
    hb = 3 * 128 * 2
    t = _bw_time(lambda: K.copy_chunks(dst, src, hb, (8, 3, 4 * 4608), (hb, 8 * hb, 3 * 8 * hb),
                                       (3 * 4 * 4608 * hb, 4 * 4608 * hb, hb)))
    add("copy_chunks", "copy_chunks_kernel", t, 2 * src.numel() * 2, "8 x 3 x 18432 chunks of 768 B (170 MB)")
    del xa, codes, src, dst
    # block top-k selection: pooling reads Q and K once
    qs = torch.randn(1, 24, 16384, 128, device=dev, generator=g).to(bf)
    ks = torch.randn(1, 24, 16384, 128, device=dev, generator=g).to(bf)
    t = _bw_time(lambda: block_topk_select(qs, ks, 16))
    add("blocktopk_select", "blocktopk_pool_kernel + blocktopk_select_kernel", t, 2 * qs.numel() * 2,
        "q, k [1, 24, 16384, 128] bf16 read once (pooling); select on 128 x 128 pooled scores")
    del qs, ks
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------- ours --
def make_inputs(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.float32)
    k = torch.randn(B, H, S, D, device=dev, generator=g) + 3.0 * torch.randn(1, H, 1, D, device=dev, generator=g)
    v = torch.randn(B, H, S, D, device=dev, generator=g)
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def run_flux_step(rank: int, world: int, dev, sides=(64, 128), warmup: int = 2, steps: int = 5,
                  mode: str = "fp8_w8a8", check_side: int | None = 64) -> dict:
    """Flux-dev-shaped forwards (19 double + 38 single blocks, hidden 3072, 24 x 128 heads,
    512 txt tokens + a side x side image-token grid, Sage attention; linears FP8 e4m3 W8A8
    by default, "fp8" = the reference's qfloat8 weight-only form): side 64 -> 4608 tokens
    (the metric's shape), side 128 -> 16,896 tokens (2048^2 latent).
    With N ranks the joint sequence is split N ways and attention runs head-parallel
    (Ulysses all-to-all).  At N > 1 and side `check_side`, rank 0 also runs the same
    inputs on one GPU alone: the gathered Ulysses output is compared with it (cosine,
    max-abs) and its time is the strong-scaling reference."""
    from quantfun2_b200.dit import FluxDiT, SeqParallel, flux_position_ids, flux_step_flops, rope_freqs

    T = 512
    if T % world or 24 % world:
        return {"skipped": f"{world} ranks do not divide 512 txt tokens and 24 heads"}
    model = FluxDiT(device=dev, seed=0, mode=mode)
    sp = SeqParallel(torch.distributed.group.WORLD if world > 1 else None)
    linears = ("FP8 e4m3 W8A8 (per-token activation, per-channel weight scales)" if mode == "fp8_w8a8"
               else "FP8 e4m3 weight-only (per-channel scales), bf16 activations")
    out = {}
    for side in sides:
        I = side * side
        g = torch.Generator(device=dev).manual_seed(0)  # identical inputs on every rank
        img = torch.randn(1, I, 64, device=dev, generator=g).bfloat16()
        txt = torch.randn(1, T, 4096, device=dev, generator=g).bfloat16()
        t = torch.rand(1, device=dev, generator=g)
        y = torch.randn(1, 768, device=dev, generator=g).bfloat16()
        freqs = rope_freqs(flux_position_ids(1, T, side, side, dev), (16, 56, 56))
        tl, il = T // world, I // world
        img_l, txt_l = img[:, rank * il:(rank + 1) * il].contiguous(), txt[:, rank * tl:(rank + 1) * tl].contiguous()
        f_l = torch.cat([freqs[:, rank * tl:(rank + 1) * tl], freqs[:, T + rank * il:T + (rank + 1) * il]],
                        1).contiguous()
        fwd = lambda: model(img_l, txt_l, t, y, f_l, sp)  # noqa: E731
        nsteps = steps if I <= 4096 else max(2, steps // 2)
        r = _time_forward(fwd, world, dev, warmup if I <= 4096 else 1, nsteps)
        fl = flux_step_flops(T + I)
        sec = r.pop("sec")
        entry = {"ms_per_step": sec * 1e3, "tflops": fl / sec / 1e12, "flops_per_step": fl, "tokens": T + I, **r,
                 "parallelism": f"ulysses sp{world}" if world > 1 else "single GPU", "linears": linears,
                 "attention": "Sage INT8 QK / FP8 PV"}
        if world > 1 and side == check_side:
            entry.update(_flux_ulysses_check(model, fwd, rank, world, dev, img, txt, t, y, freqs, il, sec))
        out[f"tokens_{T + I}"] = entry
        del img, txt, img_l, txt_l, f_l, freqs
        torch.cuda.empty_cache()
    del model
    torch.cuda.empty_cache()
    return out


def _flux_ulysses_check(model, fwd, rank, world, dev, img, txt, t, y, freqs, il, sec_sp) -> dict:
    """The gathered N-rank output against rank 0's single-GPU forward of the same inputs,
    and rank 0's single-GPU step time (CUDA graph) for the strong-scaling efficiency."""
    from quantfun2_b200.dit import SeqParallel

    with torch.inference_mode():
        o_l = fwd().contiguous()
        parts = [torch.empty_like(o_l) for _ in range(world)]
        torch.distributed.all_gather(parts, o_l)
        res = {}
        if rank == 0:
            o_sp = torch.cat(parts, 1).float()
            single = lambda: model(img, txt, t, y, freqs, SeqParallel(None))  # noqa: E731
            o_1 = single().float()
            cos = torch.nn.functional.cosine_similarity(o_sp.flatten(), o_1.flatten(), dim=0).item()
            res = {"vs_single_gpu": {"cosine": cos, "max_abs": (o_sp - o_1).abs().max().item(),
                                     "ref_max_abs": o_1.abs().max().item(),
                                     "what": "gathered Ulysses output vs rank 0 alone, same inputs and weights"}}
            r1 = _time_forward(single, 1, dev, 2, 5)
            res["single_gpu_ms_per_step"] = r1["sec"] * 1e3
            res["strong_scaling_efficiency"] = r1["sec"] / (world * sec_sp)
            del o_sp, o_1
        torch.distributed.barrier()
    return res


def run_blocksparse(dev, S: int = 16384, H: int = 24, D: int = 128, keep_frac: float = 0.125, warmup: int = 3,
                    steps: int = 10) -> dict:
    """Top-k block-sparse attention at B=1, H=24, D=128, S=16384, bf16, 128-token blocks,
    keeping 12.5 % of the key blocks: block pooling + scores + top-k selection + exact
    softmax attention over the kept blocks.  Seeded inputs: Q, K, V ~ N(0, 1), each query
    block's rows shifted by 2.0 along a random unit direction that 4 random key blocks
    share (the query-aligned hot blocks)."""
    from quantfun2_b200.attention import block_topk_select, blocksparse_attn

    g = torch.Generator(device=dev).manual_seed(0)
    nb = S // 128
    keep = max(1, math.ceil(keep_frac * nb))
    q = torch.randn(1, H, S, D, device=dev, generator=g)
    k = torch.randn(1, H, S, D, device=dev, generator=g)
    v = torch.randn(1, H, S, D, device=dev, generator=g).bfloat16()
    u = torch.randn(1, H, nb, D, device=dev, generator=g)
    u = 2.0 * u / u.norm(dim=-1, keepdim=True)
    q.view(1, H, nb, 128, D).add_(u[:, :, :, None, :])
    hot = torch.rand(1, H, nb, nb, device=dev, generator=g).argsort(dim=-1)[..., :4]  # 4 distinct key blocks
    kadd = torch.zeros(1, H, nb, D, device=dev)
    kadd.scatter_add_(2, hot.reshape(1, H, nb * 4, 1).expand(-1, -1, -1, D),
                      u[:, :, :, None, :].expand(-1, -1, -1, 4, -1).reshape(1, H, nb * 4, D))
    k.view(1, H, nb, 128, D).add_(kadd[:, :, :, None, :])
    q, k = q.bfloat16(), k.bfloat16()
    del kadd, u, hot

    def step():
        idx = block_topk_select(q, k, keep)
        return blocksparse_attn(q, k, v, idx)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    for _ in range(steps):
        idx = block_topk_select(q, k, keep)
    e[1].record()
    for _ in range(steps):
        o = blocksparse_attn(q, k, v, idx)
    e[2].record()
    torch.cuda.synchronize()
    sel = e[0].elapsed_time(e[1]) / steps / 1e3
    att = e[1].elapsed_time(e[2]) / steps / 1e3
    fl = 4.0 * H * S * (keep * 128) * D
    finite = bool(torch.isfinite(o.float()).all())
    del q, k, v, o, idx
    torch.cuda.empty_cache()
    return {"workload": f"B=1 H={H} S={S} D={D} bf16, 128-token blocks, keep {keep}/{nb}",
            "ms_per_step": (sel + att) * 1e3, "select_ms": sel * 1e3, "attention_ms": att * 1e3,
            "kept_attention_flops": fl, "attention_tflops": fl / att / 1e12,
            "step_tflops": fl / (sel + att) / 1e12, "output_finite": finite, "steps": steps}


def _time_forward(fwd, world: int, dev, warmup: int, steps: int) -> dict:
    """Warm up, time `steps` eager forwards, then capture one forward as a CUDA graph and
    time its replays (CUDA events on the launching stream; max over ranks)."""

    def timed(fn):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        sec = e0.elapsed_time(e1) / 1e3 / steps
        if world > 1:
            tt = torch.tensor([sec], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            sec = float(tt[0])
        return sec

    graph_error = None
    with torch.inference_mode():
        for _ in range(warmup):
            fwd()
        eager = timed(fwd)
        # the whole step as one CUDA graph: the thousands of launches of a step replay
        # without host-side launch cost
        graph, sec, out = None, eager, None
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fwd()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = fwd()
            for _ in range(warmup):
                graph.replay()
            sec = timed(graph.replay)
        except Exception as e:  # noqa: BLE001
            graph = None
            out = fwd()
            graph_error = f"{type(e).__name__}: {e}"[:200]
        finite = bool(torch.isfinite(out.float()).all())
    res = {"sec": sec, "steps": steps, "warmup": warmup, "cuda_graph": graph is not None,
           "eager_ms_per_step": eager * 1e3, "output_finite": finite}
    if graph_error:
        res["graph_error"] = graph_error
    del graph
    return res


def run_lumina_step(rank: int, world: int, dev, batch: int = 1, warmup: int = 2, steps: int = 5) -> dict:
    """One Lumina-Image-2.0-2B-shaped forward (26 layers + 2 + 2 refiners, dim 2304, 24 / 8
    heads of 96, SwiGLU 6144, 4096 img + 256 caption tokens, INT8 weight-only linears, Sage
    attention) on `batch` samples per rank.  Ranks are batch-parallel: each denoises its own
    samples, no collective in the step."""
    from quantfun2_b200.lumina import LuminaDiT, lumina_step_flops

    Lc, side = 256, 64
    Li = side * side
    model = LuminaDiT(device=dev, seed=0)
    g = torch.Generator(device=dev).manual_seed(100 + rank)  # each rank its own samples
    img = torch.randn(batch, Li, 64, device=dev, generator=g).bfloat16()
    cap = torch.randn(batch, Lc, 2304, device=dev, generator=g).bfloat16()
    t = torch.rand(batch, device=dev, generator=g)
    freqs = model.make_freqs(batch, Lc, side, side, dev)
    r = _time_forward(lambda: model(img, t, cap, freqs), world, dev, warmup, steps)
    del model
    torch.cuda.empty_cache()
    fl = lumina_step_flops(batch)
    sec = r.pop("sec")
    return {"ms_per_step": sec * 1e3, "tflops_per_gpu": fl / sec / 1e12, "flops_per_step_per_gpu": fl,
            "batch_per_gpu": batch, "global_batch": batch * world, "samples_per_s": batch * world / sec,
            "tokens": Lc + Li, **r, "parallelism": f"batch-parallel dp{world}" if world > 1 else "single GPU",
            "linears": "INT8 weight-only (per-channel scales), bf16 activations",
            "attention": "Sage INT8 QK / FP8 PV, GQA 24/8, head_dim 96"}


def profile_cases(dev) -> dict:
    """One case per kernel for single-kernel ncu captures (`--profile-kernel NAME`): inputs
    of 0.1-1.2 GB (above the 126 MB L2) in the DiT steps' shapes; each case runs its
    kernel(s) three times."""
    from quantfun2_b200 import kernels as K
    from quantfun2_b200 import quant as Q
    from quantfun2_b200.attention import block_topk_select, blocksparse_attn, sageattn
    from quantfun2_b200.dit import flux_position_ids, rope_freqs

    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1)
    rn = lambda *sh: torch.randn(*sh, device=dev, generator=g)  # noqa: E731

    def rope():
        q, k = rn(4, 4608, 24, 128).to(bf), rn(4, 4608, 24, 128).to(bf)
        f = rope_freqs(flux_position_ids(4, 512, 64, 64, dev), (16, 56, 56))
        return lambda: K.rope_apply_(q, k, f, fp16_trig=False)

    def qkv_norm_rope():
        qkv = rn(4, 4608, 9216).to(bf)
        o = [torch.empty(4, 4608, 24, 128, device=dev, dtype=bf) for _ in range(3)]
        w = torch.ones(128, device=dev, dtype=bf)
        f = rope_freqs(flux_position_ids(4, 512, 64, 64, dev), (16, 56, 56))
        return lambda: K.qkv_norm_rope(qkv, 24, w, w, f, *o)

    def rmsnorm():
        x, w = rn(65536, 2304).to(bf), torch.ones(2304, device=dev, dtype=bf)
        return lambda: K.rmsnorm_apply(x, w, 1e-5)

    def softmax():
        x = rn(8192, 16384).to(bf)
        return lambda: K.inplace_softmax(x)

    def gate_residual():
        x, y, h = (rn(65536, 2304).to(bf) for _ in range(3))
        w, gt = torch.ones(2304, device=dev, dtype=bf), rn(1, 2304).to(bf)
        return lambda: K.rms_gate_residual(x, y, h, 65536, w, 1e-5, gt, True, w, 1e-5, gt)

    def ln_modulate():
        x, mod = rn(36864, 3072).to(bf), rn(1, 6144).to(bf)
        return lambda: (Q.ln_modulate(x, mod[:, :3072], mod[:, 3072:], 36864, "bf16"),
                        Q.ln_modulate(x, mod[:, :3072], mod[:, 3072:], 36864, "e4m3"))

    def quantize_rows():
        x = rn(36864, 3072).to(bf)
        return lambda: Q.quantize_rows(x, "e4m3")

    def codes_to_bf16():
        c, _ = Q.quantize_rows(rn(36864, 3072).to(bf), "int8")
        return lambda: Q.codes_to_bf16(c, "int8")

    def quantize_weight():
        w = rn(12288, 3072).half()
        return lambda: Q.quantize_weight(w, "int8")

    def copy_chunks():
        src = rn(8 * 3 * 4 * 4608 * 3 * 128).to(bf)
        dst = torch.empty_like(src)
        hb = 768
        return lambda: K.copy_chunks(dst, src, hb, (8, 3, 4 * 4608), (hb, 8 * hb, 24 * hb),
                                     (3 * 4 * 4608 * hb, 4 * 4608 * hb, hb))

    def sage():
        q, v = rn(2, 24, 4608, 128).to(bf), rn(2, 24, 4608, 128).to(bf)
        k = (rn(2, 24, 4608, 128) + 3 * rn(1, 24, 1, 128)).to(bf)
        return lambda: sageattn(q, k, v)

    def sage_split():   # 3 heads per GPU: split-KV attention + sage_combine_kernel
        q, k, v = (rn(1, 3, 4608, 128).to(bf) for _ in range(3))
        return lambda: sageattn(q, k, v)

    def gemm_fp8():
        a, _ = Q.quantize_rows(rn(4608, 3072).to(bf), "e4m3")
        b, _ = Q.quantize_rows(rn(12288, 3072).to(bf), "e4m3")
        return lambda: Q.gemm(a, b, fp8=True)

    def gemm_bf16_glu():
        a, b = rn(4352, 2304).to(bf), rn(12288, 2304).to(bf)
        return lambda: Q.gemm(a, b, glu=True)

    def gemm_single():   # M <= 128: single-CTA tiles (adaLN linear)
        a, b = rn(1, 3072).to(bf), rn(18432, 3072).to(bf)
        return lambda: Q.gemm(a, b)

    def gemm_codes():    # weight-only int8 codes read directly by the GEMM (M <= 128)
        a = rn(1, 3072).to(bf)
        c, sc = Q.quantize_weight(rn(18432, 3072).to(bf), "int8")
        return lambda: Q.gemm(a, c, col_scale=sc, codes="int8")

    def blocksparse():
        q, k, v = (rn(1, 24, 16384, 128).to(bf) for _ in range(3))
        idx = block_topk_select(q, k, 16)
        return lambda: (block_topk_select(q, k, 16), blocksparse_attn(q, k, v, idx))

    def ras():
        x = rn(2, 2048, 24, 128).to(bf)
        f = rn(2048, 128)
        idx = torch.randperm(4608, device=dev)[:2048]
        y = torch.empty(2, 4608, 24, 128, device=dev, dtype=bf)
        xa, w = rn(2, 2048, 3072).to(bf), rn(3072, 3072).to(bf)
        out = torch.empty(2, 4608, 3072, device=dev, dtype=bf)
        return lambda: (K.rope_scatter(x, f, idx, y), K.partially_linear(xa, w, idx, out=out, check_index=False))

    def lumina_step():   # one Lumina-2B-shaped forward, B=1, eager (launch lists)
        from quantfun2_b200.lumina import LuminaDiT

        m = LuminaDiT(device=dev, seed=0)
        img, cap = rn(1, 4096, 64).to(bf), rn(1, 256, 2304).to(bf)
        t, fr = torch.rand(1, device=dev, generator=g), m.make_freqs(1, 256, 64, 64, dev)
        return lambda: m(img, t, cap, fr)

    def flux_step():     # one Flux-dev-shaped forward at 4608 tokens, eager (launch lists)
        from quantfun2_b200.dit import FluxDiT

        m = FluxDiT(device=dev, seed=0)
        img, txt = rn(1, 4096, 64).to(bf), rn(1, 512, 4096).to(bf)
        t, y = torch.rand(1, device=dev, generator=g), rn(1, 768).to(bf)
        fr = rope_freqs(flux_position_ids(1, 512, 64, 64, dev), (16, 56, 56))
        return lambda: m(img, txt, t, y, fr)

    return {"lumina_step": lumina_step, "flux_step": flux_step, "rope": rope, "qkv_norm_rope": qkv_norm_rope, "rmsnorm": rmsnorm, "softmax": softmax,
            "gate_residual": gate_residual, "ln_modulate": ln_modulate, "quantize_rows": quantize_rows,
            "codes_to_bf16": codes_to_bf16, "quantize_weight": quantize_weight, "copy_chunks": copy_chunks,
            "sage": sage, "sage_split": sage_split, "gemm_fp8": gemm_fp8, "gemm_bf16_glu": gemm_bf16_glu,
            "gemm_single": gemm_single, "gemm_codes": gemm_codes, "blocksparse": blocksparse, "ras": ras}


def run_profile_kernel(name: str, dev) -> None:
    cases = profile_cases(dev)
    if name not in cases:
        raise SystemExit(f"unknown kernel case {name!r}; one of {sorted(cases)}")
    fn = cases[name]()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    print(f"profile case {name}: ok", flush=True)


def run_ours(args, rank: int, world: int, dev):
    from quantfun2_b200 import _lib
    from quantfun2_b200._lib import check, i64, stream_ptr
    from quantfun2_b200.attention import _workspace, sageattn

    lib = _lib.load()
    q, k, v = make_inputs(dev, 1234 + rank)
    out = torch.empty_like(q)
    nbytes = int(lib.qf2_sage_workspace_bytes(B, H, H, B * S, B * S, S, S, D))
    ws = _workspace(nbytes, dev)
    st = lambda t: i64(t.stride(0), t.stride(1), t.stride(2))  # noqa: E731
    sq, sk, sv, so = st(q), st(k), st(v), st(out)
    sm = 1.0 / math.sqrt(D)
    stream = stream_ptr(dev)

    def quant():
        check(lib.qf2_sage_quantize(q.data_ptr(), sq, k.data_ptr(), sk, v.data_ptr(), sv, None, None, B, S, S, 0, 0,
                                    0, 0, H, H, D, sm, _lib.QF2_BF16, ws.data_ptr(), ws.numel(), stream), "quant")

    def attn():
        check(lib.qf2_sage_attn_quantized(out.data_ptr(), so, None, None, B, S, S, 0, 0, 0, 0, H, H, D,
                                          _lib.QF2_BF16, ws.data_ptr(), ws.numel(), stream), "attn")

    flops_step = 4.0 * B * H * S * S * D
    peaks = measured_peaks()
    fp8_peak = fp8_gemm_peak_tflops(dev) if rank == 0 and not args.profile else None

    sampler = ClockSampler(dev.index or 0) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(max(args.warmup, 3)):
        quant()
        attn()
    # keep the GPU busy ~1.5 s before timing so the clock record covers steady load
    t_soak = time.time()
    while not args.profile and time.time() - t_soak < 1.5:
        for _ in range(20):
            quant()
            attn()
        torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for i in range(args.steps):
        quant()
        evs[i][0].record()
        attn()
        evs[i][1].record()
    e_end.record()
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if world > 1:
        torch.distributed.barrier()
    total_s = e_start.elapsed_time(e_end) / 1e3
    attn_s = sum(a.elapsed_time(b) for a, b in evs) / 1e3 / args.steps
    if world > 1:
        t = torch.tensor([total_s, attn_s], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_s, attn_s = float(t[0]), float(t[1])
    clocks = sampler.summary(t_wall0, t_wall1) if sampler else None
    if sampler:
        sampler.stop()

    # ---- end to end through the public API with host buffers.  Every step copies its
    # inputs in from pinned host memory and its output back; the copies of neighbouring
    # steps overlap the attention of this one (in / compute / out streams, two device
    # buffer slots), as a serving loop would run it.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        houts = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
        dins = [tuple(torch.empty_like(x) for x in (q, k, v)) for _ in range(2)]
        douts = [torch.empty_like(out) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        comp = torch.cuda.current_stream(dev)
        e2e_steps = max(2, min(args.steps, 50))
        ev = lambda: torch.cuda.Event()  # noqa: E731
        in_done, comp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]

        def run_e2e(nsteps):
            for i in range(nsteps):
                sl = i & 1
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(comp_done[sl])  # attention of step i - 2 has read this slot
                    for d, hsrc in zip(dins[sl], (hq, hk, hv)):
                        d.copy_(hsrc, non_blocking=True)
                    in_done[sl].record(s_in)
                comp.wait_event(in_done[sl])
                if i >= 2:
                    comp.wait_event(out_done[sl])  # the output of step i - 2 has left this slot
                sageattn(*dins[sl], out=douts[sl])
                comp_done[sl].record(comp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(comp_done[sl])
                    houts[sl].copy_(douts[sl], non_blocking=True)
                    out_done[sl].record(s_out)
            comp.wait_stream(s_in)
            comp.wait_stream(s_out)

        run_e2e(3)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(comp)
        run_e2e(e2e_steps)
        a1.record(comp)
        torch.cuda.synchronize()
        e2e_s = a0.elapsed_time(a1) / 1e3 / e2e_steps
        if world > 1:
            t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_s = float(t[0])
        ok_out = bool(torch.isfinite(houts[(e2e_steps - 1) & 1][:, :1].float()).all())
        e2e = {"value": world * flops_step / e2e_s / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
               "d2h_bytes_per_step": out.numel() * out.element_size(), "ms_per_step": e2e_s * 1e3,
               "steps": e2e_steps, "overlap": "copies of steps i-1 / i+1 overlap step i (3 streams, 2 slots)",
               "output_finite": ok_out}
        del hq, hk, hv, houts, dins, douts

    quant_s = total_s / args.steps - attn_s
    # ---- achieved HBM bandwidth of the bandwidth-bound kernels (one GPU's view; rank 0)
    bandwidth = None
    if world == 1 and not args.profile and not args.no_bandwidth:
        del q, k, v, out, ws
        torch.cuda.empty_cache()
        bandwidth = run_bandwidth_kernels(dev, peaks.get("hbm_gbs") or 6650.0, quant_s)
    # ---- the Flux-shaped denoise step (Ulysses over the ranks when N > 1)
    flux, flux_wo = None, None
    if not args.no_flux:
        if bandwidth is None:
            del q, k, v, out, ws
            torch.cuda.empty_cache()
        flux = run_flux_step(rank, world, dev, sides=tuple(int(x) for x in args.flux_sides.split(",")))
        if world == 1 and not args.profile:
            flux_wo = run_flux_step(rank, world, dev, sides=(64,), mode="fp8")
    # ---- the Lumina-shaped denoise step (batch-parallel: one sample per rank; on one GPU
    # also the 8-sample batch)
    lumina = None
    if not args.no_lumina:
        if flux is None and bandwidth is None:
            del q, k, v, out, ws
            torch.cuda.empty_cache()
        lumina = {"b1_per_gpu": run_lumina_step(rank, world, dev, batch=1)}
        if world == 1 and not args.profile:
            lumina["b8_single_gpu"] = run_lumina_step(rank, world, dev, batch=8, warmup=1, steps=3)
    # ---- top-k block-sparse attention (one GPU's workload; rank 0 only)
    blocksparse = None
    if not args.no_blocksparse and rank == 0:
        blocksparse = run_blocksparse(dev)

    if rank != 0:
        return
    # ---- CPU baseline: the reference's SDPA branch on the same workload (rank 0, N=1 only),
    # and the other configurations' CPU paths
    cpu, cpu_more = None, None
    if world == 1 and not args.profile:
        from oracle.baseline import sdpa_cpu

        sdpa_cpu(1, 2, S, D)
        dt, fl, thr = sdpa_cpu(B, H, S, D)
        cpu = {"value": fl / dt / 1e12, "unit": "TFLOPS", "cores": thr, "kind": "port",
               "sample": f"the full workload, B={B} x {H} heads x {S} tokens x D={D}, fp32 torch SDPA on the "
                         "host (the reference's SDPA branch, src/models/flux/attn.py:42-43), one call",
               "ms": dt * 1e3}
        if not args.no_cpu_baselines:
            cpu_more = run_cpu_baselines()

    per_step = total_s / args.steps
    value = world * flops_step / per_step / 1e12
    attn_tflops = flops_step / attn_s / 1e12
    if fp8_peak:
        peak, peak_src = fp8_peak, "measured in this run: cuBLAS e4m3 GEMM 8192^3 burst (torch._scaled_mm)"
    elif peaks.get("bf16_tflops"):
        peak, peak_src = 2 * peaks["bf16_tflops"], "2 x measured bf16 burst (MEASURED_PEAKS.json)"
    else:
        peak, peak_src = 2 * 1590.0, "2 x fallback bf16 1.59 PFLOP/s"
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8+e4m3", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": S, "heads": H, "head_dim": D,
                   "parallelism": f"independent sequences per rank x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (q+k+v 170 MB + 85 MB of codes per rank)",
                   "step": "qf2_sage_quantize + qf2_sage_attn_quantized (sage_prep_kernel + sage_attn_kernel, and a 32-byte memset)"},
        "roofline": {"bound": "tensor", "achieved": attn_tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": attn_tflops / peak, "traffic": NCU_ATTN_TRAFFIC_BYTES, "kernel": "sage_attn_kernel",
                     "kernel_ms": attn_s * 1e3, "peak_source": peak_src,
                     "frac_of_bf16_measured": (attn_tflops / peaks["bf16_tflops"]) if peaks.get("bf16_tflops")
                     else None},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 2 * args.steps,  # sage_prep_kernel and sage_attn_kernel per step (no KV split at this shape)
        "clocks": clocks,
        "cpu_baselines_other_configs": cpu_more,
        "bandwidth_kernels": bandwidth,
        "lumina_step": lumina,
        "blocksparse": blocksparse,
        "flux_step_weight_only_fp8": flux_wo,
        "flux_step": flux,
    }
    # the Flux step summary last (ms per step, and at N > 1 the single-GPU comparison)
    if flux and "skipped" not in flux:
        line["flux_summary"] = {
            k: {kk: v[kk] for kk in ("ms_per_step", "tflops", "single_gpu_ms_per_step", "strong_scaling_efficiency",
                                     "vs_single_gpu") if kk in v}
            for k, v in flux.items()}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.profile_kernel:
        run_profile_kernel(args.profile_kernel, dev)
        return
    if world > 1:
        from datetime import timedelta

        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        run_ours(args, rank, world, dev)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
