"""CPU baseline of the attention hot path (test / benchmark infrastructure only).

The reference's CPU path for Flux-shaped attention is its SDPA branch,
``F.scaled_dot_product_attention(xq, xk, xv)`` in src/models/flux/attn.py:42-43
(torch-eager, fp32 on the host).  The reference tree itself is not importable on
the GPU box, and that branch is a single torch call, so it is restated here
verbatim as that call; it is timed on a bounded sample of the benchmark workload
(a few heads of one sequence) and scaled to TFLOPS with the same FLOP count as
the GPU path (4 * S_q * S_kv * D per head).
"""
from __future__ import annotations

import os
import time

import torch


def attention_flops(B: int, H: int, Sq: int, Skv: int, D: int) -> float:
    return 4.0 * B * H * Sq * Skv * D


def sdpa_cpu_sample(heads: int = 4, S: int = 4608, D: int = 128, seed: int = 0, threads: int | None = None):
    """Time one call of the reference SDPA branch on `heads` heads of one S-token
    sequence, fp32 on the CPU.  Returns (seconds, flops, threads_used)."""
    if threads is None:
        threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(1, heads, S, D, generator=g)
        k = torch.randn(1, heads, S, D, generator=g) + 3.0 * torch.randn(1, heads, 1, D, generator=g)
        v = torch.randn(1, heads, S, D, generator=g)
        t0 = time.perf_counter()
        torch.nn.functional.scaled_dot_product_attention(q, k, v)
        dt = time.perf_counter() - t0
        return dt, attention_flops(1, heads, S, S, D), torch.get_num_threads()
    finally:
        torch.set_num_threads(prev)
