"""Shared builders for the GPU tests and the bench: a complete noisy-GEMM
problem laid out the way the reference's callers lay it out
(miner/vllm-miner/src/vllm_miner/gemm_operators.py:68-333)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

import pearl_b200 as pg


@dataclass
class Problem:
    m: int
    n: int
    k: int
    r: int
    A: torch.Tensor
    B: torch.Tensor
    key_a: torch.Tensor
    key_b: torch.Tensor
    A_scales: torch.Tensor
    B_scales: torch.Tensor
    noise: dict
    out: dict


def seeded_operands(m, n, k, seed, lo=-64, hi=63):
    g = torch.Generator().manual_seed(seed)
    A = torch.randint(lo, hi + 1, (m, k), generator=g, dtype=torch.int8)
    B = torch.randint(lo, hi + 1, (n, k), generator=g, dtype=torch.int8)
    return A, B


def random_key(seed: int) -> bytes:
    return np.random.default_rng(seed).integers(0, 256, 32, dtype=np.uint8).tobytes()


def make_problem(m, n, k, r=128, seed=0, device="cuda", scales="const", int32_factors=False):
    A, B = seeded_operands(m, n, k, seed)
    ka, kb = random_key(seed + 1000), random_key(seed + 2000)
    dev = torch.device(device)
    key_a = torch.frombuffer(bytearray(ka), dtype=torch.uint8).to(dev)
    key_b = torch.frombuffer(bytearray(kb), dtype=torch.uint8).to(dev)
    if scales == "const":
        sa = torch.full((m,), 1.0 / 128, dtype=torch.float32)
        sb = torch.full((n,), 1.0 / 128, dtype=torch.float32)
    else:
        g = torch.Generator().manual_seed(seed + 7)
        sa = torch.rand(m, generator=g, dtype=torch.float32) / 64
        sb = torch.rand(n, generator=g, dtype=torch.float32) / 64
    e = lambda *s, dt=torch.int8: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
    noise = dict(EAL=e(m, r), EBR=e(n, r), EAR_R_major=e(k, r), EBL_R_major=e(k, r),
                 EAR_K_major=e(r, k), EBL_K_major=e(r, k), EAL_fp16=e(m, r, dt=torch.float16),
                 EBR_fp16=e(n, r, dt=torch.float16))
    out = dict(ApEA=e(m, k), BpEB=e(n, k), AxEBL_fp16=e(m, r, dt=torch.float16),
               EARxBpEB_fp16=e(n, r, dt=torch.float16), C=e(m, n, dt=torch.bfloat16))
    if int32_factors:
        out["AxEBL_int32"] = torch.zeros(m, r, dtype=torch.int32, device=dev)
        out["EARxBpEB_int32"] = torch.zeros(n, r, dtype=torch.int32, device=dev)
    return Problem(m, n, k, r, A.to(dev), B.to(dev), key_a, key_b, sa.to(dev), sb.to(dev), noise, out)


def gen_noise(p: Problem) -> None:
    pg.noise_gen(R=p.r, key_A=p.key_a, key_B=p.key_b, **p.noise)


def signal_buffers(device="cuda"):
    header = torch.zeros(pg.get_host_signal_header_size(), dtype=torch.int8, pin_memory=True)
    sync = torch.zeros(pg.get_host_signal_sync_size(), dtype=torch.int8, device=device)
    return header, sync


def run_noisy_gemm(p: Problem, target: int, header=None, sync=None, **kw) -> tuple:
    if header is None:
        header, sync = signal_buffers(p.A.device)
    pg.noisy_gemm(
        A=p.A, B=p.B, A_scales=p.A_scales, B_scales=p.B_scales,
        host_signal_header_pinned=header, host_signal_sync=sync,
        pow_target=pg.make_pow_target_tensor(target, p.A.device),
        pow_key=p.key_a.view(torch.uint32), **p.noise, **p.out, **kw)
    return header, sync
