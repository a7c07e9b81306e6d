"""The mined GEMM on FP8 operands (C ABI pb2_mined_gemm_fp8).

The protocol mines 7-bit integer GEMMs only (zk-pow/src/api/proof.rs:23-25)
and the reference's one FP8 GEMM, the MoE layer's GEMM2
(miner/vllm-miner/src/vllm_miner/pearl_moe_experts.py:377-434), is not mined.
This build extends the mined contraction to FP8: E4M3 (or E5M2) operands with
per-tensor scales on kind::f8f6f4 tensor-core MMAs with f32 accumulators,
the transcript folded from the accumulators' f32 bit patterns on the
protocol's hash tiles and R-chunk cadence, keyed BLAKE3 and the target
compare, and C = bf16(S * A_scale * B_scale).  There is no noise: FP8 has no
protocol noise definition.  The tensor core's f32 accumulation order is not
specified, so the transcript can be reproduced off the device only for
operands whose partial sums are exact (integer values, |sums| < 2^24)."""

from __future__ import annotations

import torch

from . import _lib
from .pearl_gemm_interface import _check_common, _check_tensor, _device_index, _fail, _ptr, _stream

FORMATS = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}


def mined_gemm_fp8(A, B, A_scale, B_scale, C, host_signal_header_pinned, host_signal_sync, pow_target, pow_key,
                   *, r: int = 128, skip_reduction: bool = False, hits=None, transcripts=None, digests=None):
    """A (m, k), B (n, k): float8_e4m3fn or float8_e5m2 (the same for both);
    A_scale, B_scale: one float32 each; C (m, n) bf16; the signalling buffers,
    target, key and the optional hit list and transcript / digest dumps as
    for ``noisy_gemm``."""
    if A.dtype not in FORMATS or B.dtype != A.dtype:
        _fail("A and B must both be float8_e4m3fn or both float8_e5m2")
    m, k = A.shape
    n = B.shape[0]
    _check_tensor(A, (m, k), A.dtype, "A")
    _check_tensor(B, (n, k), B.dtype, "B")
    _check_tensor(C, (m, n), torch.bfloat16, "C")
    _check_tensor(A_scale.reshape(-1), (1,), torch.float32, "A_scale")
    _check_tensor(B_scale.reshape(-1), (1,), torch.float32, "B_scale")
    _check_tensor(pow_target, (8,), torch.uint32, "pow_target")
    _check_tensor(pow_key, (8,), torch.uint32, "pow_key")
    if host_signal_sync is None or not host_signal_sync.is_cuda:
        _fail("host_signal_sync must be on CUDA")
    p = _lib.Fp8GemmParams()
    p.device = _device_index(A)
    p.m, p.n, p.k, p.r = m, n, k, r
    p.A, p.B, p.format = _ptr(A), _ptr(B), FORMATS[A.dtype]
    p.A_scale, p.B_scale, p.C = _ptr(A_scale), _ptr(B_scale), _ptr(C)
    p.host_signal_header_pinned, p.host_signal_sync = _ptr(host_signal_header_pinned), _ptr(host_signal_sync)
    p.pow_target, p.pow_key = _ptr(pow_target), _ptr(pow_key)
    p.skip_reduction = int(bool(skip_reduction))
    if hits is not None:
        _check_common(hits, "hits", (torch.int32, torch.uint32))
        p.hits, p.hit_capacity = _ptr(hits), hits.shape[0]
    for t, words, name in ((transcripts, 16, "transcripts"), (digests, 8, "digests")):
        if t is not None:
            _check_tensor(t, ((m // 2) * (n // 64), words), (torch.int32, torch.uint32), name)
    p.transcripts, p.digests = _ptr(transcripts), _ptr(digests)
    with torch.cuda.device(A.device):
        _lib.call("pb2_mined_gemm_fp8", p, _stream(A.device), "mined_gemm_fp8")


__all__ = ["mined_gemm_fp8", "FORMATS"]
