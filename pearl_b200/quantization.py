"""Mirror of ``pearl_gemm.quantization`` (miner/pearl-gemm/src/pearl_gemm/
quantization/__init__.py, hadamard.py:530-611): the fused block-Hadamard +
smooth-scale + symmetric per-token quantization that turns a layer's bf16 /
fp16 activations into the int7 (max_val 63) or int8 (127) operand of the
mined GEMM.  Runs the B200 kernel in pearl_b200/csrc/quant.cu."""

from __future__ import annotations

import torch

from . import _lib
from .pearl_gemm_interface import _device_index, _fail, _stream

DEFAULT_HADAMARD_BLOCK_SIZE = 16  # hadamard.py:520


def quantize(
    x: torch.Tensor,
    xq: torch.Tensor,
    xq_scales: torch.Tensor,
    smooth_scale: torch.Tensor | None = None,
    max_val: int = 63,
    block_size: int = DEFAULT_HADAMARD_BLOCK_SIZE,
) -> None:
    """xq = rint(v * inv) with v = Hadamard_k(x) * smooth (k = block_size,
    0 = no transform), inv = max_val * rcp.approx(amax_row(v) + 1e-30) and
    xq_scales = amax_row(v) * fl(1 / max_val): the reference's float32 steps
    (hadamard.py:443-466), so the same bytes come out.

    x: (M, N) fp16 / bf16 contiguous; xq: (M, N) int8; xq_scales: (M, 1)
    fp32; smooth_scale: (1, N) broadcast or (M, N) per token, fp32."""
    if x.dim() != 2:
        _fail("x must be 2D (M, N)")
    M, N = x.shape
    if x.dtype not in (torch.bfloat16, torch.float16):
        _fail(f"x must be float16 or bfloat16, got {x.dtype}")
    for t, name in ((x, "x"), (xq, "xq"), (xq_scales, "xq_scales")):
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
    if xq.dtype != torch.int8 or tuple(xq.shape) != (M, N):
        _fail(f"xq must be int8 of shape ({M}, {N})")
    if xq_scales.dtype != torch.float32 or xq_scales.numel() != M:
        _fail(f"xq_scales must be float32 of shape ({M}, 1)")
    per_row = 0
    if smooth_scale is not None:
        if smooth_scale.dtype != torch.float32 or not smooth_scale.is_cuda or not smooth_scale.is_contiguous():
            _fail("smooth_scale must be a contiguous float32 CUDA tensor")
        if smooth_scale.dim() != 2 or smooth_scale.shape[1] != N or smooth_scale.shape[0] not in (1, M):
            _fail(f"smooth_scale must have shape (1, {N}) or ({M}, {N})")
        per_row = int(smooth_scale.shape[0] == M and M != 1)
    if block_size > 0:
        if block_size < 2 or (block_size & (block_size - 1)) != 0:
            raise ValueError(f"block_size must be a power of 2 ≥ 2, got {block_size}")
        if N % block_size != 0:
            raise ValueError(f"N (={N}) must be divisible by block_size (={block_size})")
    p = _lib.QuantParams()
    p.device = _device_index(x)
    p.x, p.x_is_fp16, p.m, p.n = x.data_ptr(), int(x.dtype == torch.float16), M, N
    p.smooth = smooth_scale.data_ptr() if smooth_scale is not None else None
    p.smooth_per_row = per_row
    p.xq, p.scales, p.max_val, p.block_size = xq.data_ptr(), xq_scales.data_ptr(), int(max_val), int(block_size)
    with torch.cuda.device(x.device):
        _lib.call("pb2_quantize", p, _stream(x.device), "quantize")


def rcp_approx_f32(x: torch.Tensor) -> torch.Tensor:
    """rcp.approx.ftz.f32 of every element of a float32 CUDA tensor: the
    approximate reciprocal ``quantize`` takes for its inverse scale, as the
    reference's kernel does (hadamard.py:446, cute.arch.rcp_approx).  PTX
    bounds its error to 1 ulp without fixing the last bit, so a CPU
    restatement of the quantizer reads it from here (a test aid)."""
    if not x.is_cuda or x.dtype != torch.float32 or not x.is_contiguous():
        _fail("x must be a contiguous float32 CUDA tensor")
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        st = _lib.load().pb2_rcp_approx_f32(_device_index(x), x.data_ptr(), out.data_ptr(), x.numel(),
                                            _stream(x.device))
    _lib.check(st, "rcp_approx_f32")
    return out


__all__ = ["quantize", "rcp_approx_f32", "DEFAULT_HADAMARD_BLOCK_SIZE"]
