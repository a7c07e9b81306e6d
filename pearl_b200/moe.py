"""Mirror of ``pearl_gemm.moe`` (miner/pearl-gemm/src/pearl_gemm/moe.py):
the canonical MoE routing order a mined expert layer commits to, computed on
the B200 (pearl_b200/csrc/routing.cu) through the C ABI."""

from __future__ import annotations

import torch

from . import _lib
from .pearl_gemm_interface import _device_index, _fail, _stream


def get_build_routing_data_scratchpad_bytes(numel: int) -> int:
    """Scratch bytes build_routing_data needs for ``numel`` routed slots."""
    return int(_lib.load().pb2_build_routing_data_scratchpad_bytes(int(numel)))


def build_routing_data(
    topk_ids: torch.Tensor,
    routing_data: torch.Tensor,
    slot_indices: torch.Tensor,
    routing_offsets: torch.Tensor,
    scratchpad: torch.Tensor,
    num_experts: int,
) -> None:
    """Stable per-expert ordering of the routed slots
    (build_routing_data.cu:127-166): ``slot_indices`` = flat slot indices
    sorted by expert id, ``routing_data`` = their tokens
    (``slot_indices // top_k``), ``routing_offsets[e]`` = exclusive end of
    expert e's segment."""
    named = ((topk_ids, "topk_ids"), (routing_data, "routing_data"), (slot_indices, "slot_indices"),
             (routing_offsets, "routing_offsets"), (scratchpad, "scratchpad"))
    for t, name in named:
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
    for t, name in named:
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
    for t, name in named[:4]:
        if t.dtype != torch.int32:
            _fail(f"{name} must be int32")
    if scratchpad.dtype != torch.uint8:
        _fail("scratchpad must be uint8")
    if topk_ids.dim() != 2:
        _fail("topk_ids must be 2D (m, K)")
    num_tokens, top_k = topk_ids.shape
    numel = num_tokens * top_k
    if routing_data.numel() != numel:
        _fail("routing_data must have m*K elements")
    if slot_indices.numel() != numel:
        _fail("slot_indices must have m*K elements")
    if num_experts > 256:
        _fail(f"build_routing_data sorts on 8-bit expert IDs, got num_experts={num_experts}")
    if routing_offsets.numel() != num_experts:
        _fail("routing_offsets must have num_experts elements")
    required = get_build_routing_data_scratchpad_bytes(numel)
    if scratchpad.numel() < required:
        _fail(f"scratchpad too small: need {required} bytes, got {scratchpad.numel()}")
    p = _lib.RoutingParams()
    p.device = _device_index(topk_ids)
    p.topk_ids, p.num_tokens, p.top_k = topk_ids.data_ptr(), num_tokens, top_k
    p.routing_data, p.slot_indices = routing_data.data_ptr(), slot_indices.data_ptr()
    p.routing_offsets, p.num_experts = routing_offsets.data_ptr(), num_experts
    p.scratchpad, p.scratchpad_bytes = scratchpad.data_ptr(), scratchpad.numel()
    with torch.cuda.device(topk_ids.device):
        _lib.call("pb2_build_routing_data", p, _stream(topk_ids.device), "build_routing_data")


def scatter_rows(src: torch.Tensor, dst: torch.Tensor, indices: torch.Tensor) -> None:
    """``dst[indices] = src`` for whole rows (2-D, contiguous, same dtype and
    row length; ``indices`` int32 on the same device): the per-expert step
    that puts a mined expert GEMM's rows back in routing-slot order
    (pearl_moe_experts.py:347).  A B200 kernel in place of torch's index_put;
    indices outside ``dst`` are skipped."""
    if not (src.is_cuda and dst.is_cuda and indices.is_cuda):
        _fail("scatter_rows: tensors must be on CUDA")
    if src.dim() != 2 or dst.dim() != 2 or src.shape[1] != dst.shape[1] or src.dtype != dst.dtype:
        _fail("scatter_rows: src and dst must be 2-D with the same row length and dtype")
    if not (src.is_contiguous() and dst.is_contiguous() and indices.is_contiguous()):
        _fail("scatter_rows: tensors must be contiguous")
    if indices.dtype != torch.int32 or indices.numel() != src.shape[0]:
        _fail("scatter_rows: indices must be int32 with one entry per src row")
    row_bytes = src.shape[1] * src.element_size()
    if row_bytes % 16 != 0:
        _fail("scatter_rows: rows must be a multiple of 16 bytes")
    p = _lib.ScatterParams(device=_device_index(src), src=src.data_ptr(), dst=dst.data_ptr(),
                           indices=indices.data_ptr(), rows=src.shape[0], dst_rows=dst.shape[0],
                           row_bytes=row_bytes)
    with torch.cuda.device(src.device):
        _lib.call("pb2_scatter_rows", p, _stream(src.device), "scatter_rows")
