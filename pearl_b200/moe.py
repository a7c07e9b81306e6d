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


def noisy_gemm_grouped(
    A, B, EAL, EAL_fp16, EBR, EBR_fp16, EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major,
    AxEBL_fp16, EARxBpEB_fp16, ApEA, BpEB, A_scales, B_scales, C, expert_rows,
    host_signal_headers, host_signal_syncs, pow_target, pow_key, *, hits=None, transcripts=None,
    digests=None, run_noising_A: bool = True, run_noising_B: bool = True, tile_size_m: int = 128,
    tile_size_n: int = 256, tile_size_k: int = 128, c_row_index=None,
):
    """The mined GEMM1 of every expert of a MoE layer in one call: for expert
    e, exactly ``noisy_gemm`` (run_noising_A/B, reduction and denoising on) of
    its rows of A against its rows of B -- the loop of
    pearl_moe_experts.py:304-343 -- as one noising launch and one persistent
    mined launch (per 16 experts).

    A-side tensors (A, EAL, EAL_fp16, ApEA, AxEBL_fp16, A_scales, C) hold
    every expert's rows in expert order, ``expert_rows[e]`` of them for expert
    e (0 allowed); B-side tensors (B, EBR, EBR_fp16, BpEB, EARxBpEB_fp16,
    B_scales) hold n rows per expert, expert e at rows [e n, e n + n); the
    K-side factors EAR_* / EBL_* are shared.  ``host_signal_headers`` /
    ``host_signal_syncs`` (and the optional ``hits`` / ``transcripts`` /
    ``digests``) are per-expert lists, used as for that expert's own
    noisy_gemm.

    ``c_row_index`` (optional, int32 (m,) on the device) fuses the slot-order
    write-back that follows the reference's loop (pearl_moe_experts.py:347,
    ``cache_flat[idx] = out``) into the epilogue: row i of the experts' C
    goes to row c_row_index[i] of ``C``, which then has at least m rows."""
    from .pearl_gemm_interface import _check_matmul_config, _check_tensor, _gemm_params, _ptr

    E = len(expert_rows)
    if E == 0:
        _fail("expert_rows must not be empty")
    m, k = A.shape
    n_all = B.shape[0]
    if n_all % E:
        _fail("B must hold the same number of rows for every expert")
    n = n_all // E
    r = EAL.shape[1]
    if sum(int(v) for v in expert_rows) != m or any(int(v) < 0 for v in expert_rows):
        _fail(f"expert_rows must be non-negative and add up to A's {m} rows")
    _check_matmul_config("noisy_gemm", tile_size_m, tile_size_n, tile_size_k, 1, 1, None, r)
    for t, shape, dt, name in (
            (A, (m, k), torch.int8, "A"), (EAL, (m, r), torch.int8, "EAL"),
            (EAL_fp16, (m, r), torch.float16, "EAL_fp16"), (ApEA, (m, k), torch.int8, "ApEA"),
            (AxEBL_fp16, (m, r), torch.float16, "AxEBL_fp16"), (A_scales, (m,), torch.float32, "A_scales"),
            (C, (C.shape[0] if c_row_index is not None else m, n), torch.bfloat16, "C"),
            (B, (n_all, k), torch.int8, "B"),
            (EBR, (n_all, r), torch.int8, "EBR"), (EBR_fp16, (n_all, r), torch.float16, "EBR_fp16"),
            (BpEB, (n_all, k), torch.int8, "BpEB"), (EARxBpEB_fp16, (n_all, r), torch.float16, "EARxBpEB_fp16"),
            (B_scales, (n_all,), torch.float32, "B_scales"), (EAR_R_major, (k, r), torch.int8, "EAR_R_major"),
            (EBL_R_major, (k, r), torch.int8, "EBL_R_major"), (EAR_K_major, (r, k), torch.int8, "EAR_K_major"),
            (EBL_K_major, (r, k), torch.int8, "EBL_K_major")):
        _check_tensor(t, shape, dt, name)
    for t, name in ((pow_target, "pow_target"), (pow_key, "pow_key")):
        _check_tensor(t, (8,), torch.uint32, name)
    if c_row_index is not None:
        _check_tensor(c_row_index, (m,), torch.int32, "c_row_index")
        if C.shape[0] < m:
            _fail(f"C must have at least {m} rows with c_row_index")
    if len(host_signal_headers) != E or len(host_signal_syncs) != E:
        _fail("one host signal header and one sync buffer per expert")
    p = _gemm_params(m, n, k, r, _device_index(A), tile_size_m, tile_size_n, tile_size_k, 1, 1, None, None,
                     True)
    p.A, p.B, p.EAL, p.EBR = _ptr(A), _ptr(B), _ptr(EAL), _ptr(EBR)
    p.EAR_R_major, p.EBL_R_major = _ptr(EAR_R_major), _ptr(EBL_R_major)
    p.EAR_K_major, p.EBL_K_major = _ptr(EAR_K_major), _ptr(EBL_K_major)
    p.ApEA, p.BpEB = _ptr(ApEA), _ptr(BpEB)
    p.EAL_fp16, p.EBR_fp16 = _ptr(EAL_fp16), _ptr(EBR_fp16)
    p.AxEBL_fp16, p.EARxBpEB_fp16 = _ptr(AxEBL_fp16), _ptr(EARxBpEB_fp16)
    p.A_scales, p.B_scales, p.C = _ptr(A_scales), _ptr(B_scales), _ptr(C)
    p.pow_target, p.pow_key = _ptr(pow_target), _ptr(pow_key)
    p.run_noising_a, p.run_noising_b = int(bool(run_noising_A)), int(bool(run_noising_B))
    p.k_blocks_per_split_noising_a = p.k_blocks_per_split_noising_b = -1
    table = (_lib.ExpertGemm * E)()
    row0 = 0
    for e in range(E):
        q = table[e]
        q.m, q.a_row0 = int(expert_rows[e]), row0
        row0 += int(expert_rows[e])
        hdr, sync = host_signal_headers[e], host_signal_syncs[e]
        if q.m > 0:
            if sync is None or not sync.is_cuda or sync.numel() != _lib.HOST_SIGNAL_SYNC_SIZE:
                _fail(f"expert {e}: host_signal_sync must be a {_lib.HOST_SIGNAL_SYNC_SIZE}-byte CUDA buffer")
            if hdr is not None and (hdr.is_cuda or not hdr.is_pinned()):
                _fail(f"expert {e}: host_signal_header_pinned must be a pinned CPU tensor")
        q.host_signal_sync = _ptr(sync)
        q.host_signal_header_pinned = _ptr(hdr)
        if hits is not None and hits[e] is not None:
            q.hits, q.hit_capacity = _ptr(hits[e]), hits[e].shape[0]
        for lst, words, field in ((transcripts, 16, "transcripts"), (digests, 8, "digests")):
            if lst is not None and lst[e] is not None:
                _check_tensor(lst[e], ((q.m // 2) * (n // 64), words), (torch.int32, torch.uint32),
                              f"{field}[{e}]")
                setattr(q, field, _ptr(lst[e]))
    g = _lib.GroupedGemmParams()
    g.shared, g.num_experts, g.experts = p, E, table
    if c_row_index is not None:
        g.c_row_index, g.c_rows = _ptr(c_row_index), C.shape[0]
    with torch.cuda.device(A.device):
        _lib.call("pb2_noisy_gemm_grouped", g, _stream(A.device), "noisy_gemm_grouped")
