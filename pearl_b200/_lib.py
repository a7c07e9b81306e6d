"""ctypes binding of the C ABI declared in include/pearl_b200.h.

The library is loaded from ``pearl_b200/_lib/libpearl_b200.so`` (built in-tree
by ``pearl_b200/build.py``).  There is no fallback: if the library is missing
or fails to load, every operator raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libpearl_b200.so")

PB2_OK = 0
PB2_ERR_INVALID_ARGUMENT = 1
PB2_ERR_UNSUPPORTED_CONFIG = 2
PB2_ERR_CUDA = 3
PB2_ERR_DEVICE_TIMEOUT = 4
PB2_ERR_NO_DRIVER_ENTRY = 5
PB2_ERR_SCRATCH_LIMIT = 6
STATIC_SCRATCH_BYTES = 8 * 1024 * 1024

HOST_SIGNAL_HEADER_SIZE = 640
HOST_SIGNAL_SYNC_SIZE = 16
HIT_WORDS = 12

EXPORTED = [
    "pb2_host_signal_header_size", "pb2_host_signal_sync_size", "pb2_status_string",
    "pb2_last_cuda_error", "pb2_abi_version", "pb2_noise_gen", "pb2_noise_A", "pb2_noise_B", "pb2_noise_AB",
    "pb2_denoise_converter", "pb2_noisy_gemm", "pb2_gemm", "pb2_inner_hash",
    "pb2_noisy_gemm_static_scratch", "pb2_tensor_hash", "pb2_required_scratchpad_bytes", "pb2_gemm_workspace_bytes",
    "pb2_commitment_hash_from_merkle_roots", "pb2_build_routing_data",
    "pb2_build_routing_data_scratchpad_bytes", "pb2_quantize", "pb2_scatter_rows",
    "pb2_merkle_layers", "pb2_merkle_nodes", "pb2_set_wait_budget_cycles", "pb2_wait_selftest",
    "pb2_rcp_approx_f32", "pb2_noisy_gemm_grouped", "pb2_mined_gemm_fp8",
]
DEFAULT_WAIT_BUDGET_CYCLES = 2000000000

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


class NoiseGenParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("m", _i64), ("n", _i64), ("k", _i64), ("r", _i64),
                ("EAL", _vp), ("EAL_fp16", _vp), ("EAR_R_major", _vp), ("EAR_K_major", _vp),
                ("EBL_R_major", _vp), ("EBL_K_major", _vp), ("EBR", _vp), ("EBR_fp16", _vp),
                ("key_a", _vp), ("key_b", _vp), ("aux_buffer", _vp), ("aux_words", _i64)]


class NoisingParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("rows", _i64), ("k", _i64), ("r", _i64),
                ("X", _vp), ("EL", _vp), ("E_rmajor", _vp), ("E_kmajor", _vp), ("XpE", _vp),
                ("proj", _vp), ("proj_is_fp16", ctypes.c_int), ("k_blocks_per_split", ctypes.c_int),
                ("host_signal_sync", _vp)]


class DenoiseConverterParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("m", _i64), ("n", _i64), ("r", _i64),
                ("EARxBpEB_in", _vp), ("AxEBL_in", _vp), ("EARxBpEB_out", _vp), ("AxEBL_out", _vp)]


class GemmParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("m", _i64), ("n", _i64), ("k", _i64), ("r", _i64),
                ("A", _vp), ("B", _vp), ("EAL", _vp), ("EBR", _vp), ("EAR_R_major", _vp),
                ("EBL_R_major", _vp), ("EAR_K_major", _vp), ("EBL_K_major", _vp),
                ("AxEBL_int32", _vp), ("EARxBpEB_int32", _vp),
                ("ApEA", _vp), ("BpEB", _vp), ("EAL_fp16", _vp), ("EBR_fp16", _vp),
                ("AxEBL_fp16", _vp), ("EARxBpEB_fp16", _vp), ("A_scales", _vp), ("B_scales", _vp),
                ("C", _vp), ("host_signal_header_pinned", _vp), ("host_signal_sync", _vp),
                ("pow_target", _vp), ("pow_key", _vp),
                ("tile_size_m", ctypes.c_int), ("tile_size_n", ctypes.c_int),
                ("tile_size_k", ctypes.c_int), ("cluster_size_m", ctypes.c_int),
                ("cluster_size_n", ctypes.c_int), ("pipeline_stages", ctypes.c_int),
                ("swizzle", ctypes.c_int), ("swizzle_n_maj", ctypes.c_int),
                ("run_noising_a", ctypes.c_int), ("run_noising_b", ctypes.c_int),
                ("k_blocks_per_split_noising_a", ctypes.c_int),
                ("k_blocks_per_split_noising_b", ctypes.c_int),
                ("skip_reduction", ctypes.c_int), ("skip_denoising", ctypes.c_int),
                ("inner_hash_counter", _vp), ("enable_debug", ctypes.c_int),
                ("hits", _vp), ("hit_capacity", _i64), ("transcripts", _vp), ("digests", _vp),
                ("workspace", _vp), ("workspace_bytes", _i64)]


class Fp8GemmParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("m", _i64), ("n", _i64), ("k", _i64), ("r", _i64), ("A", _vp),
                ("B", _vp), ("format", ctypes.c_int), ("A_scale", _vp), ("B_scale", _vp), ("C", _vp),
                ("host_signal_header_pinned", _vp), ("host_signal_sync", _vp), ("pow_target", _vp),
                ("pow_key", _vp), ("skip_reduction", ctypes.c_int), ("hits", _vp), ("hit_capacity", _i64),
                ("transcripts", _vp), ("digests", _vp)]


class ExpertGemm(ctypes.Structure):
    _fields_ = [("m", _i64), ("a_row0", _i64), ("host_signal_header_pinned", _vp), ("host_signal_sync", _vp),
                ("hits", _vp), ("hit_capacity", _i64), ("transcripts", _vp), ("digests", _vp)]


class GroupedGemmParams(ctypes.Structure):
    _fields_ = [("shared", GemmParams), ("num_experts", _i64), ("experts", ctypes.POINTER(ExpertGemm)),
                ("c_row_index", _vp), ("c_rows", _i64)]


class TensorHashParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("data", _vp), ("len", _i64), ("key", _vp), ("out", _vp),
                ("roots", _vp), ("roots_bytes", _i64), ("threads_per_block", ctypes.c_int)]


class CommitmentParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("A_merkle_root", _vp), ("B_merkle_root", _vp),
                ("key", _vp), ("A_commitment_hash", _vp), ("B_commitment_hash", _vp),
                ("routing_root", _vp), ("offsets_hash", _vp), ("salted", ctypes.c_int),
                ("salted_dim_a", ctypes.c_uint32), ("salted_dim_b", ctypes.c_uint32)]


class RoutingParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("topk_ids", _vp), ("num_tokens", _i64), ("top_k", _i64),
                ("routing_data", _vp), ("slot_indices", _vp), ("routing_offsets", _vp),
                ("num_experts", _i64), ("scratchpad", _vp), ("scratchpad_bytes", _i64)]


class QuantParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("x", _vp), ("x_is_fp16", ctypes.c_int), ("m", _i64),
                ("n", _i64), ("smooth", _vp), ("smooth_per_row", ctypes.c_int), ("xq", _vp),
                ("scales", _vp), ("max_val", ctypes.c_int), ("block_size", ctypes.c_int)]


class MerkleParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("data", _vp), ("len", _i64), ("key", _vp), ("nodes", _vp),
                ("nodes_bytes", _i64)]


class ScatterParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("src", _vp), ("dst", _vp), ("indices", _vp), ("rows", _i64),
                ("dst_rows", _i64), ("row_bytes", _i64)]


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libpearl_b200.so (raises if it is missing: there is no CPU path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"pearl_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m pearl_b200.build` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name in ("pb2_noise_gen", "pb2_noise_A", "pb2_noise_B", "pb2_denoise_converter",
                     "pb2_noisy_gemm", "pb2_gemm", "pb2_noisy_gemm_static_scratch", "pb2_noisy_gemm_grouped",
                     "pb2_mined_gemm_fp8",
                     "pb2_tensor_hash", "pb2_commitment_hash_from_merkle_roots",
                     "pb2_build_routing_data", "pb2_quantize", "pb2_scatter_rows", "pb2_merkle_layers"):
            getattr(L, name).restype = ctypes.c_int
            getattr(L, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.pb2_noise_AB.restype = ctypes.c_int
        L.pb2_noise_AB.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.pb2_inner_hash.restype = ctypes.c_int
        L.pb2_inner_hash.argtypes = [ctypes.c_int, _vp, _i64, _vp, _i64, _vp]
        L.pb2_build_routing_data_scratchpad_bytes.restype = _i64
        L.pb2_build_routing_data_scratchpad_bytes.argtypes = [_i64]
        L.pb2_merkle_nodes.restype = _i64
        L.pb2_merkle_nodes.argtypes = [_i64]
        L.pb2_required_scratchpad_bytes.restype = _i64
        L.pb2_required_scratchpad_bytes.argtypes = [_i64, ctypes.c_int]
        L.pb2_gemm_workspace_bytes.restype = _i64
        L.pb2_gemm_workspace_bytes.argtypes = [ctypes.c_int, _i64, _i64, _i64]
        L.pb2_host_signal_header_size.restype = _i64
        L.pb2_host_signal_sync_size.restype = _i64
        L.pb2_status_string.restype = ctypes.c_char_p
        L.pb2_status_string.argtypes = [ctypes.c_int]
        L.pb2_last_cuda_error.restype = ctypes.c_char_p
        L.pb2_abi_version.restype = ctypes.c_int
        L.pb2_set_wait_budget_cycles.restype = _i64
        L.pb2_set_wait_budget_cycles.argtypes = [_i64]
        L.pb2_wait_selftest.restype = ctypes.c_int
        L.pb2_wait_selftest.argtypes = [ctypes.c_int, _i64, _vp, _vp]
        L.pb2_rcp_approx_f32.restype = ctypes.c_int
        L.pb2_rcp_approx_f32.argtypes = [ctypes.c_int, _vp, _vp, _i64, _vp]
        _lib = L
    return _lib


def check(status: int, op: str) -> None:
    if status == PB2_OK:
        return
    L = load()
    msg = L.pb2_status_string(status).decode()
    if status == PB2_ERR_CUDA:
        msg += ": " + L.pb2_last_cuda_error().decode()
    raise RuntimeError(f"pearl_b200 {op} failed: {msg}")


def call(name: str, params, stream: int, op: str | None = None) -> None:
    L = load()
    st = getattr(L, name)(ctypes.byref(params), ctypes.c_void_p(stream))
    check(st, op or name)
