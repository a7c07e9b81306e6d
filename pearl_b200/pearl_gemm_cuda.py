"""The ``pearl_gemm_cuda`` extension module surface on the B200 kernels.

The reference's Python package ``pearl_gemm`` (miner/pearl-gemm/src/
pearl_gemm/) runs every operator through a compiled extension named
``pearl_gemm_cuda``: ``pearl_gemm_interface.py:1`` imports it and calls its
functions positionally, ``__init__.py:8-16`` and ``helpers.py:9`` re-export
its constants and classes, and the extension's ``TORCH_LIBRARY(pearl_gemm)``
block defines the ``torch.ops.pearl_gemm.*`` schemas whose fake (meta)
implementations the interface file then registers.  This module offers the
same names, positional signatures, defaults, constants and classes
(pearl_gemm_api.cpp:981-1084 and the C++ signatures it binds), so the
reference's unmodified Python package runs on these kernels:

    PYTHONPATH=<this repo>/pearl_b200/compat:<reference>/miner/pearl-gemm/src \\
        python -c "import pearl_gemm"

(``pearl_b200/compat/pearl_gemm_cuda.py`` makes ``import pearl_gemm_cuda``
resolve to this module.)  Each function maps its positional arguments onto
the keyword form of ``pearl_b200.pearl_gemm_interface`` -- which validates
them with the reference's rules and launches through the C ABI -- so the
two entry surfaces share one implementation.

Loaded under the extension's name (through the compat loader), it plays the
extension's part for torch.ops as well: the ``pearl_gemm`` schemas stay
defined with their CUDA implementations, and the fake implementations
pearl_b200 registers for itself are withdrawn, because the reference's
``pearl_gemm_interface.py`` / ``moe.py`` register their own
(``torch.library.register_fake`` refuses a second one)."""

from __future__ import annotations

from . import helpers as _helpers
from . import moe as _moe
from . import pearl_gemm_interface as _I

# ---------------------------------------------------------- module attrs ---
kEALScaleFactorDenoise = _I.kEALScaleFactorDenoise
kEBRScaleFactorDenoise = _I.kEBRScaleFactorDenoise
HostSignalStatus = _helpers.HostSignalStatus
HostSignalHeader = _helpers.HostSignalHeader
MMASize = _helpers.MMASize

_DEFAULT_THREADS_PER_BLOCK = _I.DEFAULT_THREADS_PER_BLOCK
_DEFAULT_NUM_STAGES = _I.DEFAULT_NUM_STAGES
_DEFAULT_LEAVES_PER_MT_BLOCK = _I.DEFAULT_LEAVES_PER_MT_BLOCK


# --------------------------------------------------------------- operators -
def denoise_converter(EARxBpEB_in, AxEBL_in, EARxBpEB_out, AxEBL_out):
    """pearl_gemm_api.cpp:114-119."""
    _I.denoise_converter(EARxBpEB_in=EARxBpEB_in, AxEBL_in=AxEBL_in, EARxBpEB_out=EARxBpEB_out,
                         AxEBL_out=AxEBL_out)


def noise_gen(R, num_threads, EAL, EAL_fp16, EAR_R_major, EAR_K_major, EBL_R_major, EBL_K_major, EBR,
              EBR_fp16, key_A, key_B, aux_buffer):
    """pearl_gemm_api.cpp:168-179."""
    _I.noise_gen(R=R, num_threads=num_threads, EAL=EAL, EAL_fp16=EAL_fp16, EAR_R_major=EAR_R_major,
                 EAR_K_major=EAR_K_major, EBL_R_major=EBL_R_major, EBL_K_major=EBL_K_major, EBR=EBR,
                 EBR_fp16=EBR_fp16, key_A=key_A, key_B=key_B, aux_buffer=aux_buffer)


def noise_A(A, EAL, AxEBL, ApEA, EAR, EBL, tile_size_m=None, tile_size_k=None, pipeline_stages=2,
            k_blocks_per_split=None):
    """pearl_gemm_api.cpp:300-309."""
    _I.noise_A(A, EAL, AxEBL, ApEA, EAR=EAR, EBL=EBL, tile_size_m=tile_size_m, tile_size_k=tile_size_k,
               pipeline_stages=pipeline_stages, k_blocks_per_split=k_blocks_per_split)


def noise_B(B, EBR, EARxBpEB, BpEB, EAR, EBL, tile_size_n=None, tile_size_k=None, pipeline_stages=2,
            k_blocks_per_split=None):
    """pearl_gemm_api.cpp:400-409."""
    _I.noise_B(B, EBR, EARxBpEB, BpEB, EAR=EAR, EBL=EBL, tile_size_n=tile_size_n, tile_size_k=tile_size_k,
               pipeline_stages=pipeline_stages, k_blocks_per_split=k_blocks_per_split)


def gemm(A, B, A_scales, B_scales, C, bM, bN, bK, cM, cN, pipeline_stages=None, swizzle=None,
         swizzle_n_maj=True):
    """pearl_gemm_api.cpp:502-510."""
    _I.gemm(A, B, A_scales, B_scales, C, tile_size_m=bM, tile_size_n=bN, tile_size_k=bK, cluster_size_m=cM,
            cluster_size_n=cN, pipeline_stages=pipeline_stages, swizzle=swizzle, swizzle_n_maj=swizzle_n_maj)


def noisy_gemm(A, B, EAL, EAL_fp16, EBR, EBR_fp16, EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major,
               AxEBL_fp16, EARxBpEB_fp16, ApEA, BpEB, A_scales, B_scales, C, host_signal_header_pinned,
               host_signal_sync, pow_target, pow_key, AxEBL_int32, EARxBpEB_int32, bM, bN, bK, cM, cN,
               pipeline_stages=None, swizzle=None, swizzle_n_maj=True, tile_size_m_noising_A=None,
               tile_size_n_noising_B=None, tile_size_k_noising_A=None, tile_size_k_noising_B=None,
               pipeline_stages_noising_A=2, pipeline_stages_noising_B=2, k_blocks_per_split_noising_A=None,
               k_blocks_per_split_noising_B=None, run_noising_a=True, run_noising_b=True,
               skip_reduction=False, skip_denoising=False, inner_hash_counter=None, enable_debug=False):
    """pearl_gemm_api.cpp:618-656 (the C++ defaults: both noisings on,
    reduction on)."""
    _I.noisy_gemm(
        A, B, EAL, EAL_fp16, EBR, EBR_fp16, EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major, AxEBL_fp16,
        EARxBpEB_fp16, ApEA, BpEB, A_scales, B_scales, C, host_signal_header_pinned, host_signal_sync,
        pow_target, pow_key, AxEBL_int32=AxEBL_int32, EARxBpEB_int32=EARxBpEB_int32, tile_size_m=bM,
        tile_size_n=bN, tile_size_k=bK, cluster_size_m=cM, cluster_size_n=cN, pipeline_stages=pipeline_stages,
        swizzle=swizzle, swizzle_n_maj=swizzle_n_maj, tile_size_m_noising_A=tile_size_m_noising_A,
        tile_size_n_noising_B=tile_size_n_noising_B, tile_size_k_noising_A=tile_size_k_noising_A,
        tile_size_k_noising_B=tile_size_k_noising_B, pipeline_stages_noising_A=pipeline_stages_noising_A,
        pipeline_stages_noising_B=pipeline_stages_noising_B,
        k_blocks_per_split_noising_A=k_blocks_per_split_noising_A,
        k_blocks_per_split_noising_B=k_blocks_per_split_noising_B, run_noising_A=run_noising_a,
        run_noising_B=run_noising_b, skip_reduction=skip_reduction, skip_denoising=skip_denoising,
        inner_hash_counter=inner_hash_counter, enable_debug=enable_debug)


def get_host_signal_header(host_signal_header_pinned):
    """pearl_gemm_api.cpp:938-943: a copy of the pinned header."""
    return _helpers.get_host_signal_header(host_signal_header_pinned)


def inner_hash(input_buffer, iterations):
    """pearl_gemm_api.cpp:945-979."""
    return _I.inner_hash(input_buffer, iterations)


def tensor_hash(data, key, out, roots, threads_per_block=_DEFAULT_THREADS_PER_BLOCK,
                num_stages=_DEFAULT_NUM_STAGES, leaves_per_mt_block=_DEFAULT_LEAVES_PER_MT_BLOCK):
    """pearl_gemm_api.cpp:996-1001 (tensor_hash_api.hpp:49-58)."""
    _I.tensor_hash(data, key, out, roots, threads_per_block, num_stages, leaves_per_mt_block)


def commitment_hash_from_merkle_roots(A_merkle_root, B_merkle_root, key, A_commitment_hash, B_commitment_hash,
                                      routing_root=None, offsets_hash=None, salted_dim_a=None,
                                      salted_dim_b=None):
    """pearl_gemm_api.cpp:1002-1010 (tensor_hash_api.hpp:126-140): the salted
    (V3) derivation when both dimensions are given, the legacy one when
    neither is."""
    if (salted_dim_a is None) != (salted_dim_b is None):
        raise RuntimeError("salted_dim_a and salted_dim_b must be provided together")
    dims = None if salted_dim_a is None else (int(salted_dim_a), int(salted_dim_b))
    _I.commitment_hash_from_merkle_roots(A_merkle_root, B_merkle_root, key, A_commitment_hash,
                                         B_commitment_hash, routing_root, offsets_hash, salted_dims=dims)


def get_host_signal_header_size():
    return _I.get_host_signal_header_size()


def get_host_signal_sync_size():
    return _I.get_host_signal_sync_size()


def get_required_scratchpad_bytes(matrix_bytes, threads_per_block=_DEFAULT_THREADS_PER_BLOCK):
    return _I.get_required_scratchpad_bytes(matrix_bytes, threads_per_block)


def build_routing_data(topk_ids, routing_data, slot_indices, routing_offsets, scratchpad, num_experts):
    """build_routing_data.cu:127-166."""
    _moe.build_routing_data(topk_ids, routing_data, slot_indices, routing_offsets, scratchpad, num_experts)


def get_build_routing_data_scratchpad_bytes(numel):
    return _moe.get_build_routing_data_scratchpad_bytes(numel)

