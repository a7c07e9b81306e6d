"""``torch.ops.pearl_gemm.*`` registrations with the reference's schemas
(miner/pearl-gemm/csrc/gemm/pearl_gemm_api.cpp:1087-1248), including the
schema defaults that differ from the Python wrappers (noisy_gemm:
run_noising_B=False, skip_reduction=True), CUDA implementations that call
the B200 kernels and fake implementations for torch.compile.

If another library already defined the ``pearl_gemm`` namespace (the
reference extension itself), registration is skipped."""

from __future__ import annotations

import logging

import torch

from . import moe as M
from . import pearl_gemm_interface as I

_LOG = logging.getLogger(__name__)

SCHEMAS = {
    "noisy_gemm": (
        "noisy_gemm(Tensor A, Tensor B, Tensor EAL, Tensor? EAL_fp16, Tensor EBR, Tensor? EBR_fp16, "
        "Tensor? EAR_R_major, Tensor? EBL_R_major, Tensor? EAR_K_major, Tensor? EBL_K_major, "
        "Tensor(AxEBL_fp16!) AxEBL_fp16, Tensor(EARxBpEB_fp16!) EARxBpEB_fp16, Tensor(ApEA!) ApEA, "
        "Tensor(BpEB!) BpEB, Tensor A_scales, Tensor B_scales, Tensor(C!) C, "
        "Tensor(host_signal_header_pinned!) host_signal_header_pinned, "
        "Tensor(host_signal_sync!) host_signal_sync, Tensor pow_target, Tensor pow_key, "
        "Tensor(AxEBL_int32!)? AxEBL_int32 = None, Tensor(EARxBpEB_int32!)? EARxBpEB_int32 = None, "
        "int tile_size_m = 128, int tile_size_n = 256, int tile_size_k = 128, "
        "int cluster_size_m = 1, int cluster_size_n = 1, int? pipeline_stages = None, "
        "int? swizzle = None, bool swizzle_n_maj = True, int? tile_size_m_noising_A = None, "
        "int? tile_size_n_noising_B = None, int? tile_size_k_noising_A = None, "
        "int? tile_size_k_noising_B = None, int pipeline_stages_noising_A = 2, "
        "int pipeline_stages_noising_B = 2, int? k_blocks_per_split_noising_A = None, "
        "int? k_blocks_per_split_noising_B = None, bool run_noising_A = True, "
        "bool run_noising_B = False, bool skip_reduction = True, bool skip_denoising = False, "
        "Tensor(inner_hash_counter!)? inner_hash_counter = None, bool enable_debug = False) -> ()"),
    "gemm": (
        "gemm(Tensor A, Tensor B, Tensor A_scales, Tensor B_scales, Tensor(C!) C, "
        "int tile_size_m = 128, int tile_size_n = 256, int tile_size_k = 128, "
        "int cluster_size_m = 1, int cluster_size_n = 1, int? pipeline_stages = None, "
        "int? swizzle = None, bool swizzle_n_maj = True) -> ()"),
    "noise_A": (
        "noise_A(Tensor A, Tensor EAL, Tensor(AxEBL!) AxEBL, Tensor(ApEA!) ApEA, Tensor? EAR, "
        "Tensor? EBL, int? tile_size_m = None, int? tile_size_k = None, int pipeline_stages = 2, "
        "int? k_blocks_per_split = None) -> ()"),
    "noise_B": (
        "noise_B(Tensor B, Tensor EBR, Tensor(EARxBpEB!) EARxBpEB, Tensor(BpEB!) BpEB, Tensor? EAR, "
        "Tensor? EBL, int? tile_size_n = None, int? tile_size_k = None, int pipeline_stages = 2, "
        "int? k_blocks_per_split = None) -> ()"),
    "denoise_converter": (
        "denoise_converter(Tensor? EARxBpEB_in, Tensor? AxEBL_in, "
        "Tensor(EARxBpEB_out!)? EARxBpEB_out, Tensor(AxEBL_out!)? AxEBL_out) -> ()"),
    "noise_gen": (
        "noise_gen(int R, int num_threads = 64, Tensor(EAL!)? EAL = None, "
        "Tensor(EAL_fp16!)? EAL_fp16 = None, Tensor(EAR_R_major!)? EAR_R_major = None, "
        "Tensor(EAR_K_major!)? EAR_K_major = None, Tensor(EBL_R_major!)? EBL_R_major = None, "
        "Tensor(EBL_K_major!)? EBL_K_major = None, Tensor(EBR!)? EBR = None, "
        "Tensor(EBR_fp16!)? EBR_fp16 = None, Tensor? key_A = None, Tensor? key_B = None, "
        "Tensor(aux_buffer!)? aux_buffer = None) -> ()"),
    "inner_hash": "inner_hash(Tensor input_buffer, int iterations = 1) -> Tensor",
    "tensor_hash": (
        "tensor_hash(Tensor data, Tensor key, Tensor(out!) out, Tensor(roots!) roots, "
        "int num_threads = 128, int num_stages = 2, int leaves_per_mt_block = 512) -> ()"),
    "commitment_hash_from_merkle_roots": (
        "commitment_hash_from_merkle_roots(Tensor A_merkle_root, Tensor B_merkle_root, Tensor key, "
        "Tensor(A_commitment_hash!) A_commitment_hash, Tensor(B_commitment_hash!) B_commitment_hash, "
        "Tensor? routing_root=None, Tensor? offsets_hash=None, int? salted_dim_a=None, "
        "int? salted_dim_b=None) -> ()"),
    "build_routing_data": (
        "build_routing_data(Tensor topk_ids, Tensor(routing_data!) routing_data, "
        "Tensor(slot_indices!) slot_indices, Tensor(routing_offsets!) routing_offsets, "
        "Tensor(scratchpad!) scratchpad, int num_experts) -> ()"),
}


def _tensor_hash_op(data, key, out, roots, num_threads=128, num_stages=2, leaves_per_mt_block=512):
    I.tensor_hash(data, key, out, roots, num_threads, num_stages, leaves_per_mt_block)


def _commitment_op(A_merkle_root, B_merkle_root, key, A_commitment_hash, B_commitment_hash,
                   routing_root=None, offsets_hash=None, salted_dim_a=None, salted_dim_b=None):
    if (salted_dim_a is None) != (salted_dim_b is None):
        raise RuntimeError("salted_dim_a and salted_dim_b must be provided together")
    dims = None if salted_dim_a is None else (salted_dim_a, salted_dim_b)
    I.commitment_hash_from_merkle_roots(A_merkle_root, B_merkle_root, key, A_commitment_hash,
                                        B_commitment_hash, routing_root, offsets_hash,
                                        salted_dims=dims)


_IMPLS = {
    "noisy_gemm": I.noisy_gemm,
    "gemm": I.gemm,
    "noise_A": I.noise_A,
    "noise_B": I.noise_B,
    "denoise_converter": I.denoise_converter,
    "noise_gen": I.noise_gen,
    "inner_hash": I.inner_hash,
    "tensor_hash": _tensor_hash_op,
    "commitment_hash_from_merkle_roots": _commitment_op,
    "build_routing_data": M.build_routing_data,
}

# The reference registers these without the pt2_compliant tag
# (pearl_gemm_api.cpp:1207-1224).
_UNTAGGED = ("inner_hash", "tensor_hash", "commitment_hash_from_merkle_roots", "build_routing_data")

_TAGS = (torch.Tag.pt2_compliant_tag,)
_lib = None
_fake_lib = None
REGISTERED = False


def _register() -> None:
    global _lib, _fake_lib, REGISTERED
    try:
        lib = torch.library.Library("pearl_gemm", "DEF")
    except RuntimeError as e:  # namespace already owned (e.g. the reference extension)
        _LOG.warning("torch.ops.pearl_gemm already defined; not registering B200 ops (%s)", e)
        return
    for name, schema in SCHEMAS.items():
        lib.define(schema, tags=() if name in _UNTAGGED else _TAGS)
        lib.impl(name, _IMPLS[name], "CUDA")
    # The fake implementations live in a library object of their own, so
    # that release_fake_impls() can hand them over to the reference's
    # interface files (which register theirs at import).
    fake = torch.library.Library("pearl_gemm", "FRAGMENT")
    for name in SCHEMAS:
        if name == "inner_hash":
            torch.library.register_fake(f"pearl_gemm::{name}", lib=fake)(
                lambda input_buffer, iterations=1: input_buffer.new_empty((1,)))
        else:
            torch.library.register_fake(f"pearl_gemm::{name}", lib=fake)(lambda *a, **k: None)
    _lib, _fake_lib = lib, fake
    REGISTERED = True


def release_fake_impls() -> None:
    """Withdraw pearl_b200's fake implementations of torch.ops.pearl_gemm.*,
    leaving the schemas and CUDA implementations.  The reference's extension
    defines the ops and its Python files (pearl_gemm_interface.py:36-628,
    moe.py:34) register the fakes; running that package on these kernels
    (through pearl_b200.pearl_gemm_cuda) needs the same split."""
    global _fake_lib
    if _fake_lib is not None:
        _fake_lib._destroy()
        _fake_lib = None


_register()
