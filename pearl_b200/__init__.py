"""pearl_b200 -- B200 (sm_100a) kernels for Pearl's mining hot path, behind
the ``pearl_gemm`` package surface (miner/pearl-gemm/src/pearl_gemm/__init__.py).

    import pearl_b200 as pearl_gemm

gives the reference's operators (noise_gen, noise_A, noise_B, gemm,
noisy_gemm, denoise_converter, tensor_hash,
commitment_hash_from_merkle_roots), helpers and constants, and registers the same
``torch.ops.pearl_gemm.*`` schemas.
"""

from . import _lib
from .helpers import (
    HostSignalHeader,
    HostSignalHeaderPinnedPool,
    HostSignalStatus,
    ProofTileIndices,
    extract_indices,
    get_host_signal_header,
    get_host_signal_header_size,
    get_host_signal_sync_fields,
    get_host_signal_sync_size,
)
from . import pearl_gemm_interface
from .pearl_gemm_interface import (
    commitment_hash_from_merkle_roots,
    denoise_converter,
    gemm,
    get_required_scratchpad_bytes,
    inner_hash,
    kEALScaleFactorDenoise,
    kEBRScaleFactorDenoise,
    make_pow_target_tensor,
    noise_A,
    noise_AB,
    noise_B,
    noise_gen,
    noisy_gemm,
    tensor_hash,
)
from . import moe
from . import quantization
from . import device_waits
from . import fp8
from . import merkle
from . import proof
from . import ops  # noqa: F401  (registers torch.ops.pearl_gemm.*)

__all__ = [
    "HostSignalHeader",
    "HostSignalHeaderPinnedPool",
    "HostSignalStatus",
    "ProofTileIndices",
    "commitment_hash_from_merkle_roots",
    "get_required_scratchpad_bytes",
    "tensor_hash",
    "denoise_converter",
    "extract_indices",
    "gemm",
    "get_host_signal_header",
    "get_host_signal_header_size",
    "get_host_signal_sync_fields",
    "get_host_signal_sync_size",
    "inner_hash",
    "moe",
    "quantization",
    "device_waits",
    "fp8",
    "kEALScaleFactorDenoise",
    "kEBRScaleFactorDenoise",
    "make_pow_target_tensor",
    "noise_A",
    "noise_AB",
    "noise_B",
    "noise_gen",
    "noisy_gemm",
    "pearl_gemm_interface",
]
