"""CPU tests of the drop-in boundary: the C-ABI library loads and exports
every entry point include/pearl_b200.h declares, the ctypes mirrors agree
with the C structs, the torch.ops schemas carry the reference's defaults,
and argument validation fails loudly (no GPU needed: nothing is launched)."""

import ctypes
import os
import re
import subprocess

import pytest
import torch

import pearl_b200 as pg
from pearl_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pearl_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PB2_API\s+[\w\s\*]+?\b(pb2_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = declared_symbols()
    assert len(names) >= 12
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(_lib.EXPORTED)


def test_library_is_sm100a_only_and_standalone():
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libtorch" not in out and "libc10" not in out
    assert "libcudart" not in out  # static runtime


def test_sizes_and_abi_version():
    L = _lib.load()
    assert L.pb2_abi_version() == 1
    assert L.pb2_host_signal_header_size() == 640 == pg.get_host_signal_header_size()
    assert L.pb2_host_signal_sync_size() == 16 == pg.get_host_signal_sync_size()
    assert ctypes.sizeof(pg.helpers._HeaderLayout) == 636  # padded to 640 by alignas(128)


def _c_sizeof(struct: str) -> int:
    src = f'#include "pearl_b200.h"\n#include <stdio.h>\nint main(){{printf("%zu", sizeof({struct}));}}'
    exe = os.path.join("/tmp", f"pb2_sizeof_{struct}")
    subprocess.run(["gcc", "-x", "c", "-", "-I", os.path.join(ROOT, "include"), "-o", exe],
                   input=src, text=True, check=True)
    return int(subprocess.run([exe], capture_output=True, text=True).stdout)


@pytest.mark.parametrize("cname,pyname", [
    ("pb2_noise_gen_params", "NoiseGenParams"), ("pb2_noising_params", "NoisingParams"),
    ("pb2_denoise_converter_params", "DenoiseConverterParams"), ("pb2_gemm_params", "GemmParams"),
    ("pb2_tensor_hash_params", "TensorHashParams"), ("pb2_commitment_params", "CommitmentParams"),
    ("pb2_routing_params", "RoutingParams"), ("pb2_quant_params", "QuantParams"),
    ("pb2_scatter_params", "ScatterParams"), ("pb2_merkle_params", "MerkleParams"),
    ("pb2_fp8_gemm_params", "Fp8GemmParams"), ("pb2_expert_gemm", "ExpertGemm"),
    ("pb2_grouped_gemm_params", "GroupedGemmParams")])
def test_param_struct_layout_matches_header(cname, pyname):
    assert _c_sizeof(cname) == ctypes.sizeof(getattr(_lib, pyname))


def test_status_strings():
    L = _lib.load()
    for code in range(6):
        assert L.pb2_status_string(code)
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(_lib.PB2_ERR_INVALID_ARGUMENT, "x")


def test_null_params_rejected():
    L = _lib.load()
    for name in ("pb2_noise_gen", "pb2_noise_A", "pb2_noise_B", "pb2_denoise_converter",
                 "pb2_noisy_gemm", "pb2_gemm"):
        assert getattr(L, name)(None, None) == _lib.PB2_ERR_INVALID_ARGUMENT
    assert L.pb2_noise_AB(None, None, None) == _lib.PB2_ERR_INVALID_ARGUMENT


def test_torch_ops_schemas_keep_reference_defaults():
    s = torch.ops.pearl_gemm.noisy_gemm.default._schema
    d = {a.name: a.default_value for a in s.arguments}
    assert d["run_noising_A"] is True and d["run_noising_B"] is False
    assert d["skip_reduction"] is True and d["skip_denoising"] is False
    assert d["tile_size_m"] == 128 and d["tile_size_n"] == 256 and d["tile_size_k"] == 128
    for op in ("gemm", "noise_A", "noise_B", "denoise_converter", "noise_gen", "inner_hash"):
        assert hasattr(torch.ops.pearl_gemm, op)


def test_python_wrapper_defaults_match_reference():
    import inspect
    sig = inspect.signature(pg.noisy_gemm)
    assert sig.parameters["run_noising_B"].default is True
    assert sig.parameters["skip_reduction"].default is False
    names = list(sig.parameters)[:21]
    assert names == ["A", "B", "EAL", "EAL_fp16", "EBR", "EBR_fp16", "EAR_R_major", "EBL_R_major",
                     "EAR_K_major", "EBL_K_major", "AxEBL_fp16", "EARxBpEB_fp16", "ApEA", "BpEB",
                     "A_scales", "B_scales", "C", "host_signal_header_pinned", "host_signal_sync",
                     "pow_target", "pow_key"]


def test_validation_is_loud_on_cpu_tensors():
    A = torch.zeros(128, 256, dtype=torch.int8)
    C = torch.zeros(128, 256, dtype=torch.bfloat16)
    s = torch.ones(128)
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        pg.gemm(A, A, s, torch.ones(128), C)
    with pytest.raises(RuntimeError, match="No noise_gen kernel found"):
        pg.noise_gen(R=96, EAL=torch.zeros(4, 96, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="Need at least one int32"):
        pg.denoise_converter()


def test_constants():
    assert pg.kEALScaleFactorDenoise == -1 and pg.kEBRScaleFactorDenoise == -4
    t = pg.make_pow_target_tensor(2 ** 200 + 5, device="cpu")
    assert t.dtype == torch.uint32 and int(t[0]) == 5 and int(t[6]) == 2 ** 8


def test_pinned_pool_and_extract_indices():
    pool = pg.HostSignalHeaderPinnedPool(pool_size=2) if torch.cuda.is_available() else None
    if pool is not None:
        b = pool.acquire()
        pool.release(b)
    raw = pg.helpers._HeaderLayout()
    raw.status = 1
    raw.tileCoord[0], raw.tileCoord[1] = 3, 2
    raw.num_registers_per_thread = 128
    raw.mma_tile_size.m, raw.mma_tile_size.n = 128, 256
    for j in range(128):
        raw.thread_rows[j] = 16 + 8 * ((j >> 1) & 1)
        raw.thread_cols[j] = 4 + (j & 1) + 8 * (j >> 2)
    h = pg.HostSignalHeader(raw)
    idx = pg.extract_indices(h)
    assert idx.A_row_indices == [3 * 128 + 16, 3 * 128 + 24]
    assert idx.B_column_indices == sorted(2 * 256 + 4 + d + 8 * j for j in range(32) for d in (0, 1))


def test_required_scratchpad_bytes_formula():
    # tensor_hash_api.hpp:37-43: one 32-byte root per threads_per_block KiB.
    for nbytes, tpb in [(1, 128), (128 * 1024, 128), (128 * 1024 + 1, 128), (8192 * 8192, 128),
                        (10 ** 6, 256), (3 * 512 * 1024, 512)]:
        want = -(-nbytes // (tpb * 1024)) * 32
        assert pg.get_required_scratchpad_bytes(nbytes, tpb) == want


def test_tensor_hash_and_commitment_validation_on_cpu_tensors():
    key = torch.zeros(32, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        pg.tensor_hash(torch.zeros(4, 4, dtype=torch.uint8), key, key.clone(), key.clone())
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        pg.commitment_hash_from_merkle_roots(key, key, key, key.clone(), key.clone(), salted_dims=None)
