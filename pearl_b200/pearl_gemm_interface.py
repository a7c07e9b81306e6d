"""Drop-in mirror of ``pearl_gemm.pearl_gemm_interface`` backed by the B200
kernels (miner/pearl-gemm/src/pearl_gemm/pearl_gemm_interface.py:61-636).

Function names, argument names, argument order, defaults and the in-place
output contract are the reference's; each call validates its tensors with the
reference's rules (pearl_gemm_api.cpp:42-112) and raises ``RuntimeError`` on a
violation, then launches on the current torch CUDA stream through the C ABI
(include/pearl_b200.h).  Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

BLAKE3_DIGEST_SIZE_U32 = 8
KEY_LEN = 32

# pearl_gemm_constants.hpp:4-16 (re-exported by the reference pybind module)
kAxEBLScaleFactor = 1 << 14
kEARxBpEBScaleFactor = 1 << 12
kIntToFp16ScaleFactor = 1 << 12
kEBRScaleFactorDenoise = -1 * kAxEBLScaleFactor // kIntToFp16ScaleFactor
kEALScaleFactorDenoise = -1 * kEARxBpEBScaleFactor // kIntToFp16ScaleFactor


# ------------------------------------------------------------------ checks --
def _fail(msg: str):
    raise RuntimeError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_common(t: torch.Tensor, name: str, dtypes) -> None:
    if not t.is_cuda:
        _fail(f"{name} must be on CUDA")
    if not t.is_contiguous():
        _fail(f"{name} must be contiguous")
    if t.dtype not in dtypes:
        exp = " or ".join(str(d) for d in dtypes)
        _fail(f"expected dtype: {exp}but got this dtype: {t.dtype}")


def _check_tensor(t: torch.Tensor, shape: tuple, dtypes, name: str) -> None:
    _check_common(t, name, dtypes if isinstance(dtypes, (tuple, list)) else (dtypes,))
    if tuple(t.shape) != tuple(shape):
        _fail(f"{name} must have shape {tuple(shape)}")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _device_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def make_pow_target_tensor(value: int, device="cuda") -> torch.Tensor:
    """Create a pow_target tensor (8 x uint32, little-endian words) from a
    uint256 integer value (pearl_gemm_interface.py:8-16)."""
    words = [(value >> (32 * i)) & 0xFFFFFFFF for i in range(BLAKE3_DIGEST_SIZE_U32)]
    return torch.from_numpy(np.array(words, dtype=np.uint32)).to(device)


# --------------------------------------------------------- denoise_converter
def denoise_converter(
    EARxBpEB_in=None,  # (n, R), int32
    AxEBL_in=None,  # (m, R), int32
    EARxBpEB_out=None,  # (n, R), fp16
    AxEBL_out=None,  # (m, R), fp16
):
    """Convert int32 denoising factors to fp16 (x 2^-12 for EARxBpEB,
    x 2^-14 for AxEBL) (pearl_gemm_api.cpp:114-166)."""
    do_b = EARxBpEB_in is not None and EARxBpEB_out is not None
    do_a = AxEBL_in is not None and AxEBL_out is not None
    if not (do_a or do_b):
        _fail("Need at least one int32 denoising factor to convert")
    m = n = r = 0
    dev = None
    if do_a:
        m, r = AxEBL_in.shape
        _check_tensor(AxEBL_in, (m, r), torch.int32, "AxEBL_in")
        _check_tensor(AxEBL_out, (m, r), torch.float16, "AxEBL_out")
        dev = AxEBL_in.device
    if do_b:
        n, r = EARxBpEB_in.shape
        _check_tensor(EARxBpEB_in, (n, r), torch.int32, "EARxBpEB_in")
        _check_tensor(EARxBpEB_out, (n, r), torch.float16, "EARxBpEB_out")
        dev = EARxBpEB_in.device
    if r not in (64, 128):
        _fail(f"No denoise converter kernel found with given config: R = {r}")
    p = _lib.DenoiseConverterParams(
        device=dev.index if dev.index is not None else torch.cuda.current_device(), m=m, n=n, r=r,
        EARxBpEB_in=_ptr(EARxBpEB_in) if do_b else None, AxEBL_in=_ptr(AxEBL_in) if do_a else None,
        EARxBpEB_out=_ptr(EARxBpEB_out) if do_b else None, AxEBL_out=_ptr(AxEBL_out) if do_a else None)
    with torch.cuda.device(dev):
        _lib.call("pb2_denoise_converter", p, _stream(dev), "denoise_converter")


# ---------------------------------------------------------------- noise_gen
def noise_gen(
    R=128,
    num_threads=64,
    EAL=None,  # (m, R), int8
    EAL_fp16=None,  # (m, R), float16
    EAR_R_major=None,  # (k, R), int8
    EAR_K_major=None,  # (R, k), int8
    EBL_R_major=None,  # (k, R), int8
    EBL_K_major=None,  # (R, k), int8
    EBR=None,  # (n, R), int8
    EBR_fp16=None,  # (n, R), float16
    key_A=None,  # (32), uint8
    key_B=None,  # (32), uint8
    aux_buffer=None,  # (S), int32 or uint32
):
    """Generate the noise factors E{A,B}{L,R} from keyed BLAKE3 of the seed
    labels (pearl_gemm_api.cpp:168-298; protocol zk-pow/src/circuit/pearl_noise.rs).
    Unrequested outputs are skipped.  ``num_threads`` selects a CTA size in
    the reference; the B200 kernel sizes its own launch, the argument is
    validated only."""
    if num_threads not in (32, 64, 128):
        _fail(f"No noise_gen kernel found with given config: R = {R}, num_threads = {num_threads}")
    if R not in (64, 128):
        _fail(f"No noise_gen kernel found with given config: R = {R}, num_threads = {num_threads}")
    dims = {"m": 0, "n": 0, "k": 0}
    device = None

    def take(t, rows_key, cols_key, name, is_int8=True):
        nonlocal device
        if t is None:
            return None
        if device is None:
            device = t.device
        if t.device != device:
            _fail("Device id mismatch")
        if is_int8 and t.dtype != torch.int8:
            _fail(f"{name} must be int8")
        r_, c_ = t.shape
        for key, v in ((rows_key, r_), (cols_key, c_)):
            if key == "R":
                continue
            if dims[key] == 0:
                dims[key] = v
        shape = tuple(R if k_ == "R" else dims[k_] for k_ in (rows_key, cols_key))
        _check_tensor(t, shape, torch.int8 if is_int8 else torch.float16, name)
        return t.data_ptr()

    p = _lib.NoiseGenParams()
    p.EAL = take(EAL, "m", "R", "EAL")
    p.EAL_fp16 = take(EAL_fp16, "m", "R", "EAL_fp16", False)
    p.EAR_R_major = take(EAR_R_major, "k", "R", "EAR_R_major")
    p.EAR_K_major = take(EAR_K_major, "R", "k", "EAR_K_major")
    p.EBL_R_major = take(EBL_R_major, "k", "R", "EBL_R_major")
    p.EBL_K_major = take(EBL_K_major, "R", "k", "EBL_K_major")
    p.EBR = take(EBR, "n", "R", "EBR")
    p.EBR_fp16 = take(EBR_fp16, "n", "R", "EBR_fp16", False)
    if device is None:
        _fail("No noise matrices supplied")
    if dims["k"] % 16 != 0:
        _fail("K must be divisible by 16 (the size of a 128b vectorized copy atom)")
    expect_a = any(x is not None for x in (EAL, EAR_R_major, EAR_K_major))
    expect_b = any(x is not None for x in (EBL_R_major, EBL_K_major, EBR))
    for key, expect, name in ((key_A, expect_a, "key_A"), (key_B, expect_b, "key_B")):
        if expect != (key is not None):
            _fail(f"{name} must be given exactly when its noise matrices are requested")
        if key is not None:
            if key.device != device:
                _fail("Device id mismatch")
            _check_tensor(key, (KEY_LEN,), torch.uint8, name)
    if EAL_fp16 is not None and key_A is None or EBR_fp16 is not None and key_B is None:
        _fail("fp16 noise copies need the matching key")
    p.key_a = _ptr(key_A)
    p.key_b = _ptr(key_B)
    if aux_buffer is not None:
        if aux_buffer.device != device:
            _fail("Device id mismatch")
        if aux_buffer.shape[0] % 4 != 0:
            _fail("Aux buffer must be 16 byte aligned")
        _check_tensor(aux_buffer, (aux_buffer.shape[0],), (torch.uint32, torch.int32), "aux_buffer")
        p.aux_buffer = aux_buffer.data_ptr()
        p.aux_words = aux_buffer.shape[0]
    p.device = device.index if device.index is not None else torch.cuda.current_device()
    p.m, p.n, p.k, p.r = dims["m"], dims["n"], dims["k"], R
    with torch.cuda.device(device):
        _lib.call("pb2_noise_gen", p, _stream(device), "noise_gen")


# ---------------------------------------------------------- noise_A / noise_B
def _noising(X, EL, proj, XpE, E_rmajor, E_kmajor, rows_name, k_blocks_per_split, op,
             tile_rows, tile_k, stages):
    p = _noising_params(X, EL, proj, XpE, E_rmajor, E_kmajor, rows_name, k_blocks_per_split, op,
                        tile_rows, tile_k, stages)
    with torch.cuda.device(X.device):
        _lib.call("pb2_noise_A" if op == "noise_A" else "pb2_noise_B", p, _stream(X.device), op)


def _noising_params(X, EL, proj, XpE, E_rmajor, E_kmajor, rows_name, k_blocks_per_split, op,
                    tile_rows, tile_k, stages):
    rows, k = X.shape
    r = EL.shape[1]
    if k % 16 != 0:
        _fail("K must be divisible by 16 (the size of a 128b vectorized copy atom)")
    if tile_rows not in (None, 64, 128) or tile_k not in (None, 64, 128) or stages not in (2, 3, 4):
        _fail(f"No {op} kernel found with given config: R = {r}, b{rows_name}_noising = {tile_rows}")
    if k_blocks_per_split is not None and k_blocks_per_split > 0 and proj.dtype != torch.int32:
        _fail(f"{'AxEBL' if op == 'noise_A' else 'EARxBpEB'} should have int32 dtype for split-K. "
              f"It currently has {proj.dtype}.")
    if r not in (64, 128):
        _fail(f"No {op} kernel found with given config: R = {r}, b{rows_name}_noising = {tile_rows}")
    p = _lib.NoisingParams(
        device=_device_index(X), rows=rows, k=k, r=r, X=_ptr(X), EL=_ptr(EL), E_rmajor=_ptr(E_rmajor),
        E_kmajor=_ptr(E_kmajor), XpE=_ptr(XpE), proj=_ptr(proj),
        proj_is_fp16=int(proj.dtype == torch.float16),
        k_blocks_per_split=-1 if k_blocks_per_split is None else int(k_blocks_per_split))
    if proj.dtype == torch.float16:
        p.k_blocks_per_split = 0
    return p


def noise_A(
    A,  # m x k
    EAL,  # m x r
    AxEBL,  # m x r
    ApEA,  # m x k
    EAR=None,  # k x r
    EBL=None,  # r x k
    tile_size_m: int | None = None,
    tile_size_k: int | None = None,
    pipeline_stages: int = 2,
    k_blocks_per_split: int | None = None,
):
    """ApEA = A + EAL . EAR^T and AxEBL = A . EBL^T (x 2^-14 in fp16, exact and
    accumulated in int32) (pearl_gemm_api.cpp:300-398)."""
    m, k = A.shape
    r = EAL.shape[1]
    if EAR is None or EBL is None:
        _fail("Expected both of EAR, EBL.")
    _check_tensor(EAR, (k, r), torch.int8, "EAR")
    _check_tensor(EBL, (r, k), torch.int8, "EBL")
    _check_tensor(A, (m, k), torch.int8, "A")
    _check_tensor(EAL, (m, r), torch.int8, "EAL")
    _check_tensor(ApEA, (m, k), torch.int8, "ApEA")
    _check_tensor(AxEBL, (m, r), (torch.float16, torch.int32), "AxEBL")
    _noising(A, EAL, AxEBL, ApEA, EAR, EBL, "M", k_blocks_per_split, "noise_A", tile_size_m,
             tile_size_k, pipeline_stages)


def _noise_A_checks(A, EAL, AxEBL, ApEA, EAR, EBL):
    m, k = A.shape
    r = EAL.shape[1]
    _check_tensor(EAR, (k, r), torch.int8, "EAR")
    _check_tensor(EBL, (r, k), torch.int8, "EBL")
    _check_tensor(A, (m, k), torch.int8, "A")
    _check_tensor(EAL, (m, r), torch.int8, "EAL")
    _check_tensor(ApEA, (m, k), torch.int8, "ApEA")
    _check_tensor(AxEBL, (m, r), (torch.float16, torch.int32), "AxEBL")


def noise_B(
    B,  # n x k
    EBR,  # n x r
    EARxBpEB,  # n x r
    BpEB,  # n x k
    EAR=None,  # r x k
    EBL=None,  # k x r
    tile_size_n: int | None = None,
    tile_size_k: int | None = None,
    pipeline_stages: int = 2,
    k_blocks_per_split: int | None = None,
):
    """BpEB = B + EBR . EBL^T and EARxBpEB = BpEB . EAR^T (x 2^-12 in fp16)
    (pearl_gemm_api.cpp:400-500)."""
    n, k = B.shape
    r = EBR.shape[1]
    if EAR is None or EBL is None:
        _fail("Expected both of EAR, EBL.")
    _check_tensor(EBL, (k, r), torch.int8, "EBL")
    _check_tensor(EAR, (r, k), torch.int8, "EAR")
    _check_tensor(B, (n, k), torch.int8, "B")
    _check_tensor(EBR, (n, r), torch.int8, "EBR")
    _check_tensor(BpEB, (n, k), torch.int8, "BpEB")
    _check_tensor(EARxBpEB, (n, r), (torch.float16, torch.int32), "EARxBpEB")
    _noising(B, EBR, EARxBpEB, BpEB, EBL, EAR, "N", k_blocks_per_split, "noise_B", tile_size_n,
             tile_size_k, pipeline_stages)


def noise_AB(A, EAL, AxEBL, ApEA, B, EBR, EARxBpEB, BpEB, EAR_R_major, EBL_K_major, EAR_K_major,
             EBL_R_major, **_unused):
    """noise_A(A, EAL, AxEBL, ApEA, EAR=EAR_R_major, EBL=EBL_K_major) and
    noise_B(B, EBR, EARxBpEB, BpEB, EAR=EAR_K_major, EBL=EBL_R_major) of one
    mined GEMM: the noising step that noisy_gemm(run_noising_A=True,
    run_noising_B=True) runs before its GEMM (pearl_gemm_api.cpp:879-892),
    as one launch when both projections are fp16.  A B200 addition with no
    reference op of its own, so a caller can time that step apart from the
    GEMM; the factor tensors may be passed as the noise_gen output dict."""
    _noise_A_checks(A, EAL, AxEBL, ApEA, EAR_R_major, EBL_K_major)
    n, k = B.shape
    r = EBR.shape[1]
    _check_tensor(EBL_R_major, (k, r), torch.int8, "EBL")
    _check_tensor(EAR_K_major, (r, k), torch.int8, "EAR")
    _check_tensor(B, (n, k), torch.int8, "B")
    _check_tensor(EBR, (n, r), torch.int8, "EBR")
    _check_tensor(BpEB, (n, k), torch.int8, "BpEB")
    _check_tensor(EARxBpEB, (n, r), (torch.float16, torch.int32), "EARxBpEB")
    pa = _noising_params(A, EAL, AxEBL, ApEA, EAR_R_major, EBL_K_major, "M", None, "noise_A",
                         None, None, 2)
    pb = _noising_params(B, EBR, EARxBpEB, BpEB, EBL_R_major, EAR_K_major, "N", None, "noise_B",
                         None, None, 2)
    with torch.cuda.device(A.device):
        st = _lib.load().pb2_noise_AB(ctypes.byref(pa), ctypes.byref(pb),
                                      ctypes.c_void_p(_stream(A.device)))
        _lib.check(st, "noise_AB")


# ------------------------------------------------------------ gemm (plain) --
def _gemm_params(m, n, k, r, dev, tile_size_m, tile_size_n, tile_size_k, cluster_size_m,
                 cluster_size_n, pipeline_stages, swizzle, swizzle_n_maj):
    p = _lib.GemmParams()
    p.device = dev
    p.m, p.n, p.k, p.r = m, n, k, r
    p.tile_size_m, p.tile_size_n, p.tile_size_k = tile_size_m, tile_size_n, tile_size_k
    p.cluster_size_m, p.cluster_size_n = cluster_size_m, cluster_size_n
    p.pipeline_stages = pipeline_stages or 0
    p.swizzle = swizzle or 0
    p.swizzle_n_maj = int(bool(swizzle_n_maj))
    return p


def _check_matmul_config(op, bM, bN, bK, cM, cN, stages, r=None, extra=""):
    if (bM, bN, bK, cM, cN) != (128, 256, 128, 1, 1) or (stages is not None and stages not in (2, 3, 4, 5)):
        _fail(f"No {op} kernel found with given config: bM = {bM}, bN = {bN}, bK = {bK}, "
              + (f"R = {r}, " if r is not None else "")
              + f"stages = {stages}, cM = {cM}, cN = {cN}{extra}")


def gemm(
    A,  # m x k
    B,  # n x k
    A_scales,  # m
    B_scales,  # n
    C,  # m x n
    tile_size_m: int = 128,
    tile_size_n: int = 256,
    tile_size_k: int = 128,
    cluster_size_m: int = 1,
    cluster_size_n: int = 1,
    pipeline_stages: int | None = None,
    swizzle: int | None = None,
    swizzle_n_maj: bool = True,
):
    """C = bf16(A_scales * (A . B^T) * B_scales) without noising, transcript or
    denoising (pearl_gemm_api.cpp:502-616)."""
    m, k = A.shape
    n = B.shape[0]
    for t, name in ((A, "A"), (B, "B"), (A_scales, "A_scales"), (B_scales, "B_scales"), (C, "C")):
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
    _check_tensor(A, (m, k), torch.int8, "A")
    _check_tensor(B, (n, k), torch.int8, "B")
    _check_tensor(A_scales, (m,), torch.float32, "A_scales")
    _check_tensor(B_scales, (n,), torch.float32, "B_scales")
    _check_tensor(C, (m, n), torch.bfloat16, "C")
    if k % tile_size_k != 0:
        _fail("K must be divisible by bK")
    if n % 8 != 0:
        _fail("N must be divisible by 8")
    _check_matmul_config("gemm", tile_size_m, tile_size_n, tile_size_k, cluster_size_m,
                         cluster_size_n, pipeline_stages)
    p = _gemm_params(m, n, k, 128, _device_index(A), tile_size_m, tile_size_n, tile_size_k,
                     cluster_size_m, cluster_size_n, pipeline_stages, swizzle, swizzle_n_maj)
    p.ApEA, p.BpEB = _ptr(A), _ptr(B)
    p.A_scales, p.B_scales, p.C = _ptr(A_scales), _ptr(B_scales), _ptr(C)
    p.skip_reduction = 1
    p.skip_denoising = 1
    # A GEMM with too few tiles for the SMs (a decode batch) splits K; the
    # int32 partials need a workspace, taken from torch's caching allocator
    # (the stream-ordered allocator keeps it for the launches queued here).
    ws_bytes = _lib.load().pb2_gemm_workspace_bytes(p.device, m, n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=A.device) if ws_bytes > 0 else None
    if ws is not None:
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws_bytes
    with torch.cuda.device(A.device):
        _lib.call("pb2_gemm", p, _stream(A.device), "gemm")


# -------------------------------------------------------------- noisy_gemm --
def noisy_gemm(
    A,  # m x k
    B,  # n x k
    EAL,  # m x r
    EAL_fp16,  # m x r
    EBR,  # n x r
    EBR_fp16,
    EAR_R_major,  # k x r
    EBL_R_major,  # k x r
    EAR_K_major,  # r x k
    EBL_K_major,  # r x k
    AxEBL_fp16,  # m x r
    EARxBpEB_fp16,  # n x r
    ApEA,  # m x k
    BpEB,  # n x k
    A_scales,  # m
    B_scales,  # n
    C,  # m x n
    host_signal_header_pinned,  # host_signal_header_size
    host_signal_sync,  # host_signal_sync_size
    pow_target: torch.Tensor,  # (8,) uint32
    pow_key: torch.Tensor,  # (8,) uint32
    AxEBL_int32=None,  # m x r
    EARxBpEB_int32=None,  # n x r
    tile_size_m: int = 128,
    tile_size_n: int = 256,
    tile_size_k: int = 128,
    cluster_size_m: int = 1,
    cluster_size_n: int = 1,
    pipeline_stages: int | None = None,
    swizzle: int | None = None,
    swizzle_n_maj: bool = True,
    tile_size_m_noising_A: int | None = None,
    tile_size_n_noising_B: int | None = None,
    tile_size_k_noising_A: int | None = None,
    tile_size_k_noising_B: int | None = None,
    pipeline_stages_noising_A: int = 2,
    pipeline_stages_noising_B: int = 2,
    k_blocks_per_split_noising_A: int | None = None,
    k_blocks_per_split_noising_B: int | None = None,
    run_noising_A: bool = True,
    run_noising_B: bool = True,
    skip_reduction: bool = False,
    skip_denoising: bool = False,
    inner_hash_counter: torch.Tensor | None = None,
    enable_debug: bool = False,
    *,
    hits: torch.Tensor | None = None,
    transcripts: torch.Tensor | None = None,
    digests: torch.Tensor | None = None,
):
    """Noising, mined matmul (transcript + keyed BLAKE3 + target compare) and
    denoising in one call (pearl_gemm_api.cpp:618-936):

        ApEA = A + EAL . EAR,  BpEB = B + EBR . EBL
        C = A_scales * (ApEA . BpEB^T - AxEBL . EBR^T - EAL . EARxBpEB^T) * B_scales

    B200 extensions (keyword-only, optional): ``hits`` (int32/uint32 tensor of
    shape (capacity, 12): every hit as {row_off, col_off, tile_m, tile_n,
    digest[8]}, count in host_signal_sync word 2), ``transcripts`` ((m/2)*(n/64),
    16) and ``digests`` ((m/2)*(n/64), 8) uint32 debug dumps of every protocol
    hash tile."""
    m, k = A.shape
    n = B.shape[0]
    r = EAL.shape[1]
    if host_signal_header_pinned.dtype != torch.int8:
        _fail("host_signal_header_pinned should have int8 dtype. It currently has "
              f"{host_signal_header_pinned.dtype}.")
    if host_signal_sync.dtype != torch.int8:
        _fail(f"host_signal_sync should have int8 dtype. It currently has {host_signal_sync.dtype}.")
    for t, name in ((pow_target, "pow_target"), (pow_key, "pow_key")):
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
        if t.dtype != torch.uint32:
            _fail(f"{name} must be uint32 dtype. It currently has {t.dtype}.")
        if tuple(t.shape) != (BLAKE3_DIGEST_SIZE_U32,):
            _fail(f"{name} must have shape (8)")
    if tile_size_m > 256:
        _fail("bN must be less than or equal to 256, host signal header limits thread rows to uint8")
    if tile_size_n > 256:
        _fail("bM must be less than or equal to 256, host signal header limits thread cols to uint8")
    if EAR_R_major is None or EBL_R_major is None or EAR_K_major is None or EBL_K_major is None:
        _fail("Expected all of EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major.")
    _check_tensor(EAR_R_major, (k, r), torch.int8, "EAR_R_major")
    _check_tensor(EBL_R_major, (k, r), torch.int8, "EBL_R_major")
    _check_tensor(EAR_K_major, (r, k), torch.int8, "EAR_K_major")
    _check_tensor(EBL_K_major, (r, k), torch.int8, "EBL_K_major")
    if EAL_fp16 is None or EBR_fp16 is None:
        _fail("Expected both of EAL_fp16, EBR_fp16.")
    _check_tensor(EAL_fp16, (m, r), torch.float16, "EAL_fp16")
    _check_tensor(EBR_fp16, (n, r), torch.float16, "EBR_fp16")
    if AxEBL_int32 is not None:
        _check_tensor(AxEBL_int32, (m, r), torch.int32, "AxEBL_int32")
    if EARxBpEB_int32 is not None:
        _check_tensor(EARxBpEB_int32, (n, r), torch.int32, "EARxBpEB_int32")
    _check_tensor(A, (m, k), torch.int8, "A")
    _check_tensor(B, (n, k), torch.int8, "B")
    _check_tensor(EAL, (m, r), torch.int8, "EAL")
    _check_tensor(EBR, (n, r), torch.int8, "EBR")
    _check_tensor(ApEA, (m, k), torch.int8, "ApEA")
    _check_tensor(BpEB, (n, k), torch.int8, "BpEB")
    _check_tensor(AxEBL_fp16, (m, r), torch.float16, "AxEBL_fp16")
    _check_tensor(EARxBpEB_fp16, (n, r), torch.float16, "EARxBpEB_fp16")
    _check_tensor(A_scales, (m,), torch.float32, "A_scales")
    _check_tensor(B_scales, (n,), torch.float32, "B_scales")
    _check_tensor(C, (m, n), torch.bfloat16, "C")
    if tuple(host_signal_header_pinned.shape) != (_lib.HOST_SIGNAL_HEADER_SIZE,):
        _fail(f"host_signal_header_pinned must have shape ({_lib.HOST_SIGNAL_HEADER_SIZE})")
    if tuple(host_signal_sync.shape) != (_lib.HOST_SIGNAL_SYNC_SIZE,):
        _fail(f"host_signal_sync must have shape ({_lib.HOST_SIGNAL_SYNC_SIZE})")
    if not host_signal_sync.is_cuda:
        _fail("host_signal_sync must be on CUDA")
    if host_signal_header_pinned.is_cuda or not host_signal_header_pinned.is_pinned():
        _fail("host_signal_header_pinned must be a pinned CPU tensor")
    if k % tile_size_k != 0:
        _fail("K must be divisible by bK")
    if n % 8 != 0:
        _fail("N must be divisible by 8")
    for kbps, t, name in ((k_blocks_per_split_noising_A, AxEBL_int32, "AxEBL"),
                          (k_blocks_per_split_noising_B, EARxBpEB_int32, "EARxBpEB")):
        if kbps is not None and kbps > 0 and t is None:
            _fail(f"{name} should have int32 dtype for split-K. It currently has torch.float16.")
    if enable_debug and inner_hash_counter is None:
        _fail("inner_hash_counter must be provided when enable_debug is True")
    extra = (f", SkipReduction = {'true' if skip_reduction else 'false'}"
             f", SkipDenoising = {'true' if skip_denoising else 'false'}")
    _check_matmul_config("noisy_gemm", tile_size_m, tile_size_n, tile_size_k, cluster_size_m,
                         cluster_size_n, pipeline_stages, r, extra)
    if r not in (64, 128):
        _fail(f"No noisy_gemm kernel found with given config: R = {r}")
    for noising_tile in (tile_size_m_noising_A, tile_size_n_noising_B, tile_size_k_noising_A,
                         tile_size_k_noising_B):
        if noising_tile not in (None, 64, 128):
            _fail(f"No noise kernel found with given config: tile = {noising_tile}")

    p = _gemm_params(m, n, k, r, _device_index(A), tile_size_m, tile_size_n, tile_size_k,
                     cluster_size_m, cluster_size_n, pipeline_stages, swizzle, swizzle_n_maj)
    p.A, p.B, p.EAL, p.EBR = _ptr(A), _ptr(B), _ptr(EAL), _ptr(EBR)
    p.EAR_R_major, p.EBL_R_major = _ptr(EAR_R_major), _ptr(EBL_R_major)
    p.EAR_K_major, p.EBL_K_major = _ptr(EAR_K_major), _ptr(EBL_K_major)
    p.AxEBL_int32, p.EARxBpEB_int32 = _ptr(AxEBL_int32), _ptr(EARxBpEB_int32)
    p.ApEA, p.BpEB = _ptr(ApEA), _ptr(BpEB)
    p.EAL_fp16, p.EBR_fp16 = _ptr(EAL_fp16), _ptr(EBR_fp16)
    p.AxEBL_fp16, p.EARxBpEB_fp16 = _ptr(AxEBL_fp16), _ptr(EARxBpEB_fp16)
    p.A_scales, p.B_scales, p.C = _ptr(A_scales), _ptr(B_scales), _ptr(C)
    p.host_signal_header_pinned = _ptr(host_signal_header_pinned)
    p.host_signal_sync = _ptr(host_signal_sync)
    p.pow_target, p.pow_key = _ptr(pow_target), _ptr(pow_key)
    p.run_noising_a, p.run_noising_b = int(bool(run_noising_A)), int(bool(run_noising_B))
    p.k_blocks_per_split_noising_a = -1 if k_blocks_per_split_noising_A is None else k_blocks_per_split_noising_A
    p.k_blocks_per_split_noising_b = -1 if k_blocks_per_split_noising_B is None else k_blocks_per_split_noising_B
    p.skip_reduction, p.skip_denoising = int(bool(skip_reduction)), int(bool(skip_denoising))
    if inner_hash_counter is not None:
        _check_common(inner_hash_counter, "inner_hash_counter", (torch.int64, torch.uint64))
        p.inner_hash_counter = _ptr(inner_hash_counter)
    p.enable_debug = int(bool(enable_debug))
    if hits is not None:
        _check_common(hits, "hits", (torch.int32, torch.uint32))
        if hits.dim() != 2 or hits.shape[1] != _lib.HIT_WORDS:
            _fail(f"hits must have shape (capacity, {_lib.HIT_WORDS})")
        p.hits, p.hit_capacity = _ptr(hits), hits.shape[0]
    for t, words, name in ((transcripts, 16, "transcripts"), (digests, 8, "digests")):
        if t is None:
            continue
        if m % 16 or n % 256:
            _fail(f"{name} dumps need m % 16 == 0 and n % 256 == 0")
        _check_tensor(t, ((m // 2) * (n // 64), words), (torch.int32, torch.uint32), name)
    p.transcripts, p.digests = _ptr(transcripts), _ptr(digests)
    with torch.cuda.device(A.device):
        _lib.call("pb2_noisy_gemm", p, _stream(A.device), "noisy_gemm")


# ------------------------------------------------------------- tensor_hash --
DEFAULT_THREADS_PER_BLOCK = 128  # tensor_hash_api.hpp:21-23
DEFAULT_NUM_STAGES = 2
DEFAULT_LEAVES_PER_MT_BLOCK = 512
BLAKE3_CHAINING_VALUE_SIZE = 32


def get_required_scratchpad_bytes(matrix_bytes: int,
                                  threads_per_block: int = DEFAULT_THREADS_PER_BLOCK) -> int:
    """Scratch bytes tensor_hash needs for a tensor of ``matrix_bytes`` bytes:
    one 32-byte subtree root per ``threads_per_block`` KiB chunks
    (tensor_hash_api.hpp:37-43)."""
    return int(_lib.load().pb2_required_scratchpad_bytes(int(matrix_bytes), int(threads_per_block)))


def tensor_hash(
    data,
    key,
    out,
    roots,
    threads_per_block=DEFAULT_THREADS_PER_BLOCK,
    num_stages=DEFAULT_NUM_STAGES,
    leaves_per_mt_block=DEFAULT_LEAVES_PER_MT_BLOCK,
):
    """out = BLAKE3 keyed by ``key`` of ``data``'s bytes zero-padded to whole
    1 KiB chunks; ``roots`` is scratch of at least
    get_required_scratchpad_bytes(data.numel(), threads_per_block) bytes
    (tensor_hash_api.hpp:45-120; pearl_gemm_interface.py:550-578).
    ``num_stages`` and ``leaves_per_mt_block`` are validated like the
    reference's tuning knobs but select nothing here."""
    for t, name in ((data, "data"), (key, "key"), (out, "out"), (roots, "roots")):
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
    if key.dtype != torch.uint8:
        _fail("key must be uint8")
    if out.dtype != torch.uint8:
        _fail("out must be uint8")
    if roots.dtype != torch.uint8:
        _fail("roots must be uint8")
    if data.dim() != 2:
        _fail("data must be 2D tensor")
    if data.data_ptr() % 16 != 0:
        _fail("data must be 16-byte aligned for TMA")
    if key.numel() != KEY_LEN:
        _fail(f"key must have exactly{KEY_LEN}bytes")
    if out.numel() != BLAKE3_CHAINING_VALUE_SIZE:
        _fail(f"out must have exactly{BLAKE3_CHAINING_VALUE_SIZE}bytes")
    if roots.numel() % BLAKE3_CHAINING_VALUE_SIZE != 0:
        _fail(f"roots must have a multiple of{BLAKE3_CHAINING_VALUE_SIZE}bytes")
    if threads_per_block not in (128, 256, 512):
        _fail("threads_per_block must be 128, 256, or 512")
    if num_stages not in (2, 3, 4):
        _fail("num_stages must be 2, 3, or 4")
    if leaves_per_mt_block not in (256, 512, 1024):
        _fail("leaves_per_mt_block must be 256, 512, or 1024")
    nbytes = data.numel() * data.element_size()
    need = get_required_scratchpad_bytes(nbytes, threads_per_block)
    if roots.numel() < need:
        _fail(f"roots must have at least {need // 32} * {BLAKE3_CHAINING_VALUE_SIZE}bytes")
    if nbytes == 0:
        _fail("data must be non-empty")
    p = _lib.TensorHashParams()
    p.device = _device_index(data)
    p.data, p.len, p.key, p.out = data.data_ptr(), nbytes, key.data_ptr(), out.data_ptr()
    p.roots, p.roots_bytes, p.threads_per_block = roots.data_ptr(), roots.numel(), threads_per_block
    with torch.cuda.device(data.device):
        _lib.call("pb2_tensor_hash", p, _stream(data.device), "tensor_hash")


def commitment_hash_from_merkle_roots(
    A_merkle_root,
    B_merkle_root,
    key,
    A_commitment_hash,
    B_commitment_hash,
    routing_root=None,
    offsets_hash=None,
    *,
    salted_dims: tuple[int, int] | None,
):
    """Noise seeds from the two tensor roots (tensor_hash_api.hpp:124-212;
    pearl_gemm_interface.py:581-608): ``salted_dims=(m, n)`` for V3 salted
    seeds, ``None`` for the legacy chain; ``routing_root`` and
    ``offsets_hash`` (MoE) fold the routing commitment into A's root."""
    named = [(A_merkle_root, "A_merkle_root"), (B_merkle_root, "B_merkle_root"), (key, "key"),
             (A_commitment_hash, "A_commitment_hash"), (B_commitment_hash, "B_commitment_hash")]
    for t, name in named:
        if name in ("A_merkle_root", "B_merkle_root", "key") and not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
        if t.dtype != torch.uint8:
            _fail(f"{name} must be uint8")
        if t.numel() != BLAKE3_CHAINING_VALUE_SIZE:
            _fail(f"{name} must have exactly{BLAKE3_CHAINING_VALUE_SIZE}bytes")
    if (routing_root is None) != (offsets_hash is None):
        _fail("routing_root and offsets_hash must be provided together")
    for t, name in ((routing_root, "routing_root"), (offsets_hash, "offsets_hash")):
        if t is None:
            continue
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
        if t.dtype != torch.uint8:
            _fail(f"{name} must be uint8")
        if t.numel() != BLAKE3_CHAINING_VALUE_SIZE:
            _fail(f"{name} must have exactly{BLAKE3_CHAINING_VALUE_SIZE}bytes")
    p = _lib.CommitmentParams()
    p.device = _device_index(A_merkle_root)
    p.A_merkle_root, p.B_merkle_root, p.key = _ptr(A_merkle_root), _ptr(B_merkle_root), _ptr(key)
    p.A_commitment_hash, p.B_commitment_hash = _ptr(A_commitment_hash), _ptr(B_commitment_hash)
    p.routing_root, p.offsets_hash = _ptr(routing_root), _ptr(offsets_hash)
    if salted_dims is not None:
        for d, name in zip(salted_dims, ("salted_dim_a", "salted_dim_b")):
            if not 0 < int(d) <= 0xFFFFFFFF:
                _fail(f"{name} must be in [1, {0xFFFFFFFF}], got {d}")
        p.salted, p.salted_dim_a, p.salted_dim_b = 1, int(salted_dims[0]), int(salted_dims[1])
    with torch.cuda.device(A_merkle_root.device):
        _lib.call("pb2_commitment_hash_from_merkle_roots", p, _stream(A_merkle_root.device),
                  "commitment_hash_from_merkle_roots")


# ------------------------------------------------------------ test helpers --
def inner_hash(input_buffer: torch.Tensor, iterations: int = 1) -> torch.Tensor:
    """XOR of a 64..256-word uint32 buffer, added up ``iterations`` times
    (pearl_gemm_api.cpp:939-970)."""
    if not input_buffer.is_cuda:
        _fail("input_buffer must be on CUDA")
    if not input_buffer.is_contiguous():
        _fail("input_buffer must be contiguous")
    if input_buffer.dtype != torch.uint32:
        _fail("Input must be uint32 tensor")
    if input_buffer.shape[0] not in (64, 96, 128, 192, 256):
        _fail("Input must have size equal to valid_sizes=(64, 96, 128, 192, 256)")
    if input_buffer.dim() != 1:
        _fail("Input must be 1D tensor")
    if iterations not in (1, 100000):
        _fail("Iterations must be 1 or 100000")
    out = torch.empty(1, dtype=torch.uint32, device=input_buffer.device)
    L = _lib.load()
    with torch.cuda.device(input_buffer.device):
        st = L.pb2_inner_hash(_device_index(input_buffer), input_buffer.data_ptr(),
                              input_buffer.shape[0], out.data_ptr(), iterations,
                              _stream(input_buffer.device))
        _lib.check(st, "inner_hash")
        torch.cuda.current_stream(input_buffer.device).synchronize()
    return out


def get_host_signal_header_size() -> int:
    return _lib.HOST_SIGNAL_HEADER_SIZE


def get_host_signal_sync_size() -> int:
    return _lib.HOST_SIGNAL_SYNC_SIZE
