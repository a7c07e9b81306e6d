"""The mining layer of miner/vllm-miner, on the B200 operators.

Mirrors the calls a mined vLLM layer makes into ``pearl_gemm``, in the
reference's order and with the reference's arguments:

* ``quant_7bit`` / ``quant_8bit``: quantization_operators.py:72-100;
* ``pearl_gemm_vanilla`` / ``pearl_gemm_noisy``: gemm_operators.py:28-333
  (tensor hashes of A and B, commitment seeds, noise generation, the mined
  GEMM with in-kernel noising);
* the MoE GEMM1 path: moe_gemm_operators.py:118-329 and
  pearl_moe_experts.py:262-375 (routing order, routing commitment, A-side
  permutation, one mined GEMM per expert);
* ``PearlLinear.apply_weights``: the mining / non-mining branches of
  vllm_kernels.py:154-247.

What sits outside the GPU path is passed in rather than fetched: the
gateway's mining job becomes a ``MiningJob`` value (its hash key, adjusted
target and seed derivation), and the asynchronous proof submission is left to
the caller, which receives the pinned host-signal header, the sync word and
the commitment hashes of every mined GEMM (``MinedGemm``)."""

from __future__ import annotations

import weakref
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from . import pearl_gemm_interface as P
from .helpers import HostSignalHeaderPinnedPool, get_host_signal_sync_fields
from .moe import build_routing_data, get_build_routing_data_scratchpad_bytes, scatter_rows
from .moe import noisy_gemm_grouped as grouped_noisy_gemm
from .quantization import quantize

MAX_VAL_7BIT = 63
MAX_VAL_8BIT = 127
NO_HADAMARD_BLOCK_SIZE = 0  # quantization_operators.py:7-9


@dataclass(frozen=True)
class MiningConfig:
    """miner-base MinerSettings fields and vllm-miner config.yaml thresholds
    the operators read (settings.py:6-48, config.yaml:9-12)."""

    noise_rank: int = 128
    tile_size_m: int = 128
    tile_size_n: int = 256
    tile_size_k: int = 128
    min_m: int = 1024
    min_n: int = 256
    min_k: int = 1024

    def should_use_noisy_gemm(self, m: int, n: int, k: int) -> bool:
        """config.py:36-44."""
        if n == 1 or k == 1 or m == 1:
            return False
        return m >= self.min_m and n >= self.min_n and k >= self.min_k


@dataclass(frozen=True)
class MiningJob:
    """The parts of the gateway's mining job the GEMM consumes: the 32-byte
    commitment key (CommitmentHasher.get_key of the block header), the
    difficulty target after the protocol's penalty (MiningJob.adjust_target)
    and whether seeds are salted with the matrix dimensions (V3 certs)."""

    hash_key: bytes
    pow_target: int
    salted_seeds: bool = True


@dataclass
class MinedGemm:
    """What one mined GEMM leaves for the proof path (the reference hands
    these to StatusCheckCallback, callbacks.py:22-64)."""

    host_signal_header_pinned: torch.Tensor
    host_signal_sync: torch.Tensor
    commitment_hash_A: torch.Tensor
    commitment_hash_B: torch.Tensor
    hits: torch.Tensor | None = None

    def sync_fields(self) -> dict:
        return get_host_signal_sync_fields(self.host_signal_sync)


_POOL: HostSignalHeaderPinnedPool | None = None


def _pinned_header() -> torch.Tensor:
    global _POOL
    if _POOL is None:
        _POOL = HostSignalHeaderPinnedPool(128)  # mining_state.py:60-66
    return _POOL.acquire()


def release_header(header: torch.Tensor) -> None:
    if _POOL is not None:
        _POOL.release(header)


def _u8(b: bytes, device) -> torch.Tensor:
    return torch.frombuffer(bytearray(b), dtype=torch.uint8).to(device)


_JOB_TENSORS: "OrderedDict[tuple, tuple[torch.Tensor, torch.Tensor]]" = OrderedDict()


def _job_tensors(job: MiningJob, device) -> tuple[torch.Tensor, torch.Tensor]:
    """The job's commitment key and pow target as device tensors, made once
    per (job, device): a copy from pageable host memory waits for the
    stream, and every mined GEMM of a job reads the same two values.  The
    cached tensors are never written."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    k = (job.hash_key, job.pow_target, idx)
    hit = _JOB_TENSORS.get(k)
    if hit is None:
        hit = (_u8(job.hash_key, dev), P.make_pow_target_tensor(job.pow_target, dev))
        _JOB_TENSORS[k] = hit
        while len(_JOB_TENSORS) > 64:
            _JOB_TENSORS.popitem(last=False)
    else:
        _JOB_TENSORS.move_to_end(k)
    return hit


# ------------------------------------------------------------ quantization --
def quant_7bit(x, smooth_scale=None, block_size: int = NO_HADAMARD_BLOCK_SIZE):
    return _quant(x, MAX_VAL_7BIT, smooth_scale, block_size)


def quant_8bit(x, smooth_scale=None, block_size: int = NO_HADAMARD_BLOCK_SIZE):
    return _quant(x, MAX_VAL_8BIT, smooth_scale, block_size)


def _quant(x, max_val, smooth_scale, block_size):
    """quantization_operators.py:38-69: (x_q int8, x_s (M, 1) fp32, None)."""
    m, n = x.shape
    x_q = torch.empty_like(x, dtype=torch.int8)
    x_s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    smooth = None
    if smooth_scale is not None:
        s = smooth_scale.to(dtype=torch.float32, device=x.device)
        smooth = (s.unsqueeze(0) if s.ndim == 1 else s).contiguous()
    quantize(x, x_q, x_s, smooth_scale=smooth, max_val=max_val, block_size=block_size)
    return x_q, x_s, None


# ------------------------------------------------------------------ dense --
def pearl_gemm_vanilla(A, B, scale_a, scale_b, out_dtype, config: MiningConfig = MiningConfig()):
    """C = A . B^T scaled, without mining (gemm_operators.py:28-65)."""
    assert out_dtype is torch.bfloat16 or out_dtype is torch.float16
    C = torch.empty((A.shape[0], B.shape[0]), dtype=out_dtype, device=A.device)
    P.gemm(A=A, B=B, A_scales=scale_a, B_scales=scale_b, C=C, tile_size_m=config.tile_size_m,
           tile_size_n=config.tile_size_n, tile_size_k=config.tile_size_k)
    return C


def generate_noise_factors(m, n, k, r, commitment_hash_A, commitment_hash_B, device):
    """gemm_operators.py:267-333."""
    e = lambda *s, dt=torch.int8: torch.empty(s, dtype=dt, device=device)  # noqa: E731
    EAL, EBR = e(m, r), e(n, r)
    EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major = e(k, r), e(k, r), e(r, k), e(r, k)
    EAL_fp16, EBR_fp16 = e(m, r, dt=torch.float16), e(n, r, dt=torch.float16)
    P.noise_gen(R=r, EAL=EAL, EAL_fp16=EAL_fp16, EAR_R_major=EAR_R_major, EAR_K_major=EAR_K_major,
                EBL_R_major=EBL_R_major, EBL_K_major=EBL_K_major, EBR=EBR, EBR_fp16=EBR_fp16,
                key_A=commitment_hash_A, key_B=commitment_hash_B)
    return EAL, EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major, EBR, EAL_fp16, EBR_fp16


def _tensor_root(data_u8: torch.Tensor, key: torch.Tensor, scratch: torch.Tensor | None = None):
    out = torch.empty(32, dtype=torch.uint8, device=data_u8.device)
    if scratch is None:
        scratch = torch.empty(P.get_required_scratchpad_bytes(data_u8.numel()), dtype=torch.uint8,
                              device=data_u8.device)
    P.tensor_hash(data_u8, key, out, scratch)
    return out


_SIDE_STREAMS: dict[int, torch.cuda.Stream] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = _SIDE_STREAMS.get(idx)
    if s is None:
        s = _SIDE_STREAMS[idx] = torch.cuda.Stream(device)
    return s


def _tensor_root_async(data_u8: torch.Tensor, key: torch.Tensor):
    """The tensor_hash root of ``data_u8`` computed on a side stream, so that
    it overlaps the caller's next kernels (the other operand's hash, the
    activation quantization).  Returns (root, event); the caller's stream
    waits on the event before it reads root."""
    main = torch.cuda.current_stream(data_u8.device)
    side = _side_stream(data_u8.device)
    side.wait_stream(main)  # the data and the key are ready
    with torch.cuda.stream(side):
        root = _tensor_root(data_u8, key)
    data_u8.record_stream(side)
    key.record_stream(side)
    root.record_stream(main)
    done = torch.cuda.Event()
    done.record(side)
    return root, done


_B_ROOTS: "OrderedDict[tuple, tuple]" = OrderedDict()


def weight_root(weight: torch.Tensor, job: MiningJob):
    """(root, event) of the tensor_hash of a weight under a job's key,
    hashed once per (weight, job) instead of once per GEMM.

    Within a job the key is fixed and a layer's weight bytes do not change,
    so the root -- and the commitment seeds built from it -- are the same
    for every GEMM of that weight: the reference re-hashes B each time
    (gemm_operators.py:96-100), here the first GEMM hashes it (on the side
    stream, as _tensor_root_async) and later ones reuse the result.  An
    entry is keyed by the weight object itself (held weakly, so a new tensor
    at a recycled address never matches) and by its version counter, which
    every in-place write to the weight advances."""
    dev = weight.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    k = (id(weight), weight._version, job.hash_key, idx)
    hit = _B_ROOTS.get(k)
    if hit is not None and hit[0]() is weight:
        _B_ROOTS.move_to_end(k)
        return hit[1], hit[2]
    key_tensor = _job_tensors(job, dev)[0]
    root, done = _tensor_root_async(weight.contiguous().view(torch.uint8), key_tensor)
    _B_ROOTS[k] = (weakref.ref(weight), root, done)
    while len(_B_ROOTS) > 1024:
        _B_ROOTS.popitem(last=False)
    return root, done


def pearl_gemm_noisy(a, b, scale_a, scale_b, out_dtype, job: MiningJob,
                     config: MiningConfig = MiningConfig(), *, hits: torch.Tensor | None = None,
                     b_root=None):
    """Mined C = A . B^T (gemm_operators.py:68-264): commitment to A and B,
    seeded noise, noisy GEMM with the fused transcript / BLAKE3 / target
    check, denoised bf16 output.  Returns (C, MinedGemm).  B's root is
    hashed on a side stream beside A's, or taken from ``b_root`` (the
    (root, event) of an earlier _tensor_root_async of the same B and key)."""
    assert out_dtype is torch.bfloat16 or out_dtype is torch.float16
    m, k = a.shape
    n = b.shape[0]
    r = config.noise_rank
    device = a.device
    C = torch.empty((m, n), dtype=out_dtype, device=device)
    key_tensor, target_tensor = _job_tensors(job, device)
    if b_root is None:
        b_root = _tensor_root_async(b.view(torch.uint8), key_tensor)
    A_root = _tensor_root(a.view(torch.uint8), key_tensor)
    B_root, b_ready = b_root
    torch.cuda.current_stream(device).wait_event(b_ready)
    ch_A = torch.empty(32, device=device, dtype=torch.uint8)
    ch_B = torch.empty(32, device=device, dtype=torch.uint8)
    P.commitment_hash_from_merkle_roots(A_root, B_root, key_tensor, ch_A, ch_B,
                                        salted_dims=(m, n) if job.salted_seeds else None)
    EAL, EAR_R, EBL_R, EAR_K, EBL_K, EBR, EAL_fp16, EBR_fp16 = generate_noise_factors(
        m, n, k, r, ch_A, ch_B, device)
    BpEB = torch.empty((n, k), dtype=torch.int8, device=device)
    EARxBpEB = torch.empty((n, r), dtype=torch.float16, device=device)
    ApEA = torch.empty((m, k), dtype=torch.int8, device=device)
    A_E_BL = torch.empty((m, r), dtype=torch.float16, device=device)
    sync = torch.zeros((P.get_host_signal_sync_size(),), dtype=torch.int8, device=device)
    header = _pinned_header()
    P.noisy_gemm(A=a, B=b, EAL=EAL, EAL_fp16=EAL_fp16, EBR=EBR, EBR_fp16=EBR_fp16,
                 EAR_R_major=EAR_R, EBL_R_major=EBL_R, EAR_K_major=EAR_K, EBL_K_major=EBL_K,
                 AxEBL_fp16=A_E_BL, EARxBpEB_fp16=EARxBpEB, ApEA=ApEA, BpEB=BpEB, A_scales=scale_a,
                 B_scales=scale_b, C=C, host_signal_header_pinned=header, host_signal_sync=sync,
                 pow_target=target_tensor,
                 pow_key=ch_A.view(torch.uint32), tile_size_m=config.tile_size_m,
                 tile_size_n=config.tile_size_n, tile_size_k=config.tile_size_k, run_noising_A=True,
                 run_noising_B=True, skip_reduction=False, skip_denoising=False, hits=hits)
    return C, MinedGemm(header, sync, ch_A, ch_B, hits)


class PearlLinear:
    """The mining / non-mining ``apply_weights`` of PearlKernel
    (vllm_kernels.py:154-247) for a layer holding ``weight`` (n, k) int7/int8,
    ``weight_scale`` (n,) or (n, 1) fp32 and optionally ``smooth_quant_scale``
    (k,) and ``hadamard_block_size``."""

    def __init__(self, mining_enabled: bool = True, config: MiningConfig = MiningConfig(),
                 job: MiningJob | None = None):
        self.mining_enabled = mining_enabled
        self.config = config
        self.job = job
        self.mined: list[MinedGemm] = []

    def apply_weights(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        w_q, w_s = layer.weight, layer.weight_scale
        smooth = getattr(layer, "smooth_quant_scale", None)
        block = int(getattr(layer, "hadamard_block_size", NO_HADAMARD_BLOCK_SIZE))
        if self.mining_enabled:
            k, n = x.shape[-1], w_q.shape[0]
            m = x.numel() // k
            noisy = self.config.should_use_noisy_gemm(m, n, k) and self.job is not None
            # the weight's commitment root does not depend on x: hashed once
            # per (weight, job), beside the quantization
            b_root = weight_root(w_q, self.job) if noisy else None
            x_q, x_s, _ = quant_7bit(x, smooth_scale=smooth, block_size=block)
            if noisy:
                C, mined = pearl_gemm_noisy(x_q.contiguous(), w_q.contiguous(), x_s.squeeze(-1),
                                            w_s.reshape(-1), x.dtype, self.job, self.config, b_root=b_root)
                self.mined.append(mined)
                return C
            return pearl_gemm_vanilla(x_q.contiguous(), w_q.contiguous(), x_s.squeeze(-1),
                                      w_s.reshape(-1), x.dtype, self.config)
        x_q, x_s, _ = quant_8bit(x, smooth_scale=smooth, block_size=block)
        return pearl_gemm_vanilla(x_q.contiguous(), w_q.contiguous(), x_s.squeeze(-1),
                                  w_s.reshape(-1), x.dtype, self.config)


# --------------------------------------------------------------------- MoE --
@dataclass
class MoERoutingLayout:
    """Canonical per-expert slot order (moe_gemm_operators.py:27-64)."""

    token_indices: torch.Tensor
    slot_indices: torch.Tensor
    routing_offsets: torch.Tensor
    routing_offsets_host: list[int]
    num_experts: int
    top_k: int

    def expert_slice(self, expert_idx: int) -> tuple[int, int]:
        start = 0 if expert_idx == 0 else self.routing_offsets_host[expert_idx - 1]
        return start, self.routing_offsets_host[expert_idx] - start


@dataclass
class MoENoiseContext:
    """moe_gemm_operators.py:67-87."""

    commitment_hash_A: torch.Tensor
    commitment_hash_B: torch.Tensor
    EAL: torch.Tensor
    EAL_fp16: torch.Tensor
    EAR_R_major: torch.Tensor
    EBL_R_major: torch.Tensor
    EAR_K_major: torch.Tensor
    EBL_K_major: torch.Tensor
    EBR: torch.Tensor
    EBR_fp16: torch.Tensor
    routing_data: torch.Tensor
    routing_hash: torch.Tensor
    offsets_hash: torch.Tensor
    routing_layout: MoERoutingLayout
    pow_target: torch.Tensor
    pow_key: torch.Tensor
    noise_rank: int


def prepare_moe_noising(A_q, A_scales, topk_ids, B_stacked, num_experts: int, job: MiningJob,
                        config: MiningConfig = MiningConfig()) -> MoENoiseContext:
    """Hashes, routing order, MoE commitment and noise for one pass
    (moe_gemm_operators.py:118-234)."""
    device = A_q.device
    num_tokens, hidden = A_q.shape
    if A_scales.shape != (num_tokens, 1):
        raise ValueError(f"A_scales must have shape ({num_tokens}, 1); got {tuple(A_scales.shape)}")
    rows_b = B_stacked.shape[0]
    r = config.noise_rank
    top_k = topk_ids.shape[1]
    key, target_tensor = _job_tensors(job, device)
    B_hash, b_ready = _tensor_root_async(B_stacked.contiguous().view(torch.uint8), key)
    A_hash = _tensor_root(A_q.contiguous().view(torch.uint8), key)
    salted = (num_tokens, rows_b // num_experts) if job.salted_seeds else None
    slots = num_tokens * top_k
    routing_data = torch.empty(slots, dtype=torch.int32, device=device)
    slot_indices = torch.empty(slots, dtype=torch.int32, device=device)
    routing_offsets = torch.empty(num_experts, dtype=torch.int32, device=device)
    scratch = torch.empty(get_build_routing_data_scratchpad_bytes(slots), dtype=torch.uint8,
                          device=device)
    build_routing_data(topk_ids.to(torch.int32).contiguous(), routing_data, slot_indices,
                       routing_offsets, scratch, num_experts)
    layout = MoERoutingLayout(routing_data, slot_indices, routing_offsets, routing_offsets.tolist(),
                              num_experts, top_k)
    routing_hash = _tensor_root(routing_data.view(torch.uint8).reshape(1, -1), key)
    offsets_hash = _tensor_root(routing_offsets.view(torch.uint8).reshape(1, -1), key)
    ch_A = torch.empty(32, device=device, dtype=torch.uint8)
    ch_B = torch.empty(32, device=device, dtype=torch.uint8)
    torch.cuda.current_stream(device).wait_event(b_ready)
    P.commitment_hash_from_merkle_roots(A_hash, B_hash, key, ch_A, ch_B, routing_root=routing_hash,
                                        offsets_hash=offsets_hash, salted_dims=salted)
    EAL, EAR_R, EBL_R, EAR_K, EBL_K, EBR, EAL_fp16, EBR_fp16 = generate_noise_factors(
        num_tokens, rows_b, hidden, r, ch_A, ch_B, device)
    return MoENoiseContext(ch_A, ch_B, EAL, EAL_fp16, EAR_R, EBL_R, EAR_K, EBL_K, EBR, EBR_fp16,
                           routing_data, routing_hash, offsets_hash, layout,
                           target_tensor, ch_A.view(torch.uint32), r)


def permute_a_side_to_expert_order(layout: MoERoutingLayout, A_q, A_scales, EAL, EAL_fp16):
    """moe_gemm_operators.py:237-256."""
    t = layout.token_indices
    return A_q[t], A_scales[t], EAL[t], EAL_fp16[t]


def pearl_moe_expert_gemm(A_q_e, B_e, A_scales_e, B_scales_e, EAL_e, EAL_fp16_e, EBR_e, EBR_fp16_e,
                          EAR_R_major, EBL_R_major, EAR_K_major, EBL_K_major, C_e,
                          host_signal_header_pinned, host_signal_sync, pow_target, pow_key,
                          tile_size_m: int, tile_size_n: int, tile_size_k: int, *, hits=None):
    """One expert's mined GEMM with in-kernel noising (moe_gemm_operators.py:259-329)."""
    m_e, k = A_q_e.shape
    n_e = B_e.shape[0]
    r = EAL_e.shape[1]
    device = A_q_e.device
    ApEA = torch.empty((m_e, k), dtype=torch.int8, device=device)
    AxEBL = torch.empty((m_e, r), dtype=torch.float16, device=device)
    BpEB = torch.empty((n_e, k), dtype=torch.int8, device=device)
    EARxBpEB = torch.empty((n_e, r), dtype=torch.float16, device=device)
    host_signal_sync.zero_()
    P.noisy_gemm(A=A_q_e, B=B_e, EAL=EAL_e, EAL_fp16=EAL_fp16_e, EBR=EBR_e, EBR_fp16=EBR_fp16_e,
                 EAR_R_major=EAR_R_major, EBL_R_major=EBL_R_major, EAR_K_major=EAR_K_major,
                 EBL_K_major=EBL_K_major, AxEBL_fp16=AxEBL, EARxBpEB_fp16=EARxBpEB, ApEA=ApEA,
                 BpEB=BpEB, A_scales=A_scales_e.squeeze(-1).contiguous(),
                 B_scales=B_scales_e.squeeze(-1).contiguous(), C=C_e,
                 host_signal_header_pinned=host_signal_header_pinned, host_signal_sync=host_signal_sync,
                 pow_target=pow_target, pow_key=pow_key, tile_size_m=tile_size_m,
                 tile_size_n=tile_size_n, tile_size_k=tile_size_k, run_noising_A=True,
                 run_noising_B=True, skip_reduction=False, skip_denoising=False, hits=hits)


@dataclass
class MoEGemm1Result:
    ctx: MoENoiseContext
    per_expert: dict = field(default_factory=dict)  # expert -> MinedGemm


def moe_gemm1(A_q, A_scales, topk_ids, w1, w1_scale, job: MiningJob,
              config: MiningConfig = MiningConfig(), *, out=None, hit_capacity: int = 0,
              grouped: bool = True):
    """Mined MoE GEMM1 (pearl_moe_experts.py:262-375): w1 (E, N, K) int7,
    w1_scale (E, N) or (E, N, 1) fp32, topk_ids (M, top_k).  Returns the
    per-slot output (M * top_k, N) bf16 in flat slot order and the per-expert
    mining products.  ``grouped`` runs every expert's mined GEMM in one
    grouped launch (pb2_noisy_gemm_grouped); without it, one mined GEMM per
    expert as in the reference's loop.  Both give the same results."""
    E, N, K = w1.shape
    num_tokens = A_q.shape[0]
    top_k = topk_ids.shape[1]
    B_stacked = w1.reshape(E * N, K)
    ctx = prepare_moe_noising(A_q, A_scales, topk_ids, B_stacked, E, job, config)
    layout = ctx.routing_layout
    A_e_all, S_e_all, EAL_e_all, EAL16_e_all = permute_a_side_to_expert_order(
        layout, A_q, A_scales, ctx.EAL, ctx.EAL_fp16)
    if out is None:
        out = torch.empty((num_tokens * top_k, N), dtype=torch.bfloat16, device=A_q.device)
    res = MoEGemm1Result(ctx)
    if grouped:
        # Every expert's mined GEMM in one noising and one persistent launch
        # (pb2_noisy_gemm_grouped); the same results as the loop below.
        dev = A_q.device
        r = ctx.noise_rank
        counts = [layout.expert_slice(e)[1] for e in range(E)]
        m_all = A_e_all.shape[0]
        syncs = torch.zeros(E, P.get_host_signal_sync_size(), dtype=torch.int8, device=dev)
        headers = [_pinned_header() if counts[e] else None for e in range(E)]
        hits = ([torch.zeros(hit_capacity, 12, dtype=torch.uint32, device=dev) if counts[e] else None
                 for e in range(E)] if hit_capacity else None)
        grouped_noisy_gemm(
            A_e_all, B_stacked, EAL_e_all, EAL16_e_all, ctx.EBR, ctx.EBR_fp16, ctx.EAR_R_major,
            ctx.EBL_R_major, ctx.EAR_K_major, ctx.EBL_K_major,
            torch.empty((m_all, r), dtype=torch.float16, device=dev),
            torch.empty((E * N, r), dtype=torch.float16, device=dev),
            torch.empty((m_all, K), dtype=torch.int8, device=dev),
            torch.empty((E * N, K), dtype=torch.int8, device=dev),
            S_e_all.reshape(-1).contiguous(), w1_scale.reshape(-1).contiguous(), out, counts, headers,
            [syncs[e] for e in range(E)], ctx.pow_target, ctx.pow_key, hits=hits,
            tile_size_m=config.tile_size_m, tile_size_n=config.tile_size_n, tile_size_k=config.tile_size_k,
            # out[slot_indices] = C (pearl_moe_experts.py:347), written by the epilogue itself
            c_row_index=layout.slot_indices)
        for e in range(E):
            if counts[e]:
                res.per_expert[e] = MinedGemm(headers[e], syncs[e], ctx.commitment_hash_A,
                                              ctx.commitment_hash_B, hits[e] if hits else None)
        return out, res
    by_slot = torch.empty_like(out)
    for e in range(E):
        start, count = layout.expert_slice(e)
        if count == 0:
            continue
        header = _pinned_header()
        sync = torch.zeros(P.get_host_signal_sync_size(), dtype=torch.int8, device=A_q.device)
        hits = (torch.zeros(hit_capacity, 12, dtype=torch.uint32, device=A_q.device)
                if hit_capacity else None)
        C_e = by_slot[start:start + count]
        pearl_moe_expert_gemm(
            A_e_all[start:start + count], B_stacked[e * N:(e + 1) * N], S_e_all[start:start + count],
            w1_scale[e], EAL_e_all[start:start + count], EAL16_e_all[start:start + count],
            ctx.EBR[e * N:(e + 1) * N], ctx.EBR_fp16[e * N:(e + 1) * N], ctx.EAR_R_major,
            ctx.EBL_R_major, ctx.EAR_K_major, ctx.EBL_K_major, C_e, header, sync, ctx.pow_target,
            ctx.pow_key, config.tile_size_m, config.tile_size_n, config.tile_size_k, hits=hits)
        # out[slot_indices] = C_e (pearl_moe_experts.py:347), at HBM speed
        scatter_rows(C_e, out, layout.slot_indices[start:start + count])
        res.per_expert[e] = MinedGemm(header, sync, ctx.commitment_hash_A, ctx.commitment_hash_B, hits)
    return out, res
