"""Mining across the GPUs of one box: one process per GPU, each mining its
own part of the nonce space, with no collective on the data path.

Every hash tile of every mined GEMM is independent and the noise is a
function of the GEMM's own commitment, so ranks never exchange operands: a
rank mines GEMMs whose seeds (job keys) no other rank uses -- in production
because every rank mines a block header of its own (job_key), in the
benchmark through synthetic per-rank keys (rank_job_key).  What crosses
ranks is only what the host needs afterwards -- the winning proofs, a few
hundred bytes each at ~1e-6 hits per hash tile -- gathered to rank 0 after
the work, and the elapsed time, reduced to the maximum over ranks.  The
reference miner has no multi-GPU path of its own (one independent worker
process per GPU, miner/vllm-miner/src/vllm_miner/register.py:26-30)."""

from __future__ import annotations

import hashlib

import torch

HIT_WORDS = 12  # {row_offset, col_offset, tile_m, tile_n, digest[8]}


def job_key(incomplete_header_bytes: bytes, mining_config_bytes: bytes) -> bytes:
    """The protocol's commitment key of a mining job: BLAKE3 of the
    incomplete block header followed by the serialized mining configuration
    (miner-base commitment_hash.py:36-37, CommitmentHasher.get_key).

    This is how a rank's real work is kept apart from every other rank's:
    each rank mines a header of its own (the coinbase extranonce, and so the
    header's merkle root, differs per rank), so its key, its noise seeds and
    every hash tile it hashes are its own, and a verifier derives the same
    key from the submitted header."""
    from blake3 import blake3

    return blake3(bytes(incomplete_header_bytes) + bytes(mining_config_bytes)).digest()


def rank_job_key(base_key: bytes, rank: int, step: int) -> bytes:
    """Benchmark stand-in for job_key: a 32-byte key distinct for every
    (rank, step), so no two ranks of a benchmark mine the same noise.

    These keys come from no block header, so a verifier could not rebuild
    them and proofs mined with them would not validate; they only give the
    benchmark independent work per rank without a gateway.  Real mining
    derives each rank's key with job_key from the header that rank mines."""
    h = hashlib.blake2b(digest_size=32, key=base_key[:64])
    h.update(rank.to_bytes(4, "little") + step.to_bytes(8, "little"))
    return h.digest()


def gather_hits(hits: torch.Tensor, count: int, group=None) -> torch.Tensor | None:
    """Gather every rank's hit list (``hits`` (capacity, 12) uint32 holding
    ``count`` valid rows) to rank 0.  Returns the concatenation on rank 0 and
    None elsewhere.  Fixed-size buffers: one all_gather of the counts and one
    of the padded lists (both tiny), the same steps on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = hits.device
    n = torch.tensor([min(int(count), hits.shape[0])], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    cap = max(int(c.item()) for c in counts)
    buf = torch.zeros((max(cap, 1), HIT_WORDS), dtype=torch.int64, device=dev)
    k = int(n.item())
    if k:
        buf[:k] = hits[:k].to(torch.int64)
    bufs = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf, group=group)
    if rank != 0:
        return None
    return torch.cat([b[: int(c.item())] for b, c in zip(bufs, counts)]).to(torch.uint32)


def max_over_ranks(ms: float, device=None, group=None) -> float:
    """The slowest rank's time (the box finishes when its last GPU does)."""
    import torch.distributed as dist

    t = torch.tensor([float(ms)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
