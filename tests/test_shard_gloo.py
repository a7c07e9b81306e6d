"""The multi-GPU host logic (pearl_b200.shard) on world-size-2 gloo process
groups on CPU: disjoint nonce space per rank, winning proofs gathered to
rank 0, max-over-ranks timing, and a rank that dies before the gather makes
the surviving rank's collective fail within the group's timeout instead of
hanging."""

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pearl_b200 import shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _gather_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        keys = {shard.rank_job_key(b"k" * 32, rank, s) for s in range(64)}
        # A rank's hits as the kernel writes them: rank r finds r + 2 proofs.
        cnt = rank + 2
        hits = torch.zeros(16, shard.HIT_WORDS, dtype=torch.uint32)
        for i in range(cnt):
            hits[i, 0], hits[i, 1], hits[i, 4] = 16 * i, 2 * rank, 1000 * rank + i
        got = shard.gather_hits(hits, cnt)
        ms = shard.max_over_ranks(10.0 + rank)
        q.put((rank, sorted(keys), None if got is None else got.tolist(), ms))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc(), None))


def test_gather_hits_and_disjoint_nonce_space():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, keys, got, ms = q.get(timeout=120)
        assert keys != "error", got
        out[rank] = (keys, got, ms)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert not set(out[0][0]) & set(out[1][0])  # no shared job keys
    gathered = out[0][1]
    assert out[1][1] is None
    assert len(gathered) == 2 + 3
    assert sorted((h[1], h[4]) for h in gathered) == sorted(
        [(0, i) for i in range(2)] + [(2, 1000 + i) for i in range(3)])
    assert out[0][2] == out[1][2] == 11.0


def _dying_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message: os._exit skips the queue's feeder thread
            os._exit(0)  # leaves between steps, before the gather
        try:
            shard.gather_hits(torch.zeros(4, shard.HIT_WORDS, dtype=torch.uint32), 0)
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001
            q.put((rank, f"error: {type(e).__name__}"))
    except Exception:  # noqa: BLE001
        q.put((rank, "setup: " + traceback.format_exc()))


def test_dead_rank_fails_the_gather_instead_of_hanging():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]


def test_job_key_is_the_protocol_key():
    """A rank's real key is BLAKE3(incomplete header || mining config)
    (commitment_hash.py:36-37); ranks mining different headers (their own
    extranonce) get different keys."""
    from oracle import oracle as O

    header = bytes(range(80))
    config = bytes([3, 0, 0, 0, 128, 0, 0, 0])
    assert shard.job_key(header, config) == O.blake3(header + config)
    other = header[:-4] + (1).to_bytes(4, "little")
    assert shard.job_key(other, config) != shard.job_key(header, config)
