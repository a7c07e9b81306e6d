"""Generate the golden fixtures in this directory.

Run from the repository root in a container that has the reference checkout:

    PEARL_REFERENCE=/path/to/pearl python tests/golden/make_golden.py

The fixtures are produced WITHOUT the C oracle, from the reference's own
Python code where it is importable and from independent numpy code where it is
not, so that the oracle can be checked against them:

* ``blake3_kat.json``   -- digests from the PyPI ``blake3`` package (the
  reference's Python BLAKE3, pearl-gemm/pyproject.toml:9).
* ``noise_*.npz``       -- noise factors from the reference's
  ``miner_base.noise_generation.NoiseGenerator``.
* ``commitment.json``   -- the consensus-pinned seed-chain vectors of
  zk-pow/src/api/seed.rs (``commitment_hash_pinned_vectors`` and
  ``commitment_hash_pinned_vector_salted_moe``), recomputed with the PyPI
  ``blake3`` package following api/proof_utils.rs:361-372.
* ``jackpot_*.npz``     -- jackpot transcripts / digests computed by a chunked
  full-matrix GEMM in numpy (a different loop structure from the C oracle's
  per-tile loops), folded with the reference's
  ``miner_base.inner_hash.xor_reduction`` and the rotate-xor of
  zk-pow/src/ffi/mine.rs:95-106.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
from blake3 import blake3

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("PEARL_REFERENCE")
if not REF:
    sys.exit("set PEARL_REFERENCE to the reference checkout (see the module docstring)")
sys.path.insert(0, os.path.join(REF, "miner/miner-base/src"))
sys.path.insert(0, os.path.join(REF, "miner/miner-utils/src"))

from miner_base.inner_hash import xor_reduction  # noqa: E402
from miner_base.noise_generation import NoiseGenerator  # noqa: E402


def kat_blake3():
    cases = []
    for n in [0, 1, 31, 32, 63, 64, 65, 127, 128, 1000, 1023, 1024, 1025, 2048, 2049, 3072, 4096,
              5000, 8192, 16384, 31744, 65536]:
        data = bytes(i % 251 for i in range(n))
        key = bytes((7 * i + 3) % 256 for i in range(32))
        cases.append({"len": n, "hash": blake3(data).hexdigest(),
                      "keyed": blake3(data, key=key).hexdigest()})
    with open(os.path.join(HERE, "blake3_kat.json"), "w") as f:
        json.dump({"data": "bytes(i % 251)", "key": "bytes((7*i+3) % 256)", "cases": cases}, f, indent=1)


def noise_fixture(name, m, n, k, r, seed):
    rng = np.random.default_rng(seed)
    key_a = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
    key_b = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
    g = NoiseGenerator(noise_rank=r)
    AL, AR, BL, BR = g.generate_noise_metrices(key_a, key_b, m, k, n)
    np.savez_compressed(
        os.path.join(HERE, name),
        key_a=np.frombuffer(key_a, np.uint8), key_b=np.frombuffer(key_b, np.uint8),
        EAL=AL.numpy(), EAR_R_major=AR.numpy().T.copy(), EBL_R_major=BL.numpy(),
        EBR=BR.numpy().T.copy(), r=np.int64(r))


def commitment_fixture():
    def b3(data, key=None):
        return blake3(data, key=key).digest() if key is not None else blake3(data).digest()

    salt_a = b3(b"pearl/cert-v3/noise-seed/A")
    salt_b = b3(b"pearl/cert-v3/noise-seed/B")

    def bind(root, dim, salt):
        return b3(root + dim.to_bytes(4, "little") + bytes(28), salt)

    job_key = bytes([0x11] * 32)
    ha, hb = bytes([0xAA] * 32), bytes([0xBB] * 32)
    out = []
    for salted in (False, True):
        a, b = (bind(ha, 192, salt_a), bind(hb, 320, salt_b)) if salted else (ha, hb)
        bs = b3(job_key + b)
        as_ = b3(bs + a)
        out.append({"salted_dims": [192, 320] if salted else None, "b_seed": bs.hex(), "a_seed": as_.hex()})
    # MoE routing fold (proof_utils.rs:34-45) on the salted chain.
    a = bind(ha, 192, salt_a)
    offs = b"".join(o.to_bytes(4, "little") for o in [3, 5, 9, 12])
    h_off = b3(offs + bytes(1024 - len(offs)), job_key)
    h_route = b3(bytes([0xCC] * 32) + h_off)
    act = b3(a + h_route)
    bs = b3(job_key + bind(hb, 320, salt_b))
    out.append({"salted_dims": [192, 320], "routing_root": "cc" * 32, "offsets": [3, 5, 9, 12],
                "b_seed": bs.hex(), "a_seed": b3(bs + act).hex()})
    # The literal vectors of zk-pow/src/api/seed.rs (consensus pins).
    pinned = {
        "legacy": ("add6f7ea5feebf89c8a77e2ebfa0d82442e7dbb0046dbd48971861d12fcb0177",
                   "483b07b6f73105030b9482255f37723f3fed69ae916724ee8291848b8c28794b"),
        "salted": ("60ed9b73c5a9599b200b6cd563e7f0d5d9a67d2402d85fd4ef966c580080d0e5",
                   "301784168005ec833ab0aa60006f7fe7faaa95307d8c1fc6819b2ffdd717eccf"),
        "salted_moe": ("60ed9b73c5a9599b200b6cd563e7f0d5d9a67d2402d85fd4ef966c580080d0e5",
                       "268a2eb78b3b2d2fead262221b24c6346d0a6d201890a467751f623b7eacd5c2"),
    }
    for case, key in zip(out, ["legacy", "salted", "salted_moe"]):
        assert (case["b_seed"], case["a_seed"]) == pinned[key], key
    with open(os.path.join(HERE, "commitment.json"), "w") as f:
        json.dump({"job_key": job_key.hex(), "hash_a": ha.hex(), "hash_b": hb.hex(), "cases": out}, f, indent=1)


def jackpot_fixture(name, m, n, k, r, seed, target_frac, store_operands=True):
    """Full noisy problem through the reference NoiseGenerator + numpy."""
    rng = np.random.default_rng(seed)
    A = rng.integers(-64, 64, (m, k), dtype=np.int8)
    B = rng.integers(-64, 64, (n, k), dtype=np.int8)
    key_a = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
    key_b = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
    g = NoiseGenerator(noise_rank=r)
    AL, AR, BL, BR = g.generate_noise_metrices(key_a, key_b, m, k, n)
    EAL, EAR = AL.numpy().astype(np.int32), AR.numpy().astype(np.int32)  # (m,r), (r,k)
    EBL, EBR = BL.numpy().astype(np.int32), BR.numpy().T.astype(np.int32)  # (k,r), (n,r)
    ApEA = (A.astype(np.int32) + EAL @ EAR).astype(np.int8)
    BpEB = (B.astype(np.int32) + EBR @ EBL.T).astype(np.int8)
    AxEBL = A.astype(np.int32) @ EBL
    EARxBpEB = BpEB.astype(np.int32) @ EAR.T

    # chunked GEMM snapshots S_c, folded per protocol hash tile
    tiles_r, tiles_c = m // 2, n // 64
    T = np.zeros((tiles_r, tiles_c, 16), np.uint32)
    S = np.zeros((m, n), np.int64)
    rows = np.array([16 * (t // 8) + t % 8 for t in range(tiles_r)])
    cols = np.array([256 * (t // 4) + 2 * (t % 4) for t in range(tiles_c)])
    for c, ll in enumerate(range(r, k + 1, r)):
        S += ApEA[:, ll - r:ll].astype(np.int64) @ BpEB[:, ll - r:ll].astype(np.int64).T
        S32 = S.astype(np.int32)
        idx = c % 16
        for i, ro in enumerate(rows):
            for j, co in enumerate(cols):
                tile = S32[np.ix_([ro, ro + 8], [co + 8 * q + d for q in range(32) for d in (0, 1)])]
                x = np.uint32(xor_reduction(torch.from_numpy(np.ascontiguousarray(tile))))
                t = T[i, j, idx]
                T[i, j, idx] = np.uint32(((int(t) << 13) | (int(t) >> 19)) & 0xFFFFFFFF) ^ x
    T = T.reshape(-1, 16)
    digests = np.zeros((T.shape[0], 8), np.uint32)
    for t in range(T.shape[0]):
        digests[t] = np.frombuffer(blake3(T[t].astype("<u4").tobytes(), key=key_a).digest(), "<u4")
    # target: the digest value at the target_frac quantile so a few tiles hit
    as_int = [sum(int(w) << (32 * i) for i, w in enumerate(d)) for d in digests]
    target = sorted(as_int)[max(0, int(len(as_int) * target_frac) - 1)]
    hits = np.array([v <= target for v in as_int])
    extra = {}
    if store_operands:
        extra = dict(ApEA=ApEA, BpEB=BpEB, C=(A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32))
    np.savez_compressed(
        os.path.join(HERE, name), A=A, B=B, key_a=np.frombuffer(key_a, np.uint8),
        key_b=np.frombuffer(key_b, np.uint8), r=np.int64(r),
        AxEBL=AxEBL.astype(np.int32), EARxBpEB=EARxBpEB.astype(np.int32),
        transcripts=T, digests=digests, hits=hits,
        target=np.array([(target >> (32 * i)) & 0xFFFFFFFF for i in range(8)], np.uint32), **extra)


if __name__ == "__main__":
    kat_blake3()
    noise_fixture("noise_r128.npz", 256, 384, 512, 128, seed=1)
    noise_fixture("noise_r64.npz", 192, 256, 320, 64, seed=2)
    commitment_fixture()
    jackpot_fixture("jackpot_m128_n256_k1024_r128.npz", 128, 256, 1024, 128, seed=3, target_frac=0.05)
    jackpot_fixture("jackpot_m64_n256_k1152_r64.npz", 64, 256, 1152, 64, seed=4, target_frac=0.05,
                    store_operands=False)
    print("golden fixtures written to", HERE)
