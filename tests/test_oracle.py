"""Pins the CPU oracle against the golden fixtures made from the reference's
own Python code (tests/golden/make_golden.py) and against the Python blake3
package."""

import json
import os

import numpy as np
import pytest

from oracle import oracle as O


def test_blake3_kat(golden_dir):
    kat = json.load(open(os.path.join(golden_dir, "blake3_kat.json")))
    key = bytes((7 * i + 3) % 256 for i in range(32))
    for case in kat["cases"]:
        data = bytes(i % 251 for i in range(case["len"]))
        assert O.blake3(data).hex() == case["hash"], case["len"]
        assert O.blake3(data, key).hex() == case["keyed"], case["len"]


def test_blake3_matches_python_package_random():
    blake3 = pytest.importorskip("blake3").blake3
    rng = np.random.default_rng(5)
    for n in [7, 64, 65, 1024, 1025, 4097, 9000]:
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        k = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
        assert O.blake3(d, k) == blake3(d, key=k).digest()


@pytest.mark.parametrize("name", ["noise_r128.npz", "noise_r64.npz"])
def test_noise_matches_reference_generator(golden_dir, name):
    z = np.load(os.path.join(golden_dir, name))
    r = int(z["r"])
    ka, kb = z["key_a"].tobytes(), z["key_b"].tobytes()
    m, n, k = z["EAL"].shape[0], z["EBR"].shape[0], z["EAR_R_major"].shape[0]
    assert (O.noise_dense(ka, "A", m, r) == z["EAL"]).all()
    assert (O.noise_dense(kb, "B", n, r) == z["EBR"]).all()
    assert (O.pairs_to_r_major(O.noise_pairs(ka, "A", k, r), r) == z["EAR_R_major"]).all()
    assert (O.pairs_to_r_major(O.noise_pairs(kb, "B", k, r), r) == z["EBL_R_major"]).all()


def test_noise_value_ranges():
    key = bytes(range(32))
    e = O.noise_dense(key, "A", 512, 128)
    assert e.min() >= -32 and e.max() <= 31
    p = O.noise_pairs(key, "B", 4096, 128)
    assert (p[:, 0] != p[:, 1]).all() and p.max() < 128


def test_commitment_pinned_vectors(golden_dir):
    g = json.load(open(os.path.join(golden_dir, "commitment.json")))
    jk, ha, hb = (bytes.fromhex(g[x]) for x in ("job_key", "hash_a", "hash_b"))
    for case in g["cases"]:
        dims = tuple(case["salted_dims"]) if case["salted_dims"] else None
        rr = bytes.fromhex(case["routing_root"]) if "routing_root" in case else None
        b, a = O.commitment(jk, ha, hb, salted_dims=dims, routing_root=rr, offsets=case.get("offsets"))
        assert b.hex() == case["b_seed"] and a.hex() == case["a_seed"]


@pytest.mark.parametrize("name", ["jackpot_m128_n256_k1024_r128.npz", "jackpot_m64_n256_k1152_r64.npz"])
def test_jackpot_matches_golden(golden_dir, name):
    z = np.load(os.path.join(golden_dir, name))
    r = int(z["r"])
    ka, kb = z["key_a"].tobytes(), z["key_b"].tobytes()
    prob = O.noisy_problem(z["A"], z["B"], ka, kb, r)
    if "ApEA" in z:
        assert (prob.ApEA == z["ApEA"]).all() and (prob.BpEB == z["BpEB"]).all()
    assert (prob.AxEBL == z["AxEBL"]).all() and (prob.EARxBpEB == z["EARxBpEB"]).all()
    target = sum(int(w) << (32 * i) for i, w in enumerate(z["target"]))
    res = O.mine_tiles(prob.ApEA, prob.BpEB, r, ka, target)
    assert (res.transcripts == z["transcripts"]).all()
    assert (res.digests == z["digests"]).all()
    assert (res.hits == z["hits"]).all()
    assert res.hits.any() and not res.hits.all()


def test_jackpot_tile_linearity_of_split():
    """The transcript of a tile equals the XOR of transcripts over any split
    of its elements (the fold and rotate-xor are GF(2)-linear); the B200
    kernel relies on this to fold rows r and r+8 separately."""
    rng = np.random.default_rng(9)
    k, r = 512, 128
    ap = rng.integers(-127, 127, (32, k), dtype=np.int8)
    bp = rng.integers(-127, 127, (300, k), dtype=np.int8)
    cols = [3 + 8 * j + d for j in range(32) for d in (0, 1)]
    full = O.jackpot_tile(ap, bp, k, r, [1, 9], cols)
    a = O.jackpot_tile(ap, bp, k, r, [1], cols)
    b = O.jackpot_tile(ap, bp, k, r, [9], cols)
    assert (full == (a ^ b)).all()


def test_target_extremes():
    rng = np.random.default_rng(2)
    ap = rng.integers(-64, 64, (16, 256), dtype=np.int8)
    bp = rng.integers(-64, 64, (256, 256), dtype=np.int8)
    key = bytes(32)
    assert O.mine_tiles(ap, bp, 128, key, 2**256 - 1).hits.all()
    assert not O.mine_tiles(ap, bp, 128, key, 0).hits.any()
