"""Small / full cases for ncu captures (the summaries under profiles/).

    python tests/prof_main.py M K          the mined GEMM, M = N, depth K
    python tests/prof_main.py noise M K    the fused noising step (noise_AB), M = N
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

import pearl_b200 as pg  # noqa: E402
from tests.gpu_problem import gen_noise, make_problem, run_noisy_gemm, signal_buffers  # noqa: E402

args = sys.argv[1:]
noise_only = bool(args) and args[0] == "noise"
if noise_only:
    args = args[1:]
m = int(args[0]) if len(args) > 0 else 8192
k = int(args[1]) if len(args) > 1 else 2048
p = make_problem(m, m, k, 128, seed=1)
gen_noise(p)
if noise_only:
    factors = {n: v for n, v in p.noise.items() if n not in ("EAL", "EBR")}
    for _ in range(4):
        pg.noise_AB(p.A, p.noise["EAL"], p.out["AxEBL_fp16"], p.out["ApEA"], p.B, p.noise["EBR"],
                    p.out["EARxBpEB_fp16"], p.out["BpEB"], **factors)
else:
    header, sync = signal_buffers()
    run_noisy_gemm(p, 0, header, sync)
    for _ in range(4):
        run_noisy_gemm(p, 0, header, sync, run_noising_A=False, run_noising_B=False)
torch.cuda.synchronize()
print("prof_main done")
