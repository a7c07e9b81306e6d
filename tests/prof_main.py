"""Small / full cases of the mined GEMM for ncu captures (profiles/): python tests/prof_main.py M K."""
import sys
sys.path.insert(0, __import__("os").path.dirname(__import__("os").path.dirname(__import__("os").path.abspath(__file__))))
import torch
from tests.gpu_problem import make_problem, gen_noise, run_noisy_gemm, signal_buffers
m = int(sys.argv[1]) if len(sys.argv) > 1 else 8192
k = int(sys.argv[2]) if len(sys.argv) > 2 else 2048
p = make_problem(m, m, k, 128, seed=1)
gen_noise(p)
header, sync = signal_buffers()
run_noisy_gemm(p, 0, header, sync)
for _ in range(4):
    run_noisy_gemm(p, 0, header, sync, run_noising_A=False, run_noising_B=False)
torch.cuda.synchronize()
print("prof_main done")
