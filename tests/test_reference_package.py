"""The reference's own, unmodified Python package ``pearl_gemm`` running on
this library through ``pearl_b200.pearl_gemm_cuda`` (the stand-in for its
compiled extension).  CPU tests; they need a reference checkout and are
skipped without one (``PEARL_REFERENCE``, or a ``reference`` directory next
to this repository).

Checked in a fresh interpreter (torch op registrations are per process):

* ``import pearl_gemm`` succeeds: ``pearl_gemm_cuda`` resolves to the shim,
  the reference's ``register_fake`` calls for every ``pearl_gemm::*`` op
  succeed (the shim withdraws pearl_b200's own fakes), and the package's
  re-exported names come from the shim.
* Every reference wrapper that calls ``pearl_gemm_cuda.<op>`` positionally
  lands in ``pearl_b200.pearl_gemm_interface.<op>`` with each argument in its
  named place: the wrappers are called with a distinct marker per argument
  and the interface functions are replaced by recorders (nothing is
  launched).  The GPU tests then cover the interface functions themselves,
  and tests/test_gpu_kernels.py::test_pearl_gemm_cuda_positional_calls runs
  the shim's positional calls on the device."""

import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_src():
    base = os.environ.get("PEARL_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    src = os.path.join(base, "miner", "pearl-gemm", "src")
    return src if os.path.isfile(os.path.join(src, "pearl_gemm", "pearl_gemm_interface.py")) else None


def _run(code: str) -> str:
    src = _reference_src()
    if src is None:
        pytest.skip("no reference checkout (set PEARL_REFERENCE)")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "pearl_b200", "compat"), ROOT, src])
    res = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], env=env, capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout


def test_reference_package_imports_on_the_shim():
    out = _run("""
        import torch
        import pearl_gemm, pearl_gemm_cuda, pearl_gemm.moe
        import pearl_b200.pearl_gemm_cuda as shim
        from torch._library.simple_registry import singleton
        assert pearl_gemm_cuda is shim
        assert pearl_gemm.kEALScaleFactorDenoise == -1 and pearl_gemm.kEBRScaleFactorDenoise == -4
        assert pearl_gemm.get_host_signal_header_size() == 640 and pearl_gemm.get_host_signal_sync_size() == 16
        assert pearl_gemm.HostSignalStatus.kSignalTriggered == 1
        assert pearl_gemm.get_required_scratchpad_bytes(8192 * 8192) == 512 * 32
        for op in ("noisy_gemm", "gemm", "noise_A", "noise_B", "noise_gen", "denoise_converter",
                   "tensor_hash", "commitment_hash_from_merkle_roots", "build_routing_data"):
            getattr(torch.ops.pearl_gemm, op)
            fake = singleton.find("pearl_gemm::" + op).fake_impl.kernel
            assert fake is not None and fake.source.find("pearl_gemm") >= 0, (op, fake.source)
            assert "pearl_b200" not in fake.source, (op, fake.source)
        print("ok")
    """)
    assert out.strip().endswith("ok")


def test_reference_wrappers_reach_the_interface_with_every_argument_in_place():
    out = _run("""
        import inspect
        import pearl_gemm, pearl_gemm.moe
        import pearl_b200.moe as M
        import pearl_b200.pearl_gemm_interface as I

        names = ("noisy_gemm", "gemm", "noise_A", "noise_B", "noise_gen", "denoise_converter",
                 "tensor_hash", "commitment_hash_from_merkle_roots")
        real = {n: getattr(I, n) for n in names}
        real["build_routing_data"] = M.build_routing_data
        calls = []

        def recorder(name):
            def rec(*args, **kwargs):
                calls.append((name, args, kwargs))
            return rec

        for n in names:
            setattr(I, n, recorder(n))
        M.build_routing_data = recorder("build_routing_data")

        def check(ref_fn, name):
            # One distinct marker per argument of the reference wrapper.
            markers = {}
            for p in inspect.signature(ref_fn).parameters.values():
                markers[p.name] = (1234, 5678) if p.name == "salted_dims" else "<" + p.name + ">"
            calls.clear()
            ref_fn(**markers)
            assert len(calls) == 1 and calls[0][0] == name, (name, calls)
            _, args, kwargs = calls[0]
            got = inspect.signature(real[name]).bind(*args, **kwargs).arguments
            for pname, marker in markers.items():
                assert got.get(pname) == marker, (name, pname, got.get(pname), marker)

        for n in names:
            check(getattr(pearl_gemm, n), n)
        check(pearl_gemm.moe.build_routing_data, "build_routing_data")
        print("ok", len(real))
    """)
    assert out.strip() == "ok 9"


# The reference's vLLM plugin package (miner/vllm-miner) on this library.  Its
# imports reach two modules that are not Python in the reference: the Rust
# extension pearl_mining and the third-party bitcoinutils (gateway address
# helpers).  Only those are stubbed, inside the child interpreter.
_STUB_HOOK = """
import importlib.abc, importlib.machinery, sys, types
class _Stub(types.ModuleType):
    def __getattr__(self, n):
        if n.startswith("__"):
            raise AttributeError(n)
        if n.isupper():
            return 64  # size constants used at import time
        return type(n, (), {"__init__": lambda self, *a, **k: None})
class _Finder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def find_spec(self, name, path, target=None):
        if name.split(".")[0] in ("pearl_mining", "bitcoinutils"):
            return importlib.machinery.ModuleSpec(name, self, is_package=True)
        return None
    def create_module(self, spec):
        return _Stub(spec.name)
    def exec_module(self, m):
        m.__path__ = []
sys.meta_path.insert(0, _Finder())
"""


def _run_miner(code: str) -> str:
    src = _reference_src()
    if src is None:
        pytest.skip("no reference checkout (set PEARL_REFERENCE)")
    miner = os.path.dirname(os.path.dirname(src))
    paths = [os.path.join(ROOT, "pearl_b200", "compat"), ROOT, src] + [
        os.path.join(miner, p, "src") for p in ("miner-base", "miner-utils", "pearl-gateway", "vllm-miner")]
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(paths)
    res = subprocess.run([sys.executable, "-c", _STUB_HOOK + textwrap.dedent(code)], env=env, capture_output=True,
                         text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout


def test_reference_vllm_plugin_registers_on_the_shim():
    """vllm_miner.register.register_pearl_miner_layer (register.py:32-50)
    registers the reference's "pearl" quantization config with vLLM while
    pearl_gemm_cuda is this library's shim."""
    out = _run_miner("""
        import pearl_gemm_cuda
        import pearl_b200.pearl_gemm_cuda as shim
        from vllm_miner.register import register_pearl_miner_layer
        register_pearl_miner_layer()
        from vllm.model_executor.layers.quantization import QUANTIZATION_METHODS, get_quantization_config
        from vllm_miner.vllm_config import PearlConfig
        assert pearl_gemm_cuda is shim
        assert "pearl" in QUANTIZATION_METHODS and get_quantization_config("pearl") is PearlConfig
        print("ok")
    """)
    assert out.strip().endswith("ok")


def test_reference_vanilla_operator_reaches_the_interface():
    """vllm_miner.gemm_operators.pearl_gemm_vanilla (gemm_operators.py:28-65),
    the non-mining branch of PearlScheme.apply_weights, calls pearl_gemm.gemm
    with its operands, scales and the output it allocates; on the shim that
    call lands in pearl_b200.pearl_gemm_interface.gemm (replaced by a
    recorder: nothing is launched on the CPU)."""
    out = _run_miner("""
        import torch
        import pearl_b200.pearl_gemm_interface as I
        calls = []
        I.gemm = lambda *a, **k: calls.append((a, k))
        import vllm_miner.gemm_operators as G
        A = torch.zeros(4, 64, dtype=torch.int8)
        B = torch.zeros(8, 64, dtype=torch.int8)
        sa, sb = torch.ones(4), torch.ones(8)
        C = G.pearl_gemm_vanilla(A, B, sa, sb, torch.bfloat16)
        assert len(calls) == 1
        args, kw = calls[0]
        assert args[0] is A and args[1] is B and args[2] is sa and args[3] is sb and args[4] is C
        assert C.shape == (4, 8) and C.dtype == torch.bfloat16
        assert (kw["tile_size_m"], kw["tile_size_n"], kw["tile_size_k"]) == (128, 256, 128)
        print("ok")
    """)
    assert out.strip().endswith("ok")
