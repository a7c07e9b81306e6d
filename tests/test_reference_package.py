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
