"""Import hook for running the reference's ``pearl_gemm`` Python package on
the B200 kernels: with this directory on sys.path, ``import pearl_gemm_cuda``
(the compiled extension the reference package imports,
miner/pearl-gemm/src/pearl_gemm/pearl_gemm_interface.py:1) yields
pearl_b200.pearl_gemm_cuda, which offers that extension's surface.

The reference's extension defines the torch.ops.pearl_gemm schemas and its
Python files register their fake implementations, so pearl_b200's own fakes
are withdrawn here, before those files are imported."""

import sys

import pearl_b200.ops as _ops
import pearl_b200.pearl_gemm_cuda as _impl

_ops.release_fake_impls()
sys.modules[__name__] = _impl
