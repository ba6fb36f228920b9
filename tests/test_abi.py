"""CPU tests of the C-ABI boundary: libmxs.so loads, exports every function
include/*.h declares, and rejects bad arguments before touching a device."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

import mxs_sampler

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names |= set(re.findall(r"^MXS_API\s+[\w\s\*]+?\b(mxs_\w+)\s*\(", open(h).read(), re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    import mxs_build
    mxs_build.build()
    return mxs_sampler.load()


def test_header_declares_the_python_binding_set():
    assert declared_symbols() == set(mxs_sampler.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", mxs_sampler.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = declared_symbols() - exported
    assert not missing, missing
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_version(lib):
    assert "sm_100a" in mxs_sampler.version()


def test_invalid_arguments_rejected_without_device(lib):
    P = ctypes.c_void_p
    # rows < 0, vocab <= 0, ld < vocab, null logits / u / next
    assert lib.mxs_sample_topk(None, -1, 10, 10, 1.0, 5, None, None, None, None, None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_topk(P(16), 1, 0, 10, 1.0, 5, P(16), P(16), None, None, None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_topk(P(16), 1, 10, 5, 1.0, 5, P(16), P(16), None, None, None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_topk(None, 1, 10, 10, 1.0, 5, P(16), P(16), None, None, None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_topk(P(16), 1, 10, 10, 1.0, 5, None, P(16), None, None, None) == mxs_sampler.MXS_ERR_INVALID
    # zero rows is a successful no-op
    assert lib.mxs_sample_topk(None, 0, 10, 10, 1.0, 5, None, None, None, None, None) == mxs_sampler.MXS_OK
    # shard list capacity below k
    assert lib.mxs_shard_candidates(P(16), 1, 100, 100, 0, 50, 10, P(16), P(16), P(16), None) == \
        mxs_sampler.MXS_ERR_INVALID



def test_sharded_entry_points_check_arguments_without_device(lib):
    P = ctypes.c_void_p
    n = ctypes.c_int64(-1)
    # rank outside [0, world), world <= 0
    assert lib.mxs_sample_rowsharded(P(16), 10, 2, 2, 100, 100, 1.0, 5, 1.0, 0.0, P(16), P(16), None, None, None,
                                     ctypes.byref(n), None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_rowsharded(P(16), 10, 0, 0, 100, 100, 1.0, 5, 1.0, 0.0, P(16), P(16), None, None, None,
                                     ctypes.byref(n), None) == mxs_sampler.MXS_ERR_INVALID
    # a rank whose range is empty (10 rows over 8 ranks: 2 per rank, rank 7 has none) succeeds with 0 rows
    assert lib.mxs_sample_rowsharded(None, 10, 7, 8, 100, 100, 1.0, 5, 1.0, 0.0, None, None, None, None, None,
                                     ctypes.byref(n), None) == mxs_sampler.MXS_OK
    assert n.value == 0
    # no communicator, ld < shard columns
    assert lib.mxs_sample_vocabsharded(P(16), 4, 100, 100, 1.0, 5, 1.0, 0.0, P(16), P(16), None, None, None, None,
                                       None) == mxs_sampler.MXS_ERR_INVALID
    assert lib.mxs_sample_vocabsharded(P(16), 4, 100, 50, 1.0, 5, 1.0, 0.0, P(16), P(16), None, None, None, P(16),
                                       None) == mxs_sampler.MXS_ERR_INVALID


def test_no_cpu_fallback_without_gpu(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    P = ctypes.c_void_p
    rc = lib.mxs_sample_topk(P(256), 1, 10, 10, 1.0, 5, P(256), P(256), None, None, None)
    assert rc in (mxs_sampler.MXS_ERR_NO_DEVICE, mxs_sampler.MXS_ERR_CUDA)
