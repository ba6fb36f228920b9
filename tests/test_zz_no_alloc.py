"""GPU tests of mxs_sample_topk_noalloc, the entry point for hosts that cannot
let this library allocate device memory: a serving engine or plugin host whose
own memory pool owns the whole GPU and treats any cudaMalloc behind its back as
an error, or a per-token path where allocation is forbidden. The call takes its
scratch from a fixed array compiled into the library and must give the results
the reference's sampling block gives (checked against the CPU oracle) and the
same results as the regular entry point.

Kept in a file of its own that pytest collects last. It passes alone in a fresh
process and after the other tests; the array keeps the previous call's
contents, so calls are checked twice in a row and with alternating shapes and
kernel paths."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle_lib
import workloads

pytestmark = pytest.mark.gpu
RTOL = 1e-6  # the parity tolerance of the other GPU tests for probabilities
LIMIT = 48 << 20  # MXS_NOALLOC_SCRATCH_BYTES (include/mxs_sampler.h)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call_noalloc(lib, lg, T, k, u, nxt, idx, prob, flg, top_p=1.0, min_p=0.0):
    rows, vocab = lg.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.mxs_sample_topk_noalloc(_p(lg), rows, vocab, lg.stride(0), T, k, top_p, min_p, _p(u), _p(nxt),
                                       _p(idx), _p(prob), _p(flg), stream)


def _noalloc_outputs(mxs, x, T, k, u, top_p=1.0, min_p=0.0):
    rows, vocab = x.shape
    kk = mxs.k_use(k, vocab)
    lg = torch.from_numpy(x).cuda()
    uu = torch.from_numpy(u).cuda()
    nxt = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    idx = torch.full((rows, kk), -7, dtype=torch.int32, device="cuda")
    prob = torch.full((rows, kk), -7.0, dtype=torch.float64, device="cuda")
    flg = torch.zeros(rows, dtype=torch.int32, device="cuda")
    rc = _call_noalloc(mxs.load(), lg, T, k, uu, nxt, idx, prob, flg, top_p, min_p)
    assert rc == mxs.MXS_OK, rc
    torch.cuda.synchronize()
    return nxt.cpu().numpy(), idx.cpu().numpy(), prob.cpu().numpy(), flg.cpu().numpy()


def _check_oracle(x, T, k, u, got, what, top_p=1.0, min_p=0.0):
    n0, i0, p0 = oracle_lib.oracle_sample(x, T, k, u, top_p, min_p)
    np.testing.assert_array_equal(got[0], n0, err_msg=f"{what}: next")
    np.testing.assert_array_equal(got[1], i0, err_msg=f"{what}: top-k order")
    np.testing.assert_allclose(got[2], p0, rtol=RTOL, atol=0, err_msg=f"{what}: probabilities")


@pytest.mark.parametrize("rows,k,T", [(64, 40, 0.7), (4, 8, 0.8), (300, 50, 0.8), (16, 128, 1.0)])
def test_noalloc_matches_oracle_and_regular_entry_point_twice(mxs, rows, k, T):
    x = workloads.spiked(200 + rows, rows, workloads.V_QWEN)
    if rows >= 4:
        x[1, 500:560] = 40.0  # a tie row: the exact replay path uses the scratch too
    u = oracle_lib.uniforms(7, rows)
    ref_next, ref_idx, ref_prob, ref_flg = mxs.sample(torch.from_numpy(x).cuda(), T, k, torch.from_numpy(u).cuda(),
                                                      return_flags=True)
    for call in range(2):  # two calls in a row on the shared array
        got = _noalloc_outputs(mxs, x, T, k, u)
        _check_oracle(x, T, k, u, got, f"call {call}")
        np.testing.assert_array_equal(got[0], ref_next.cpu().numpy())
        np.testing.assert_array_equal(got[1], ref_idx.cpu().numpy())
        np.testing.assert_allclose(got[2], ref_prob.cpu().numpy(), rtol=RTOL, atol=0)
        np.testing.assert_array_equal(got[3], ref_flg.cpu().numpy())


def test_noalloc_alternating_shapes_and_paths(mxs):
    """Stale state from a call with another layout must not leak into the next:
    a CTA-kernel call (k > 128), then two-kernel calls of other shapes, each
    with a tie row, then the first shape again."""
    cases = [(64, 200, 0.8), (300, 50, 0.8), (4, 8, 1.0), (64, 200, 0.8), (33, 2, 0.5)]
    for n, (rows, k, T) in enumerate(cases):
        x = workloads.normal(300 + n, rows, workloads.V_QWEN, 2.0)
        x[min(2, rows - 1), 1000:1300] = 30.0  # a tie block above every other logit
        u = oracle_lib.uniforms(300 + n, rows)
        got = _noalloc_outputs(mxs, x, T, k, u, top_p=0.9 if n == 2 else 1.0)
        _check_oracle(x, T, k, u, got, f"case {n} rows={rows} k={k}", top_p=0.9 if n == 2 else 1.0)


def test_noalloc_limit_over_the_throughput_batches(mxs):
    """The throughput configuration's batch sizes at V = 151,936, k = 50: a
    shape is accepted exactly when its workspace fits the fixed array; the
    accepted ones match the regular entry point."""
    lib = mxs.load()
    V = workloads.V_QWEN
    for rows in (1, 16, 256, 1024, 4096):
        need = mxs.workspace_bytes(rows, V, 50)
        gen = torch.Generator(device="cuda").manual_seed(rows)
        lg = torch.randn((rows, V), generator=gen, device="cuda") * 2.0
        u = torch.rand(rows, generator=gen, device="cuda", dtype=torch.float64)
        nxt = torch.empty(rows, dtype=torch.int32, device="cuda")
        rc = _call_noalloc(lib, lg, 0.8, 50, u, nxt, None, None, None)
        if need > LIMIT:
            assert rc == mxs.MXS_ERR_WORKSPACE, (rows, need, rc)
            continue
        assert rc == mxs.MXS_OK, (rows, need, rc)
        ref, _, _ = mxs.sample(lg, 0.8, 50, u, return_topk=False)
        torch.cuda.synchronize()
        assert torch.equal(nxt, ref), rows
        del lg
    # the headline batch fits on the two-kernel path
    assert mxs.workspace_bytes(4096, V, 50) <= LIMIT
    # a shape whose scratch exceeds the fixed array is refused with a clear code
    big = torch.zeros((4096, 40000), dtype=torch.float32, device="cuda")
    ub = torch.zeros(4096, dtype=torch.float64, device="cuda")
    nb = torch.empty(4096, dtype=torch.int32, device="cuda")
    assert mxs.workspace_bytes(4096, 40000, 40000) > LIMIT
    assert _call_noalloc(lib, big, 1.0, 40000, ub, nb, None, None, None) == mxs.MXS_ERR_WORKSPACE


def test_noalloc_timeout_reaches_get_status(mxs):
    """A timed-out row of an allocation-free call shows in mxs_get_status."""
    rows = 512
    x = workloads.normal(21, rows, workloads.V_QWEN, 2.0)
    u = oracle_lib.uniforms(21, rows)
    mxs.get_status(clear=True)
    mxs.set_test_hooks(drop_tile=5)
    try:
        got = _noalloc_outputs(mxs, x, 0.8, 50, u)
    finally:
        mxs.set_test_hooks()
    assert got[3][0] & mxs.ROW_TIMEOUT and got[0][0] == -1
    assert mxs.get_status(clear=True) & mxs.ROW_TIMEOUT
    got = _noalloc_outputs(mxs, x, 0.8, 50, u)  # the next call is exact again
    n0, _, _ = oracle_lib.oracle_sample(x, 0.8, 50, u)
    np.testing.assert_array_equal(got[0], n0)
    assert mxs.get_status(clear=True) == 0


_FRESH = r"""
import ctypes, sys
import torch
sys.path.insert(0, sys.argv[1])
import mxs_sampler as mxs
lib = mxs.load()
rows, V = 256, 151936
g = torch.Generator(device="cuda").manual_seed(5)
lg = torch.randn((rows, V), generator=g, device="cuda")
u = torch.rand(rows, generator=g, device="cuda", dtype=torch.float64)
nxt = torch.empty(rows, dtype=torch.int32, device="cuda")
# The library's CUDA runtime loads its modules (the fixed array among them) on
# its first call on the device; a size query is such a call and allocates nothing.
need = ctypes.c_size_t()
assert lib.mxs_workspace_size(rows, V, 50, ctypes.byref(need)) == 0
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
p = lambda t: ctypes.c_void_p(t.data_ptr())
s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
for _ in range(2):
    rc = lib.mxs_sample_topk_noalloc(p(lg), rows, V, V, 0.8, 50, 1.0, 0.0, p(u), p(nxt), None, None, None, s)
    assert rc == 0, rc
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
ref, _, _ = mxs.sample(lg, 0.8, 50, u, return_topk=False)
torch.cuda.synchronize()
assert torch.equal(nxt, ref)
print("FREE", free0, free1)
"""


def test_noalloc_first_call_of_a_fresh_process_allocates_nothing(mxs):
    """In a fresh process, device free memory is the same before and after the
    first two allocation-free calls. Modules load eagerly, so the library's
    module (with the fixed array) is resident after its first call of any kind,
    here a workspace-size query made before the measurement."""
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _FRESH, os.path.join(ROOT, "minxfmr.cpp_b200")], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith("FREE")][-1]
    free0, free1 = map(int, line.split()[1:])
    assert free0 == free1, (free0, free1)
