"""GPU test of mxs_sample_topk_noalloc, the entry point for hosts that cannot
let this library allocate device memory (their own pool owns the GPU, or their
per-token path forbids allocation): it must give the same results as the
regular entry point while taking its scratch from the library's fixed array.

Kept in a file of its own that pytest collects last; it passes alone in a fresh
process and after the other tests (the array keeps the previous call's
contents, which is why two calls in a row are checked)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle_lib
import workloads

pytestmark = pytest.mark.gpu
RTOL = 1e-6  # the parity tolerance of the other GPU tests for probabilities


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call_noalloc(lib, lg, T, k, u, nxt, idx, prob, flg, top_p=1.0, min_p=0.0):
    rows, vocab = lg.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.mxs_sample_topk_noalloc(_p(lg), rows, vocab, lg.stride(0), T, k, top_p, min_p, _p(u), _p(nxt),
                                       _p(idx), _p(prob), _p(flg), stream)


@pytest.mark.parametrize("rows,k,T", [(64, 40, 0.7), (4, 8, 0.8), (300, 50, 0.8), (16, 128, 1.0)])
def test_noalloc_matches_regular_entry_point_twice(mxs, rows, k, T):
    lib = mxs.load()
    x = workloads.spiked(200 + rows, rows, workloads.V_QWEN)
    if rows >= 4:
        x[1, 500:560] = 40.0  # a tie row: the exact replay path uses the scratch too
    lg = torch.from_numpy(x).cuda()
    ref_next, ref_idx, ref_prob, ref_flg = mxs.sample(lg, T, k, torch.from_numpy(oracle_lib.uniforms(7, rows)).cuda(),
                                                      return_flags=True)
    kk = mxs.k_use(k, x.shape[1])
    for call in range(2):  # two calls in a row on the shared array
        u = torch.from_numpy(oracle_lib.uniforms(7, rows)).cuda()
        nxt = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
        idx = torch.full((rows, kk), -7, dtype=torch.int32, device="cuda")
        prob = torch.full((rows, kk), -7.0, dtype=torch.float64, device="cuda")
        flg = torch.zeros(rows, dtype=torch.int32, device="cuda")
        rc = _call_noalloc(lib, lg, T, k, u, nxt, idx, prob, flg)
        assert rc == mxs.MXS_OK, rc
        torch.cuda.synchronize()
        np.testing.assert_array_equal(nxt.cpu().numpy(), ref_next.cpu().numpy(), err_msg=f"call {call}")
        np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx.cpu().numpy(), err_msg=f"call {call}")
        np.testing.assert_allclose(prob.cpu().numpy(), ref_prob.cpu().numpy(), rtol=RTOL, atol=0)
        np.testing.assert_array_equal(flg.cpu().numpy(), ref_flg.cpu().numpy())


def test_noalloc_python_wrapper_and_size_limit(mxs):
    x = workloads.normal(9, 8, workloads.V_QWEN, 2.0)
    lg = torch.from_numpy(x).cuda()
    u = torch.from_numpy(oracle_lib.uniforms(9, 8)).cuda()
    n0, i0, p0 = mxs.sample(lg, 0.8, 50, u)
    n1, i1, p1 = mxs.sample_noalloc(lg, 0.8, 50, u)
    torch.cuda.synchronize()
    assert torch.equal(n0, n1) and torch.equal(i0, i1)
    # a shape whose scratch exceeds the fixed array is refused with a clear code
    big = torch.zeros((4096, 40000), dtype=torch.float32, device="cuda")
    ub = torch.zeros(4096, dtype=torch.float64, device="cuda")
    nb = torch.empty(4096, dtype=torch.int32, device="cuda")
    rc = _call_noalloc(mxs.load(), big, 1.0, 40000, ub, nb, None, None, None)
    assert rc == mxs.MXS_ERR_WORKSPACE
