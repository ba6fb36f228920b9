"""CUDA-graph capture of a sampling call (decode loops replay one graph per
step). A captured call passes its own workspace (the library-owned one can be
reallocated by later calls); every replay must sample its current inputs
exactly, tie rows (replayed in the finish kernel) included."""
import numpy as np
import pytest
import torch

import oracle_lib
import workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k", [(1, 8), (16, 50), (256, 128)])
def test_captured_call_replays_new_inputs(mxs, rows, k):
    V = workloads.V_QWEN
    xs = [workloads.normal(600 + i, rows, V, 2.0) for i in range(3)]
    xs[1][0, 500:503] = xs[1][0].max() + 1.0  # a tie at the top of row 0: the exact replay runs in the graph
    us = [oracle_lib.uniforms(600 + i, rows) for i in range(3)]
    lg = torch.empty((rows, V), dtype=torch.float32, device="cuda")
    u = torch.empty(rows, dtype=torch.float64, device="cuda")
    kk = mxs.k_use(k, V)
    out = (torch.empty(rows, dtype=torch.int32, device="cuda"), torch.empty((rows, kk), dtype=torch.int32, device="cuda"),
           torch.empty((rows, kk), dtype=torch.float64, device="cuda"), torch.empty(rows, dtype=torch.int32, device="cuda"))
    ws = mxs.make_workspace(rows, V, k)
    lg.copy_(torch.from_numpy(xs[0]))
    u.copy_(torch.from_numpy(us[0]))
    mxs.sample(lg, 0.8, k, u, out=out, workspace=ws, return_flags=True)  # first call outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        mxs.sample(lg, 0.8, k, u, out=out, workspace=ws, return_flags=True)
    for i, (x, uu) in enumerate(zip(xs, us)):
        lg.copy_(torch.from_numpy(x))
        u.copy_(torch.from_numpy(uu))
        g.replay()
        torch.cuda.synchronize()
        n0, i0, p0 = oracle_lib.oracle_sample(x, 0.8, k, uu)
        np.testing.assert_array_equal(out[0].cpu().numpy(), n0)
        np.testing.assert_array_equal(out[1].cpu().numpy(), i0)
        np.testing.assert_allclose(out[2].cpu().numpy(), p0, rtol=1e-6, atol=0)
        if i == 1 and kk > 1:
            assert out[3][0].item() & mxs.ROW_EXACT, "the tied row must have taken the exact replay"
