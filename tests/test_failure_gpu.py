"""Failure detection without a GPU fault: a bounded device wait is made to run
out (the test hook drop_tile of mxs_set_test_hooks makes CTA 0's producer stop before one
of its tiles, so the mbarrier that tile would complete is never completed).
The consumers give up after ~1 s, the affected rows come back with
MXS_ROW_TIMEOUT and next = -1, mxs_get_status reports it, every other row is
still exact, and the context stays usable for the next call."""
import numpy as np
import pytest
import torch

import oracle_lib
import workloads

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(mxs):
    rows, k, T = 512, 50, 0.8
    x = workloads.normal(21, rows, workloads.V_QWEN, 2.0)
    u = oracle_lib.uniforms(21, rows)
    lg = torch.from_numpy(x).cuda()
    uu = torch.from_numpy(u).cuda()
    n0, _, _ = oracle_lib.oracle_sample(x, T, k, u)
    mxs.get_status(clear=True)

    mxs.set_test_hooks(drop_tile=5)
    try:
        nxt, _, _, flags = mxs.sample(lg, T, k, uu, return_topk=False, return_flags=True)
    finally:
        mxs.set_test_hooks()
    torch.cuda.synchronize()
    nxt, flags = nxt.cpu().numpy(), flags.cpu().numpy()
    timed_out = (flags & mxs.ROW_TIMEOUT) != 0
    assert timed_out[0], "row 0 (CTA 0's first unit) must report the timeout"
    assert (nxt[timed_out] == -1).all()
    assert timed_out.sum() <= 4  # only CTA 0's rows
    np.testing.assert_array_equal(nxt[~timed_out], n0[~timed_out])
    assert mxs.get_status(clear=True) & mxs.ROW_TIMEOUT

    nxt2, _, _ = mxs.sample(lg, T, k, uu, return_topk=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(nxt2.cpu().numpy(), n0)
    assert mxs.get_status(clear=True) == 0
