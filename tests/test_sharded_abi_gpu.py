"""The C ABI's sharded entry points on one GPU (the 2-GPU runs are in
test_multi_gpu.py):

- mxs_sample_vocabsharded over a one-rank NCCL communicator: the shard is the
  whole row, so the call runs every step (candidates, all-gather, merge, and the
  full-row pass for tie rows) and must equal the oracle on every row;
- mxs_sample_rowsharded: the ranks' row ranges of one batch, sampled one rank
  after another on the same GPU, must equal one unsharded call."""
import numpy as np
import pytest
import torch

import oracle_lib
import workloads

pytestmark = pytest.mark.gpu
RTOL = 1e-6


@pytest.fixture(scope="module")
def comm1(mxs):
    from mxs_sampler import nccl
    c = nccl.comm_init_rank(1, nccl.get_unique_id(), 0)
    yield c
    nccl.comm_destroy(c)


def _vocab_case(mxs, comm, x, T, k, u, top_p=1.0, min_p=0.0):
    nxt, idx, prob, fl = mxs.sample_vocabsharded(torch.from_numpy(x).cuda(), T, k, torch.from_numpy(u).cuda(), comm,
                                                 top_p, min_p)
    torch.cuda.synchronize()
    n0, i0, p0 = oracle_lib.oracle_sample(x, T, k, u, top_p, min_p)
    np.testing.assert_array_equal(nxt.cpu().numpy(), n0)
    np.testing.assert_array_equal(idx.cpu().numpy(), i0)
    np.testing.assert_allclose(prob.cpu().numpy(), p0, rtol=RTOL, atol=0)
    return fl.cpu().numpy()


@pytest.mark.parametrize("k", [1, 8, 50, 128])
def test_vocabsharded_one_rank_normal_rows(mxs, comm1, k):
    x = workloads.normal(500 + k, 64, workloads.V_QWEN, 2.0)
    x[3, 1000:1040] = x[3].max() + 1.0  # a tie row
    u = oracle_lib.uniforms(500 + k, 64)
    fl = _vocab_case(mxs, comm1, x, 0.8, k, u)
    if k >= 8:
        assert fl[3] & mxs.ROW_EXACT


def test_vocabsharded_one_rank_all_rows_tied(mxs, comm1):
    """bf16-rounded logits: nearly every row ties; their ties are resolved from
    lists, with no row gathered whole."""
    x = torch.from_numpy(workloads.normal(510, 600, 32768, 2.0)).bfloat16().float().numpy()
    u = oracle_lib.uniforms(510, 600)
    fl = _vocab_case(mxs, comm1, x, 1.0, 50, u, top_p=0.9)
    assert (fl & mxs.ROW_EXACT).mean() > 0.9
    from_lists, whole = mxs.vocabsharded_stats()
    assert whole == 0 and from_lists == int((fl & mxs.ROW_EXACT).sum())


def test_vocabsharded_one_rank_large_k_takes_full_rows(mxs, comm1):
    """top_k above 128: tie rows are gathered whole (in more than one chunk:
    600 rows > 512 per chunk)."""
    x = torch.from_numpy(workloads.normal(511, 600, 32768, 2.0)).bfloat16().float().numpy()
    u = oracle_lib.uniforms(511, 600)
    fl = _vocab_case(mxs, comm1, x, 1.0, 200, u)
    from_lists, whole = mxs.vocabsharded_stats()
    assert from_lists == 0 and whole == int((fl & mxs.ROW_EXACT).sum()) > 512


def test_vocabsharded_special_rows(mxs, comm1):
    x = workloads.normal(520, 8, 5000, 1.0)
    x[1, 7] = np.nan
    x[2, :] = -np.inf
    x[4, :] = 3.0
    u = oracle_lib.uniforms(520, 8)
    for T in (0.0, 0.7):
        _vocab_case(mxs, comm1, x, T, 40, u)


@pytest.mark.parametrize("world", [1, 3, 8])
def test_rowsharded_ranges_equal_one_call(mxs, world):
    rows, V, k = 37, 20000, 50
    x = torch.from_numpy(workloads.normal(530, rows, V, 2.0)).cuda()
    u = torch.from_numpy(oracle_lib.uniforms(530, rows)).cuda()
    n0, i0, p0 = mxs.sample(x, 0.8, k, u)
    per = (rows + world - 1) // world
    got = []
    for r in range(world):
        lo, hi = min(rows, r * per), min(rows, (r + 1) * per)
        got.append(mxs.sample_rowsharded(x[lo:hi], rows, r, world, 0.8, k, u))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([g[0] for g in got]), n0)
    assert torch.equal(torch.cat([g[1] for g in got]), i0)
    assert torch.equal(torch.cat([g[2] for g in got]), p0)


def test_vocabsharded_one_rank_k_above_merge_limit(mxs, comm1):
    """top_k > 2048: every row goes to the full-row pass."""
    x = np.round(workloads.normal(540, 6, 9000, 1.0) * 32) / 32
    x = x.astype(np.float32)
    u = oracle_lib.uniforms(540, 6)
    fl = _vocab_case(mxs, comm1, x, 1.0, 3000, u)
    assert (fl & mxs.ROW_EXACT).all()
