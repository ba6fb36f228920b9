"""The output projection on the device (mxs_sample_from_hidden, the reference's
lm_head step src/api/minxfmr.cpp:1918-2036 kept in HBM): the logits equal an
fp32 matmul of the bf16 operands within fp32 accumulation error, and the
sampled ids, top-k order and probabilities equal the CPU oracle's on those
logits (bit-exact ids and order, probabilities within 1e-6)."""
import numpy as np
import pytest
import torch

import oracle_lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,d,vocab,k", [(1, 896, 151936, 8), (64, 512, 32000, 40), (256, 1024, 50000, 50)])
def test_hidden_logits_and_samples(mxs, rows, d, vocab, k):
    g = torch.Generator(device="cuda").manual_seed(rows + d)
    hidden = (torch.randn((rows, d), generator=g, device="cuda")).bfloat16()
    weight = (torch.randn((vocab, d), generator=g, device="cuda") * (3.0 / d ** 0.5)).bfloat16()
    u = torch.rand(rows, generator=g, device="cuda", dtype=torch.float64)
    logits = torch.empty((rows, vocab), dtype=torch.float32, device="cuda")
    nxt, idx, prob = mxs.sample_from_hidden(hidden, weight, 0.8, k, u, logits_out=logits)
    torch.cuda.synchronize()
    ref = hidden.float() @ weight.float().T
    torch.testing.assert_close(logits, ref, rtol=1e-4, atol=1e-4)
    x = logits.cpu().numpy()
    n0, i0, p0 = oracle_lib.oracle_sample(x, 0.8, k, u.cpu().numpy())
    np.testing.assert_array_equal(nxt.cpu().numpy(), n0)
    np.testing.assert_array_equal(idx.cpu().numpy(), i0)
    np.testing.assert_allclose(prob.cpu().numpy(), p0, rtol=1e-6, atol=0)
    # the library-owned logits buffer gives the same samples
    n2, i2, _ = mxs.sample_from_hidden(hidden, weight, 0.8, k, u)
    torch.cuda.synchronize()
    assert torch.equal(n2, nxt) and torch.equal(i2, idx)
