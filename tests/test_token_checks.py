"""The reference's checks on the sampled token (src/api/minxfmr.cpp:2189-2205
first-token fallback, :2232-2243 EOS stop), with the tokenizer's answers given
per token id: mxs_token_checks through the C ABI against the oracle's
restatement (GPU), and the restatement against a direct reading of those
lines (CPU)."""
import numpy as np
import pytest
import torch

import oracle_lib
import workloads


def _classes(rng, V):
    cls = np.zeros(V, np.uint8)
    cls[rng.random(V) < 0.3] |= 1          # invisible pieces / role tokens
    eos = rng.choice(V, 3, replace=False)
    cls[eos] |= 3                          # EOS: also not usable as a first token
    return cls


def test_oracle_token_checks_follow_the_reference_lines():
    rng = np.random.default_rng(3)
    V, rows, k = 500, 64, 10
    cls = _classes(rng, V)
    order = np.stack([rng.permutation(V)[:k] for _ in range(rows)]).astype(np.int32)
    nxt = order[np.arange(rows), rng.integers(0, k, rows)].copy()
    first = (rng.random(rows) < 0.5).astype(np.uint8)
    got, stop = oracle_lib.token_checks(nxt, order, cls, first)
    for r in range(rows):
        want = nxt[r]
        if first[r] and cls[want] & 1:  # :2189 (!visible || eos || role) on the first token
            for i in range(1, k):        # :2190-2202 the first acceptable alternative
                if not cls[order[r, i]] & 1:
                    want = order[r, i]
                    break
        assert got[r] == want
        assert stop[r] == (1 if cls[want] & 2 else 0)  # :2232 EOS stops the row


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 8, 50, 100])
def test_gpu_token_checks_match_oracle(mxs, k):
    rng = np.random.default_rng(k)
    rows, V = 256, 4096
    x = workloads.normal(40 + k, rows, V, 2.0)
    u = oracle_lib.uniforms(40 + k, rows)
    cls = _classes(rng, V)
    top = np.argsort(-x, axis=1)[:, 0]
    cls[top[: rows // 2]] |= 1  # many rows' likely picks are not usable first tokens
    first = (rng.random(rows) < 0.7).astype(np.uint8)
    nxt, idx, prob = mxs.sample(torch.from_numpy(x).cuda(), 0.8, k, torch.from_numpy(u).cuda())
    stop = mxs.token_checks(nxt, idx, torch.from_numpy(cls).cuda(), torch.from_numpy(first).cuda())
    torch.cuda.synchronize()
    n0, i0, _ = oracle_lib.oracle_sample(x, 0.8, k, u)
    want_next, want_stop = oracle_lib.token_checks(n0, i0, cls, first)
    np.testing.assert_array_equal(nxt.cpu().numpy(), want_next)
    np.testing.assert_array_equal(stop.cpu().numpy(), want_stop)
