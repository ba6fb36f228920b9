"""CPU tests of the oracle: pinned against the reference's own sampling block
(golden fixtures generated from oracle/_ref, and oracle/_ref itself when it was
built here), its heap restatement against the real std::partial_sort, and the
injected-u draw against std::discrete_distribution."""
import os

import numpy as np
import pytest

import oracle_lib
import workloads

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sampler_golden.npz")


def load_golden():
    z = np.load(GOLDEN, allow_pickle=False)
    cases = []
    for name in z["cases"]:
        name = str(name)
        p = name + "/"
        c = {"name": name}
        T, k, top_p, min_p, seed = z[p + "params"]
        c.update(T=float(T), k=int(k), top_p=float(top_p), min_p=float(min_p), seed=int(seed))
        if p + "logits" in z:
            c["logits"] = z[p + "logits"]
        else:
            c["gen"] = str(z[p + "gen"])
            c["shape"] = tuple(int(v) for v in z[p + "shape"])
            c["sha"] = str(z[p + "sha"])
        for key in ("next", "idx", "prob", "plen", "idx_sha", "idx_head", "prob_head"):
            if p + key in z:
                c[key] = z[p + key]
        cases.append(c)
    return cases


def golden_logits(c):
    if "logits" in c:
        return c["logits"]
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    x = mg.regenerate(c["gen"], c["seed"], *c["shape"])
    assert mg.sha(x) == c["sha"], "regenerated logits differ from the fixture's"
    return x


def truncated_probs(p, top_p, min_p):
    """The reference's top-p then min-p truncation with renormalisation
    (src/api/minxfmr.cpp:2104-2111 clamps, :2128-2165), applied to one row's
    first-normalised probabilities p[0, k) with the same double operations in
    the same order (Python floats are IEEE doubles). Returns the whole vector
    as the reference leaves it (the kept prefix renormalised in place, the rest
    untouched) and the kept count."""
    if top_p <= 0.0 or top_p > 1.0:
        top_p = 1.0
    min_p = min(max(min_p, 0.0), 1.0)
    q = [float(v) for v in p]
    n = len(q)
    if top_p < 1.0:
        cum, n = 0.0, 0
        for i in range(len(q)):
            cum += q[i]
            n = i + 1
            if cum >= top_p:
                break
        n = max(n, 1)
        renorm = 0.0
        for i in range(n):
            renorm += q[i]
        if renorm > 0.0:
            for i in range(n):
                q[i] /= renorm
    if min_p > 0.0 and n > 1:
        thr = q[0] * min_p
        keep = 1
        for i in range(1, n):
            if q[i] >= thr:
                keep = i + 1
            else:
                break
        n = keep
        renorm = 0.0
        for i in range(n):
            renorm += q[i]
        if renorm > 0.0:
            for i in range(n):
                q[i] /= renorm
    return np.array(q), n


def check_against_golden(c, nxt, idx, prob):
    """Compare sampler outputs with a golden case: ids and order bit-exact;
    probabilities within 1e-6 relative. The reference's probs vector is the
    first-normalised one when top_p = 1 and min_p = 0; otherwise it is the
    truncated, renormalised one, which the sampler's first-normalised output
    must reproduce through the reference's truncation steps."""
    import hashlib
    np.testing.assert_array_equal(nxt, c["next"], err_msg=c["name"])
    if "idx" in c:
        np.testing.assert_array_equal(idx, c["idx"], err_msg=c["name"])
    else:
        assert hashlib.sha256(np.ascontiguousarray(idx).tobytes()).hexdigest() == str(c["idx_sha"]), c["name"]
        np.testing.assert_array_equal(idx[:, :256], c["idx_head"], err_msg=c["name"])
    ref_prob = c["prob"] if "prob" in c else c["prob_head"]
    got = prob[:, :ref_prob.shape[1]]
    neutral = c["top_p"] >= 1.0 and c["min_p"] <= 0.0
    for r in range(len(nxt)):
        n = int(c["plen"][r])
        if n <= 0:
            continue
        if neutral:
            np.testing.assert_allclose(got[r, :n], ref_prob[r, :n], rtol=1e-6, atol=0, err_msg=c["name"])
        elif "prob" in c:
            t, _ = truncated_probs(prob[r], c["top_p"], c["min_p"])
            np.testing.assert_allclose(t[:n], ref_prob[r, :n], rtol=1e-6, atol=0, err_msg=c["name"])


GOLDEN_CASES = load_golden()


@pytest.mark.parametrize("c", GOLDEN_CASES, ids=[c["name"] for c in GOLDEN_CASES])
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["stl", "restated", "top_down"])
def test_oracle_matches_reference_golden(c, mode):
    x = golden_logits(c)
    u = oracle_lib.uniforms(c["seed"], x.shape[0])
    nxt, idx, prob = oracle_lib.oracle_sample(x, c["T"], c["k"], u, c["top_p"], c["min_p"], mode=mode)
    check_against_golden(c, nxt, idx, prob)


@pytest.mark.skipif(not oracle_lib.ref_available(), reason="oracle/_ref not built (reference tree absent)")
def test_oracle_matches_live_reference_block():
    rng = np.random.default_rng(5)
    for trial in range(40):
        V = int(rng.integers(1, 3000))
        rows = 3
        x = (np.round(rng.standard_normal((rows, V)) * 4) / 4).astype(np.float32)
        k = int(rng.integers(0, V + 3))
        T = float(rng.choice([0.0, 0.5, 1.0]))
        seed = int(rng.integers(0, 2**31))
        u = oracle_lib.uniforms(seed, rows)
        n0, i0, _ = oracle_lib.oracle_sample(x, T, k, u)
        n1, i1, _, _ = oracle_lib.ref_sample(x, T, k, seed)
        np.testing.assert_array_equal(n0, n1)
        np.testing.assert_array_equal(i0, i1)


def test_heap_restatement_matches_std_partial_sort():
    rng = np.random.default_rng(7)
    for trial in range(400):
        V = int(rng.integers(1, 600))
        k = int(rng.integers(0, V + 2))
        q = float(rng.choice([0.5, 0.25, 1.0, 4.0]))
        x = (np.round(rng.standard_normal(V) * q) / q).astype(np.float32)
        if trial % 5 == 0:
            x[rng.random(V) < 0.05] = -np.inf
        np.testing.assert_array_equal(oracle_lib.topk_order(x, k, 0), oracle_lib.topk_order(x, k, 1))


def test_top_down_replacement_matches_std_partial_sort():
    """Mode 2 (the replacement the CUDA replays use on rows without NaN) against
    the real std::partial_sort, on heavily tied rows and rows with NaN."""
    rng = np.random.default_rng(17)
    for trial in range(600):
        V = int(rng.integers(1, 900))
        k = int(rng.integers(0, min(V, 200) + 2))
        q = float(rng.choice([0.25, 1.0, 4.0, 64.0]))
        x = (np.round(rng.standard_normal(V) * q) / q).astype(np.float32)
        if trial % 7 == 0:
            x[rng.random(V) < 0.05] = -np.inf
        if trial % 11 == 0:
            x[rng.random(V) < 0.02] = np.nan
        if trial % 13 == 0:
            x = np.sort(x)  # increasing: every logit enters
        np.testing.assert_array_equal(oracle_lib.topk_order(x, k, 0), oracle_lib.topk_order(x, k, 2), err_msg=str(trial))


def test_known_tie_order():
    # 12 equal logits, k = 5: libstdc++'s heap leaves 3 4 1 0 2, not 0 1 2 3 4.
    x = np.zeros(12, np.float32)
    assert list(oracle_lib.topk_order(x, 5, 0)) == [3, 4, 1, 0, 2]
    assert list(oracle_lib.topk_order(x, 5, 1)) == [3, 4, 1, 0, 2]
    assert list(oracle_lib.topk_order(x, 5, 2)) == [3, 4, 1, 0, 2]


def test_injected_u_equals_discrete_distribution():
    import ctypes
    lib = oracle_lib.oracle()
    rng = np.random.default_rng(9)
    for trial in range(2000):
        n = int(rng.integers(1, 60))
        w = rng.random(n) ** 3
        w /= w.sum()
        a, b = ctypes.c_int32(), ctypes.c_int32()
        lib.mxs_oracle_check_draw(trial, w.ctypes.data_as(ctypes.c_void_p), n, ctypes.byref(a), ctypes.byref(b))
        assert a.value == b.value, (trial, n)


def test_uniforms_in_unit_interval():
    u = oracle_lib.uniforms(123, 10000)
    assert (u >= 0).all() and (u < 1).all()
    assert abs(u.mean() - 0.5) < 0.02


def test_workload_generators_shapes():
    x = workloads.gumbel_ties(1, 2, 1000)
    assert x.dtype == np.float32 and x.shape == (2, 1000)
    assert np.all(np.round(x * 16) == x * 16)
    y = workloads.spiked(1, 2, 1000)
    assert (y > 8).sum() >= 16
