"""The reference's pre-sampler edits (special-token mask and repetition /
frequency / presence penalties, src/api/minxfmr.cpp:2047-2089) before the
sampling block.

CPU: the oracle's restatement against the reference's own edit block and
sampling block (oracle/_ref) and against the committed golden fixtures made
from it. GPU (marked gpu): mxs_sample_topk_edits through the C ABI against
the golden fixtures and the oracle, penalised logits carried as the doubles
the reference computes (ids and order bit-exact, probabilities within 1e-6)."""
import os

import numpy as np
import pytest

import oracle_lib

HERE = os.path.dirname(os.path.abspath(__file__))
RTOL = 1e-6


def load_edit_golden():
    z = np.load(os.path.join(HERE, "golden", "edits_golden.npz"))
    cases = {}
    for key in z.files:
        name, field = key.split("/", 1)
        v = z[key]
        cases.setdefault(name, {})[field] = v.item() if v.ndim == 0 else v
    return [cases[n] for n in sorted(cases, key=lambda s: int(s[5:]))]


EDIT_CASES = load_edit_golden()


def edits_of(c):
    return oracle_lib.Edits(c["special"], c["hist"], c["hist_len"], c["repeat_last_n"], c["repeat_penalty"],
                            c["frequency_penalty"], c["presence_penalty"])


def check_edit_golden(c, nxt, idx, prob):
    from test_oracle import truncated_probs
    np.testing.assert_array_equal(nxt, c["next"], err_msg=c["name"])
    np.testing.assert_array_equal(idx, c["idx"], err_msg=c["name"])
    for r in range(len(nxt)):
        n = int(c["plen"][r])
        if n <= 0:
            continue
        t, _ = truncated_probs(prob[r], c["top_p"], c["min_p"])
        np.testing.assert_allclose(t[:n], c["prob"][r, :n], rtol=RTOL, atol=0, err_msg=c["name"])


@pytest.mark.parametrize("c", EDIT_CASES, ids=[c["name"] for c in EDIT_CASES])
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["stl", "restated", "top_down"])
def test_oracle_edits_match_reference_golden(c, mode):
    u = oracle_lib.uniforms(c["seed"], c["logits"].shape[0])
    nxt, idx, prob = oracle_lib.oracle_sample_edits(c["logits"], c["T"], c["k"], u, edits_of(c), c["top_p"],
                                                    c["min_p"], mode=mode)
    check_edit_golden(c, nxt, idx, prob)


@pytest.mark.skipif(not oracle_lib.ref_available(), reason="oracle/_ref not built")
def test_oracle_edits_match_live_reference():
    rng = np.random.default_rng(5)
    for t in range(60):
        V = int(rng.integers(20, 3000))
        rows = int(rng.integers(1, 4))
        x = (np.round(rng.standard_normal((rows, V)) * 4) / 4).astype(np.float32)
        hl = rng.integers(0, 100, rows).astype(np.int32)
        hist = rng.integers(-3, V + 3, (rows, max(int(hl.max()), 1))).astype(np.int32)
        ed = oracle_lib.Edits(rng.integers(-2, V + 2, int(rng.integers(0, 6))), hist, hl,
                              int(rng.choice([-1, 0, 8, 64])), float(rng.choice([1.0, 1.1, 0.9])),
                              float(rng.choice([0.0, 0.5])), float(rng.choice([0.0, -0.1])))
        T, k = float(rng.choice([0.0, 0.7])), int(rng.choice([1, 5, 40, V]))
        u = oracle_lib.uniforms(t, rows)
        n0, i0, p0 = oracle_lib.oracle_sample_edits(x, T, k, u, ed)
        n1, i1, p1, _ = oracle_lib.ref_sample_edits(x, T, k, t, ed)
        np.testing.assert_array_equal(n0, n1)
        np.testing.assert_array_equal(i0, i1)


def _gpu(mxs, x, T, k, u, ed, top_p=1.0, min_p=0.0):
    """Through mxs_sample_topk_edits; rows padded to a leading dimension that is
    a multiple of 4 (the entry point wants 16-byte aligned rows)."""
    import torch
    rows, V = x.shape
    ld = (V + 3) // 4 * 4
    buf = torch.full((rows, ld), float("nan"), dtype=torch.float32)
    buf[:, :V] = torch.from_numpy(np.ascontiguousarray(x))
    lg = buf.cuda()[:, :V]
    out = mxs.sample_edits(lg, T, k, torch.from_numpy(u).cuda(), torch.from_numpy(ed.special).cuda(),
                           torch.from_numpy(ed.hist).cuda(), torch.from_numpy(ed.hist_len).cuda(), ed.repeat_last_n,
                           ed.repeat_penalty, ed.frequency_penalty, ed.presence_penalty, top_p, min_p,
                           return_flags=True)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in out]


@pytest.mark.gpu
@pytest.mark.parametrize("c", EDIT_CASES, ids=[c["name"] for c in EDIT_CASES])
def test_gpu_edits_match_reference_golden(mxs, c):
    x = c["logits"]
    u = oracle_lib.uniforms(c["seed"], x.shape[0])
    nxt, idx, prob, _ = _gpu(mxs, x, c["T"], c["k"], u, edits_of(c), c["top_p"], c["min_p"])
    check_edit_golden(c, nxt, idx, prob)


def _penalty_rows(seed, rows, V, bf16=False):
    """Rows whose histories sit on their largest logits, plus crafted cases: a
    penalised value just above an equal float (the fp32 key ties, the double
    does not), two penalised tokens with equal doubles (a real tie), a special
    token inside the first k columns."""
    import workloads
    x = workloads.normal(seed, rows, V, 2.0)
    if bf16:
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)
    rng = np.random.default_rng(seed)
    H = 64
    hist = np.zeros((rows, H), np.int32)
    for r in range(rows):
        top = np.argsort(-x[r])[:32]
        hist[r] = rng.choice(top, H)
    hl = np.full(rows, H, np.int32)
    # row 0: token a's penalised value 9.0 - 0.1 (one use, presence 0) is a
    # double just above float(8.9) rounded down; token b holds that float
    a, b = 1000, 2000
    x[0, a] = 9.0
    x[0, b] = np.float32(np.nextafter(np.float32(8.9), np.float32(-np.inf))) if np.float32(8.9) > 8.9 else np.float32(8.9)
    hist[0, :] = a
    hl[0] = 1
    # row 1: two tokens with equal logits and equal counts: equal doubles after the penalty
    if rows > 1:
        x[1, 3000] = x[1, 4000] = 8.5
        hist[1, :2] = [3000, 4000]
        hist[1, 2:] = hist[1, 2]
    special = np.array([5, 17, int(np.argmax(x[min(2, rows - 1)]))], np.int32)
    return x, oracle_lib.Edits(special, hist, hl, 64, 1.0, 0.1, 0.0)


@pytest.mark.gpu
@pytest.mark.parametrize("k,bf16", [(8, False), (50, False), (128, False), (50, True)])
def test_gpu_edits_match_oracle_full_size(mxs, k, bf16):
    import workloads
    rows, V = 64, workloads.V_QWEN
    x, ed = _penalty_rows(900 + k, rows, V, bf16)
    for rp, fp, pp in [(1.0, 0.1, 0.0), (1.1, 0.0, 0.0), (1.3, 0.37, 0.2)]:
        ed.repeat_penalty, ed.frequency_penalty, ed.presence_penalty = rp, fp, pp
        u = oracle_lib.uniforms(900 + k, rows)
        nxt, idx, prob, fl = _gpu(mxs, x, 0.8, k, u, ed)
        n0, i0, p0 = oracle_lib.oracle_sample_edits(x, 0.8, k, u, ed, threads=8)
        np.testing.assert_array_equal(nxt, n0, err_msg=f"rp={rp} fp={fp} pp={pp}")
        np.testing.assert_array_equal(idx, i0, err_msg=f"rp={rp} fp={fp} pp={pp}")
        np.testing.assert_allclose(prob, p0, rtol=RTOL, atol=0)


@pytest.mark.gpu
def test_gpu_edits_limits(mxs):
    import torch
    x = torch.zeros((4, 1000), device="cuda")
    u = torch.zeros(4, dtype=torch.float64, device="cuda")
    with pytest.raises(mxs.SamplerError):
        mxs.sample_edits(x, 1.0, 200, u)  # top_k above 128
    h = torch.zeros((4, 2000), dtype=torch.int32, device="cuda")
    hl = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(mxs.SamplerError):
        mxs.sample_edits(x, 1.0, 8, u, history=h, history_len=hl, repeat_last_n=-1)  # window above 1024
