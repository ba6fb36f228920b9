"""Generate tests/golden/edits_golden.npz from the reference's OWN pre-sampler
edits and sampling block (oracle/_ref/libref_sampler.so: src/api/minxfmr.cpp
:2047-2089 and :2091-2171 compiled inside a harness; `make -C oracle` where the
reference tree exists).

Each case: its logits (fp32), the special token ids, the per-row histories and
the penalty parameters, and the reference's outputs (next, order[0, k_use),
the probs vector and its length). Rows draw from std::mt19937(seed + row), the
u mxs_oracle_uniforms gives. Run: python tests/golden/make_golden_edits.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_lib  # noqa: E402

OUT = os.path.join(HERE, "edits_golden.npz")


def make_case(rng, i):
    V = int(rng.choice([257, 1000, 4096]))
    rows = int(rng.integers(1, 4))
    kind = i % 3
    x = rng.standard_normal((rows, V)).astype(np.float32) * 2
    if kind == 1:
        x = (np.round(x * 4) / 4).astype(np.float32)  # ties
    elif kind == 2:
        x = x.astype(np.float16).astype(np.float32)
    # histories drawn mostly from each row's largest logits, so the penalties
    # move tokens across the top-k
    H = int(rng.integers(1, 96))
    hist = np.zeros((rows, H), np.int32)
    for r in range(rows):
        top = np.argsort(-x[r])[:24]
        hist[r] = np.where(rng.random(H) < 0.8, rng.choice(top, H), rng.integers(-2, V + 2, H))
    hist_len = rng.integers(0, H + 1, rows).astype(np.int32)
    special = np.concatenate([np.argsort(-x[0])[:int(rng.integers(0, 4))],
                              rng.integers(-1, V + 1, int(rng.integers(0, 3)))]).astype(np.int32)
    e = dict(special=special, hist=hist, hist_len=hist_len,
             repeat_last_n=int(rng.choice([-1, 8, 64])), repeat_penalty=float(rng.choice([1.0, 1.1, 1.3, 0.8])),
             frequency_penalty=float(rng.choice([0.0, 0.1, 0.37])), presence_penalty=float(rng.choice([0.0, 0.2, -0.15])))
    k = int(rng.choice([1, 5, 40, 50, 128]))
    T = float(rng.choice([0.0, 0.7, 1.0]))
    top_p = float(rng.choice([1.0, 1.0, 0.9]))
    min_p = float(rng.choice([0.0, 0.0, 0.05]))
    return dict(name=f"edits{i}", logits=x, k=k, T=T, top_p=top_p, min_p=min_p, seed=2000 + i, **e)


def main():
    if not oracle_lib.ref_available():
        raise SystemExit("oracle/_ref not built (needs the reference tree): make -C oracle")
    rng = np.random.default_rng(20261202)
    out = {}
    cases = [make_case(rng, i) for i in range(40)]
    for c in cases:
        ed = oracle_lib.Edits(c["special"], c["hist"], c["hist_len"], c["repeat_last_n"], c["repeat_penalty"],
                              c["frequency_penalty"], c["presence_penalty"])
        n, idx, prob, plen = oracle_lib.ref_sample_edits(c["logits"], c["T"], c["k"], c["seed"], ed, c["top_p"],
                                                         c["min_p"])
        c.update(next=n, idx=idx, prob=prob, plen=plen)
        for key, v in c.items():
            out[f"{c['name']}/{key}"] = np.asarray(v)
    np.savez_compressed(OUT, **out)
    print(f"{len(cases)} cases -> {OUT}")


if __name__ == "__main__":
    main()
