"""Generate tests/golden/sampler_golden.npz from the reference's OWN sampling
block (oracle/_ref/libref_sampler.so: src/api/minxfmr.cpp:2091-2171 compiled
inside a harness; built by `make -C oracle` where the reference tree exists).

Each case stores its parameters, either its logits (small cases) or the seed
that regenerates them plus a SHA-256 of the bytes, and the reference's outputs:
next, order[0, k_use) (the full list, or its SHA-256 plus a head for k = V),
and the probs vector. Rows draw from std::mt19937(seed + row), the same u the
oracle's mxs_oracle_uniforms gives. Run: python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_lib  # noqa: E402
import workloads  # noqa: E402

OUT = os.path.join(HERE, "sampler_golden.npz")
BIG_K = 4096  # above this, store a hash and a head of the order


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def tiny_cases(rng):
    cases = []
    specials = np.array([0.0, -0.0, -np.inf, np.inf], np.float32)
    for i in range(60):
        V = int(rng.integers(1, 400))
        rows = int(rng.integers(1, 4))
        kind = i % 4
        if kind == 0:
            x = (np.round(rng.standard_normal((rows, V)) * 2) / 2).astype(np.float32)
        elif kind == 1:
            x = rng.standard_normal((rows, V)).astype(np.float32)
        elif kind == 2:
            x = rng.integers(-2, 3, (rows, V)).astype(np.float32)
        else:
            x = (np.round(rng.standard_normal((rows, V)) * 2) / 2).astype(np.float32)
            m = rng.random((rows, V)) < 0.1
            x[m] = rng.choice(specials, size=int(m.sum()))
        k = int(rng.choice([0, 1, 2, 3, 5, 8, 40, V, V + 7]))
        T = float(rng.choice([0.0, -1.0, 0.3, 0.7, 1.0, 2.0]))
        top_p = float(rng.choice([1.0, 1.0, 0.9, 0.5, 0.0]))
        min_p = float(rng.choice([0.0, 0.0, 0.05, 0.3]))
        cases.append(dict(name=f"tiny{i}", logits=x, T=T, k=k, top_p=top_p, min_p=min_p, seed=1000 + i))
    return cases


def big_cases():
    out = []
    w = workloads
    out.append(dict(name="c1", gen="c1", seed=11, rows=1, vocab=w.V_QWEN, T=0.8, k=8))
    out.append(dict(name="c2", gen="c2", seed=12, rows=4, vocab=w.V_QWEN, T=0.7, k=40))
    out.append(dict(name="c4", gen="c4", seed=14, rows=3, vocab=w.V_QWEN, T=1.0, k=1024))
    for k in workloads.C3_KS:
        for T in workloads.C3_TS:
            out.append(dict(name=f"c3_k{k}_T{T}", gen="c3", seed=13, rows=2, vocab=w.V_LLAMA3, T=T, k=k))
    out.append(dict(name="c5", gen="c5", seed=15, rows=4, vocab=w.V_QWEN, T=0.8, k=50))
    return out


def regenerate(gen, seed, rows, vocab):
    if gen == "c1" or gen == "c5":
        return workloads.normal(seed, rows, vocab, 2.0)
    if gen == "c2":
        return workloads.spiked(seed, rows, vocab)
    if gen == "c3":
        return workloads.c3_edge(seed, rows, vocab)
    if gen == "c4":
        return workloads.gumbel_ties(seed, rows, vocab)
    raise KeyError(gen)


def main():
    if not oracle_lib.ref_available():
        print("oracle/_ref/libref_sampler.so missing: run make -C oracle with the reference tree present")
        return 2
    rng = np.random.default_rng(20261201)
    blob = {}
    names = []
    for c in tiny_cases(rng) + big_cases():
        if "logits" in c:
            x = c["logits"]
            blob[c["name"] + "/logits"] = x
        else:
            x = regenerate(c["gen"], c["seed"], c["rows"], c["vocab"])
            blob[c["name"] + "/gen"] = np.array(c["gen"])
            blob[c["name"] + "/shape"] = np.array([c["rows"], c["vocab"]], np.int64)
            blob[c["name"] + "/sha"] = np.array(sha(x))
        nxt, idx, prob, plen = oracle_lib.ref_sample(x, c["T"], c["k"], c["seed"], c.get("top_p", 1.0),
                                                     c.get("min_p", 0.0))
        p = c["name"] + "/"
        blob[p + "params"] = np.array([c["T"], c["k"], c.get("top_p", 1.0), c.get("min_p", 0.0), c["seed"]],
                                      np.float64)
        blob[p + "next"] = nxt
        if idx.shape[1] > BIG_K:
            blob[p + "idx_sha"] = np.array(sha(idx))
            blob[p + "idx_head"] = idx[:, :256].copy()
            blob[p + "prob_head"] = prob[:, :256].copy()
        else:
            blob[p + "idx"] = idx
            blob[p + "prob"] = prob
        blob[p + "plen"] = plen
        names.append(c["name"])
    blob["cases"] = np.array(names)
    np.savez_compressed(OUT, **blob)
    print(f"{OUT}: {len(names)} cases, {os.path.getsize(OUT) / 1024:.0f} KB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
