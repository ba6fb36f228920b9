"""Seeded synthetic inputs for the sampler's configurations (numpy, host).

The reference measures on no public dataset; these generators stand in for
decode-step logits with the shapes and value distributions of each
configuration. Uniforms come from the oracle: u[r] is what
std::discrete_distribution draws from std::mt19937(seed + r), so the
reference's own block (oracle/_ref) run with that seed draws the same u.
"""
import numpy as np

V_QWEN = 151936
V_LLAMA3 = 128256


def normal(seed, rows, vocab, sigma):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(sigma)).astype(np.float32)


def spiked(seed, rows, vocab, sigma=3.0, spikes=16, add=12.0):
    """N(0, sigma^2) plus `spikes` random positions per row raised by `add`."""
    x = normal(seed, rows, vocab, sigma)
    rng = np.random.default_rng(seed + 1)
    for r in range(rows):
        pos = rng.choice(vocab, size=spikes, replace=False)
        x[r, pos] += np.float32(add)
    return x


def gumbel_ties(seed, rows, vocab, step=1.0 / 16):
    """Standard Gumbel -ln(-ln U) quantised to multiples of `step` (heavy ties)."""
    rng = np.random.default_rng(seed)
    u = rng.random((rows, vocab))
    g = -np.log(-np.log(np.clip(u, 1e-300, 1.0)))
    return (np.round(g / step) * step).astype(np.float32)


CONFIGS = {
    # name: (generator, temperature, top_k)
    "c1_single_row": (lambda s, rows=1, vocab=V_QWEN: normal(s, rows, vocab, 2.0), 0.8, 8),
    "c2_batched_spiked": (lambda s, rows=64, vocab=V_QWEN: spiked(s, rows, vocab), 0.7, 40),
    "c4_ties_k1024": (lambda s, rows=256, vocab=V_QWEN: gumbel_ties(s, rows, vocab), 1.0, 1024),
    "c5_throughput": (lambda s, rows=4096, vocab=V_QWEN: normal(s, rows, vocab, 2.0), 0.8, 50),
}
C3_KS = (1, 2, 128, V_LLAMA3)
C3_TS = (0.1, 1.0, 2.0)


def c3_edge(seed, rows=512, vocab=V_LLAMA3):
    return normal(seed, rows, vocab, 1.5)
