"""ctypes bindings for the CPU oracle (oracle/liboracle.so) and the reference
harness (oracle/_ref/libref_sampler.so). Test infrastructure: only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use these."""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "liboracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_sampler.so")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_I = ctypes.c_int


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_P)


_oracle = None
_ref = None


def build():
    """Compile the oracle (and oracle/_ref when the reference tree is present)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)


def oracle():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.mxs_oracle_sample.argtypes = [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _I, _I]
        lib.mxs_oracle_sample.restype = _I
        lib.mxs_oracle_uniforms.argtypes = [ctypes.c_uint32, _I64, _P]
        lib.mxs_oracle_check_draw.argtypes = [ctypes.c_uint32, _P, _I64, _P, _P]
        lib.mxs_oracle_topk_order.argtypes = [_P, _I64, _I, _I, _P]
        lib.mxs_oracle_sample_edits.argtypes = [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _I, _P, _I64, _P,
                                                _I, _D, _D, _D, _P, _P, _P, _I, _I]
        lib.mxs_oracle_sample_edits.restype = _I
        lib.mxs_oracle_token_checks.argtypes = [_I64, _I64, _I64, _P, _P, _P, _P, _P]
        _oracle = lib
    return _oracle


def ref_available():
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(REF_SO)
        lib.mxs_ref_sample.argtypes = [_P, _I64, _I64, _I64, _D, _I, _D, _D, ctypes.c_uint32,
                                       _P, _P, _P, _P, _I]
        lib.mxs_ref_sample.restype = _I
        lib.mxs_ref_sample_edits.argtypes = [_P, _I64, _I64, _I64, _D, _I, _D, _D, ctypes.c_uint32, _P, _I, _P,
                                             _I64, _P, _I, _D, _D, _D, _P, _P, _P, _P, _I]
        lib.mxs_ref_sample_edits.restype = _I
        _ref = lib
    return _ref


def k_use(top_k, vocab):
    k = 1 if top_k <= 0 else top_k
    return min(k, vocab)


def uniforms(seed, n):
    out = np.empty(n, dtype=np.float64)
    oracle().mxs_oracle_uniforms(seed & 0xFFFFFFFF, n, _ptr(out))
    return out


def oracle_sample(logits, temperature, top_k, u, top_p=1.0, min_p=0.0, mode=0, threads=0):
    """Returns (next[rows], topk_idx[rows,k], topk_prob[rows,k])."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    k = k_use(top_k, vocab)
    nxt = np.empty(rows, np.int32)
    idx = np.empty((rows, k), np.int32)
    prob = np.empty((rows, k), np.float64)
    u = np.ascontiguousarray(u, dtype=np.float64)
    rc = oracle().mxs_oracle_sample(_ptr(logits), rows, vocab, vocab, float(temperature), int(top_k),
                                    float(top_p), float(min_p), _ptr(u), _ptr(nxt), _ptr(idx),
                                    _ptr(prob), mode, threads)
    assert rc == k, rc
    return nxt, idx, prob


def ref_sample(logits, temperature, top_k, seed, top_p=1.0, min_p=0.0, threads=0):
    """The reference's own block; row r draws from std::mt19937(seed + r).
    Returns (next, topk_idx, probs, probs_len)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    k = k_use(top_k, vocab)
    nxt = np.empty(rows, np.int32)
    idx = np.empty((rows, k), np.int32)
    prob = np.full((rows, k), np.nan, np.float64)
    plen = np.empty(rows, np.int32)
    rc = ref().mxs_ref_sample(_ptr(logits), rows, vocab, vocab, float(temperature), int(top_k),
                              float(top_p), float(min_p), seed & 0xFFFFFFFF, _ptr(nxt), _ptr(idx),
                              _ptr(prob), _ptr(plen), threads)
    assert rc == k, rc
    return nxt, idx, prob, plen


def topk_order(x, top_k, mode):
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = k_use(top_k, x.shape[0])
    out = np.empty(k, np.int32)
    oracle().mxs_oracle_topk_order(_ptr(x), x.shape[0], int(top_k), mode, _ptr(out))
    return out


class Edits:
    """The reference's pre-sampler edits (src/api/minxfmr.cpp:2047-2089):
    special token ids masked to -inf in every row, then repetition /
    frequency / presence penalties over the last repeat_last_n tokens of each
    row's history (hist [rows, stride] int32, hist_len [rows] int32)."""

    def __init__(self, special, hist, hist_len, repeat_last_n=64, repeat_penalty=1.0, frequency_penalty=0.0,
                 presence_penalty=0.0):
        self.special = np.ascontiguousarray(special, dtype=np.int32)
        self.hist = np.ascontiguousarray(hist, dtype=np.int32)
        self.hist_len = np.ascontiguousarray(hist_len, dtype=np.int32)
        self.repeat_last_n = int(repeat_last_n)
        self.repeat_penalty = float(repeat_penalty)
        self.frequency_penalty = float(frequency_penalty)
        self.presence_penalty = float(presence_penalty)

    def args(self):
        return (_ptr(self.special), len(self.special), _ptr(self.hist), self.hist.shape[1], _ptr(self.hist_len),
                self.repeat_last_n, self.repeat_penalty, self.frequency_penalty, self.presence_penalty)


def oracle_sample_edits(logits, temperature, top_k, u, edits, top_p=1.0, min_p=0.0, mode=0, threads=0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    k = k_use(top_k, vocab)
    nxt = np.empty(rows, np.int32)
    idx = np.empty((rows, k), np.int32)
    prob = np.empty((rows, k), np.float64)
    u = np.ascontiguousarray(u, dtype=np.float64)
    rc = oracle().mxs_oracle_sample_edits(_ptr(logits), rows, vocab, vocab, float(temperature), int(top_k),
                                          float(top_p), float(min_p), _ptr(u), *edits.args(), _ptr(nxt),
                                          _ptr(idx), _ptr(prob), mode, threads)
    assert rc == k, rc
    return nxt, idx, prob


def ref_sample_edits(logits, temperature, top_k, seed, edits, top_p=1.0, min_p=0.0, threads=0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    k = k_use(top_k, vocab)
    nxt = np.empty(rows, np.int32)
    idx = np.empty((rows, k), np.int32)
    prob = np.full((rows, k), np.nan, np.float64)
    plen = np.empty(rows, np.int32)
    rc = ref().mxs_ref_sample_edits(_ptr(logits), rows, vocab, vocab, float(temperature), int(top_k), float(top_p),
                                    float(min_p), seed & 0xFFFFFFFF, *edits.args(), _ptr(nxt), _ptr(idx),
                                    _ptr(prob), _ptr(plen), threads)
    assert rc == k, rc
    return nxt, idx, prob, plen


def token_checks(nxt, order, cls, first_step):
    """The oracle's first-token fallback and EOS flags: returns (next, stop)."""
    nxt = np.array(nxt, dtype=np.int32)
    order = np.ascontiguousarray(order, dtype=np.int32)
    cls = np.ascontiguousarray(cls, dtype=np.uint8)
    first_step = np.ascontiguousarray(first_step, dtype=np.uint8)
    stop = np.empty(len(nxt), np.uint8)
    oracle().mxs_oracle_token_checks(len(nxt), order.shape[1], len(cls), _ptr(order), _ptr(nxt), _ptr(cls),
                                     _ptr(first_step), _ptr(stop))
    return nxt, stop
