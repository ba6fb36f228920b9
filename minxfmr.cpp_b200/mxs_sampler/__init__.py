"""Python host side of the B200 token sampler: ctypes bindings over the C ABI
(include/mxs_sampler.h, built into minxfmr.cpp_b200/lib/libmxs.so).

The sampler is the drop-in for the sampling block of the reference's
minxfmr_generate (src/api/minxfmr.cpp:2091-2171). `sample()` mirrors that
block's inputs -- logits, temperature, top_k, top_p, min_p -- and outputs --
`next` and `order[0, k_use)` -- for a batch of rows held on the GPU, with one
uniform per row in place of the reference's function-static std::mt19937.

torch is only the carrier of device memory and streams here; every computation
runs in libmxs.so's CUDA kernels. There is no CPU fallback: without the built
library or an sm_100 GPU the calls raise.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG_ROOT, "lib", "libmxs.so")

MXS_OK = 0
MXS_ERR_INVALID = -1
MXS_ERR_CUDA = -3
MXS_ERR_TIMEOUT = -4
MXS_ERR_NO_DEVICE = -5
MXS_ERR_WORKSPACE = -6
MXS_ERR_COMM = -7

ROW_EXACT = 1
ROW_NAN = 2
ROW_OVERFLOW = 4
ROW_TIMEOUT = 8
TOKEN_NOT_FIRST = 1
TOKEN_EOS = 2

# Every symbol include/mxs_sampler.h declares.
EXPORTS = (
    "mxs_sample_topk", "mxs_sample_topk_ex", "mxs_workspace_size", "mxs_workspace_init",
    "mxs_sample_topk_host", "mxs_shard_candidates", "mxs_merge_sample", "mxs_get_status",
    "mxs_version", "mxs_sample_topk_noalloc", "mxs_set_profile_events", "mxs_sample_rowsharded",
    "mxs_sample_vocabsharded", "mxs_set_test_hooks", "mxs_vocabsharded_stats", "mxs_sample_topk_edits",
    "mxs_token_checks", "mxs_sample_from_hidden",
)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_I = ctypes.c_int
_SZ = ctypes.c_size_t

_SIGS = {
    "mxs_sample_topk": [_P, _I64, _I64, _I64, _D, _I, _P, _P, _P, _P, _P],
    "mxs_sample_topk_ex": [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P, _P, _SZ, _P],
    "mxs_workspace_size": [_I64, _I64, _I, ctypes.POINTER(_SZ)],
    "mxs_workspace_init": [_P, _SZ, _P],
    "mxs_sample_topk_host": [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P],
    "mxs_shard_candidates": [_P, _I64, _I64, _I64, _I64, _I, _I, _P, _P, _P, _P],
    "mxs_merge_sample": [_P, _P, _P, _I, _I, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P, _P],
    "mxs_get_status": [ctypes.POINTER(ctypes.c_uint32), _I],
    "mxs_set_profile_events": [_P, _P],
    "mxs_sample_topk_noalloc": [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P, _P],
    "mxs_sample_rowsharded": [_P, _I64, _I, _I, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P,
                              ctypes.POINTER(_I64), _P],
    "mxs_sample_vocabsharded": [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P, _P, _P],
    "mxs_set_test_hooks": [_I64, _I, _I],
    "mxs_vocabsharded_stats": [ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "mxs_token_checks": [_I64, _I, _I64, _P, _P, _P, _P, _P, _P],
    "mxs_sample_from_hidden": [_P, _I64, _P, _I64, _I64, _I64, _I64, _D, _I, _D, _D, _P, _P, _P, _P, _P, _I64, _P],
    "mxs_sample_topk_edits": [_P, _I64, _I64, _I64, _D, _I, _D, _D, _P, _I, _P, _I64, _P, _I, _D, _D, _D, _P, _P,
                              _P, _P, _P, _P],
}

_lib = None


class SamplerError(RuntimeError):
    def __init__(self, fn, code):
        super().__init__(f"{fn} returned {code}")
        self.code = code


def load(path=LIB_PATH):
    """Load libmxs.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise RuntimeError(f"libmxs.so not built at {path}: run __graft_entry__.build()")
        lib = ctypes.CDLL(path)
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _I
        lib.mxs_version.argtypes = []
        lib.mxs_version.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def _check(fn, rc):
    if rc != MXS_OK:
        raise SamplerError(fn, rc)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def k_use(top_k, vocab):
    """The reference's clamp (src/api/minxfmr.cpp:1567, :2091-2093)."""
    k = 1 if top_k <= 0 else top_k
    return min(k, vocab)


def _need_cuda(t, name, dtype):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}")


def sample(logits, temperature, top_k, u, top_p=1.0, min_p=0.0, out=None, return_topk=True,
           return_flags=False, workspace=None, stream=None):
    """Sample one token per row of `logits` ([rows, vocab] fp32 CUDA tensor,
    rows may be strided by their leading dimension).

    u: [rows] float64 CUDA tensor of uniforms in [0, 1).
    Returns (next [rows] int32, topk_idx [rows, k_use] int32, topk_prob
    [rows, k_use] float64[, row_flags [rows] uint32 as int32]); the top-k
    tensors are None when return_topk is False.
    """
    _need_cuda(logits, "logits", torch.float32)
    _need_cuda(u, "u", torch.float64)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [rows, vocab] with unit column stride")
    rows, vocab = logits.shape
    if u.numel() != rows or not u.is_contiguous():
        raise ValueError("u must be a contiguous [rows] tensor")
    k = k_use(int(top_k), vocab)
    dev = logits.device
    if out is None:
        nxt = torch.empty(rows, dtype=torch.int32, device=dev)
        idx = torch.empty((rows, k), dtype=torch.int32, device=dev) if return_topk else None
        prob = torch.empty((rows, k), dtype=torch.float64, device=dev) if return_topk else None
        flags = torch.empty(rows, dtype=torch.int32, device=dev) if return_flags else None
    else:
        nxt, idx, prob, flags = out
    lib = load()
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = _ptr(workspace), workspace.numel() * workspace.element_size()
    with torch.cuda.device(dev):
        rc = lib.mxs_sample_topk_ex(_ptr(logits), rows, vocab, logits.stride(0), float(temperature),
                                    int(top_k), float(top_p), float(min_p), _ptr(u), _ptr(nxt),
                                    _ptr(idx), _ptr(prob), _ptr(flags), ws_ptr, ws_bytes,
                                    _stream(stream))
    _check("mxs_sample_topk_ex", rc)
    if return_flags:
        return nxt, idx, prob, flags
    return nxt, idx, prob


def sample_edits(logits, temperature, top_k, u, special=None, history=None, history_len=None, repeat_last_n=64,
                 repeat_penalty=1.0, frequency_penalty=0.0, presence_penalty=0.0, top_p=1.0, min_p=0.0,
                 return_flags=False, stream=None):
    """sample() after the reference's pre-sampler edits, on the device
    (mxs_sample_topk_edits): `special` [n] int32 token ids masked to -inf,
    `history` [rows, stride] int32 accepted tokens with `history_len` [rows]
    int32, and the repetition / frequency / presence penalties over the last
    repeat_last_n of them, in double as the reference applies them. `logits`
    is edited in place (masked and penalised tokens read -inf afterwards)."""
    _need_cuda(logits, "logits", torch.float32)
    _need_cuda(u, "u", torch.float64)
    rows, vocab = logits.shape
    k = k_use(int(top_k), vocab)
    dev = logits.device
    nxt = torch.empty(rows, dtype=torch.int32, device=dev)
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev)
    prob = torch.empty((rows, k), dtype=torch.float64, device=dev)
    flags = torch.empty(rows, dtype=torch.int32, device=dev)
    n_special = 0 if special is None else special.numel()
    stride = 0 if history is None else history.shape[1]
    with torch.cuda.device(dev):
        rc = load().mxs_sample_topk_edits(_ptr(logits), rows, vocab, logits.stride(0), float(temperature),
                                          int(top_k), float(top_p), float(min_p), _ptr(special), n_special,
                                          _ptr(history), stride, _ptr(history_len), int(repeat_last_n),
                                          float(repeat_penalty), float(frequency_penalty), float(presence_penalty),
                                          _ptr(u), _ptr(nxt), _ptr(idx), _ptr(prob), _ptr(flags), _stream(stream))
    _check("mxs_sample_topk_edits", rc)
    if return_flags:
        return nxt, idx, prob, flags
    return nxt, idx, prob


def sample_from_hidden(hidden, weight, temperature, top_k, u, top_p=1.0, min_p=0.0, logits_out=None,
                       return_topk=True, stream=None):
    """The output projection on the device, then the sampler
    (mxs_sample_from_hidden): hidden [rows, d] bf16, weight [vocab, d] bf16
    (CUDA tensors, unit column stride). logits_out (optional) [rows, vocab]
    fp32 receives the logits. Returns (next, topk_idx, topk_prob)."""
    _need_cuda(hidden, "hidden", torch.bfloat16)
    _need_cuda(weight, "weight", torch.bfloat16)
    _need_cuda(u, "u", torch.float64)
    rows, d = hidden.shape
    vocab = weight.shape[0]
    if weight.shape[1] != d or hidden.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("hidden [rows, d] and weight [vocab, d] with unit column stride")
    k = k_use(int(top_k), vocab)
    dev = hidden.device
    nxt = torch.empty(rows, dtype=torch.int32, device=dev)
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev) if return_topk else None
    prob = torch.empty((rows, k), dtype=torch.float64, device=dev) if return_topk else None
    ldl = 0 if logits_out is None else logits_out.stride(0)
    with torch.cuda.device(dev):
        rc = load().mxs_sample_from_hidden(_ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), rows, d,
                                           vocab, float(temperature), int(top_k), float(top_p), float(min_p),
                                           _ptr(u), _ptr(nxt), _ptr(idx), _ptr(prob), _ptr(logits_out), ldl,
                                           _stream(stream))
    _check("mxs_sample_from_hidden", rc)
    return nxt, idx, prob


def token_checks(nxt, topk_idx, token_class, first_step=None, stream=None):
    """mxs_token_checks on a sampling call's outputs: the first-token fallback
    for rows with first_step (uint8 [rows]) set, in place on `nxt`; returns the
    rows' EOS stop flags (uint8 [rows]). token_class: uint8 [vocab] of
    TOKEN_NOT_FIRST / TOKEN_EOS bits."""
    rows = nxt.numel()
    vocab = token_class.numel()
    k = topk_idx.shape[1] if topk_idx is not None else 1
    stop = torch.empty(rows, dtype=torch.uint8, device=nxt.device)
    with torch.cuda.device(nxt.device):
        rc = load().mxs_token_checks(rows, k, vocab, _ptr(topk_idx), _ptr(nxt), _ptr(token_class), _ptr(first_step),
                                     _ptr(stop), _stream(stream))
    _check("mxs_token_checks", rc)
    return stop


def sample_noalloc(logits, temperature, top_k, u, top_p=1.0, min_p=0.0, out=None, stream=None):
    """As sample(), through mxs_sample_topk_noalloc: for hosts that cannot let
    the library allocate device memory (their pool owns the GPU, or the
    per-token path forbids allocation). Scratch comes from a fixed array in the
    library; the caller still owns the outputs (pass them in `out` to avoid any
    allocation here: (next, topk_idx, topk_prob, row_flags), any of the last
    three may be None). Calls that overlap on the GPU share that array and race."""
    _need_cuda(logits, "logits", torch.float32)
    _need_cuda(u, "u", torch.float64)
    rows, vocab = logits.shape
    k = k_use(int(top_k), vocab)
    if out is None:
        dev = logits.device
        out = (torch.empty(rows, dtype=torch.int32, device=dev),
               torch.empty((rows, k), dtype=torch.int32, device=dev),
               torch.empty((rows, k), dtype=torch.float64, device=dev), None)
    nxt, idx, prob, flags = out
    with torch.cuda.device(logits.device):
        rc = load().mxs_sample_topk_noalloc(_ptr(logits), rows, vocab, logits.stride(0), float(temperature),
                                            int(top_k), float(top_p), float(min_p), _ptr(u), _ptr(nxt), _ptr(idx),
                                            _ptr(prob), _ptr(flags), _stream(stream))
    _check("mxs_sample_topk_noalloc", rc)
    return nxt, idx, prob


def workspace_bytes(rows, vocab, top_k, device=None):
    n = ctypes.c_size_t()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        _check("mxs_workspace_size", load().mxs_workspace_size(rows, vocab, int(top_k), ctypes.byref(n)))
    return n.value


def make_workspace(rows, vocab, top_k, device=None, stream=None):
    """A caller-owned, zero-filled workspace for sample(..., workspace=...)."""
    dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
    nbytes = workspace_bytes(rows, vocab, top_k, dev)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check("mxs_workspace_init", load().mxs_workspace_init(_ptr(ws), ws.numel(), _stream(stream)))
    return ws


def sample_host(logits, temperature, top_k, u, top_p=1.0, min_p=0.0, return_topk=False):
    """Host-buffer entry point (numpy arrays or CPU tensors; pinned memory makes
    the copies asynchronous). Synchronous: returns host arrays."""
    import numpy as np
    lg = logits.numpy() if isinstance(logits, torch.Tensor) else logits
    uu = u.numpy() if isinstance(u, torch.Tensor) else u
    if lg.dtype != np.float32 or uu.dtype != np.float64:
        raise ValueError("logits must be float32 and u float64")
    rows, vocab = lg.shape
    k = k_use(int(top_k), vocab)
    nxt = np.empty(rows, np.int32)
    idx = np.empty((rows, k), np.int32) if return_topk else None
    prob = np.empty((rows, k), np.float64) if return_topk else None
    ld = lg.strides[0] // 4
    if lg.strides[1] != 4 or not uu.flags.c_contiguous:
        raise ValueError("logits rows must be contiguous")
    p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    rc = load().mxs_sample_topk_host(p(lg), rows, vocab, ld, float(temperature), int(top_k), float(top_p),
                                     float(min_p), p(uu), p(nxt), p(idx), p(prob),
                                     _stream(None))
    _check("mxs_sample_topk_host", rc)
    return nxt, idx, prob


def shard_candidates(shard_logits, col_offset, top_k, cap, stream=None):
    """Vocab-sharded step 1 on this GPU's column shard: returns (cand [rows, cap]
    int64, count [rows] int32, flags [rows] int32)."""
    _need_cuda(shard_logits, "shard_logits", torch.float32)
    rows, cols = shard_logits.shape
    dev = shard_logits.device
    cand = torch.empty((rows, cap), dtype=torch.int64, device=dev)
    cnt = torch.empty(rows, dtype=torch.int32, device=dev)
    flg = torch.empty(rows, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = load().mxs_shard_candidates(_ptr(shard_logits), rows, cols, shard_logits.stride(0), int(col_offset),
                                         int(top_k), int(cap), _ptr(cand), _ptr(cnt), _ptr(flg), _stream(stream))
    _check("mxs_shard_candidates", rc)
    return cand, cnt, flg


def merge_sample(cand_all, count_all, flags_all, vocab, temperature, top_k, u, top_p=1.0, min_p=0.0,
                 stream=None):
    """Vocab-sharded step 2 over gathered lists: cand_all [nshards, rows, cap],
    count_all/flags_all [nshards, rows]. Returns (next, topk_idx, topk_prob,
    row_flags); rows flagged ROW_EXACT have next = -1 and must be resampled
    from their full logits."""
    nshards, rows, cap = cand_all.shape
    dev = cand_all.device
    k = k_use(int(top_k), vocab)
    nxt = torch.empty(rows, dtype=torch.int32, device=dev)
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev)
    prob = torch.empty((rows, k), dtype=torch.float64, device=dev)
    rflg = torch.empty(rows, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = load().mxs_merge_sample(_ptr(cand_all.contiguous()), _ptr(count_all.contiguous()),
                                     _ptr(flags_all.contiguous()), nshards, cap, rows, vocab, float(temperature),
                                     int(top_k), float(top_p), float(min_p), _ptr(u), _ptr(nxt), _ptr(idx),
                                     _ptr(prob), _ptr(rflg), _stream(stream))
    _check("mxs_merge_sample", rc)
    return nxt, idx, prob, rflg


def sample_rowsharded(local_logits, global_rows, rank, world, temperature, top_k, u_global, top_p=1.0,
                      min_p=0.0, stream=None):
    """This rank's rows of a batch split over `world` ranks (no collective):
    local_logits [local_rows, vocab], u_global [global_rows] float64. Returns
    (next, topk_idx, topk_prob, row_flags) for the local rows."""
    _need_cuda(local_logits, "local_logits", torch.float32)
    _need_cuda(u_global, "u_global", torch.float64)
    rows, vocab = local_logits.shape
    per = (global_rows + world - 1) // world
    want = max(0, min(global_rows, (rank + 1) * per) - min(global_rows, rank * per))
    if rows != want:
        raise ValueError(f"rank {rank} of {world} holds {want} of {global_rows} rows, got {rows}")
    dev = local_logits.device
    k = k_use(int(top_k), vocab)
    nxt = torch.empty(rows, dtype=torch.int32, device=dev)
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev)
    prob = torch.empty((rows, k), dtype=torch.float64, device=dev)
    flg = torch.empty(rows, dtype=torch.int32, device=dev)
    n = ctypes.c_int64(0)
    with torch.cuda.device(dev):
        rc = load().mxs_sample_rowsharded(_ptr(local_logits), int(global_rows), int(rank), int(world), vocab,
                                          local_logits.stride(0), float(temperature), int(top_k), float(top_p),
                                          float(min_p), _ptr(u_global), _ptr(nxt), _ptr(idx), _ptr(prob), _ptr(flg),
                                          ctypes.byref(n), _stream(stream))
    _check("mxs_sample_rowsharded", rc)
    return nxt, idx, prob, flg


def sample_vocabsharded(shard_logits, temperature, top_k, u, comm, top_p=1.0, min_p=0.0, stream=None,
                        return_topk=True):
    """One collective call per rank over an NCCL communicator (an integer
    ncclComm_t, e.g. from mxs_sampler.nccl.comm_init_rank): shard_logits is this
    rank's [rows, vocab / world] column shard, u the [rows] uniforms (the same on
    every rank). Returns (next, topk_idx, topk_prob, row_flags) for every row,
    the same on every rank (topk_idx / topk_prob None without return_topk)."""
    _need_cuda(shard_logits, "shard_logits", torch.float32)
    _need_cuda(u, "u", torch.float64)
    rows, cols = shard_logits.shape
    from . import nccl as _nccl
    vocab = cols * _nccl.comm_count(comm)
    dev = shard_logits.device
    k = k_use(int(top_k), vocab)
    nxt = torch.empty(rows, dtype=torch.int32, device=dev)
    idx = torch.empty((rows, k), dtype=torch.int32, device=dev) if return_topk else None
    prob = torch.empty((rows, k), dtype=torch.float64, device=dev) if return_topk else None
    flg = torch.empty(rows, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = load().mxs_sample_vocabsharded(_ptr(shard_logits), rows, cols, shard_logits.stride(0),
                                            float(temperature), int(top_k), float(top_p), float(min_p), _ptr(u),
                                            _ptr(nxt), _ptr(idx), _ptr(prob), _ptr(flg), ctypes.c_void_p(comm),
                                            _stream(stream))
    _check("mxs_sample_vocabsharded", rc)
    return nxt, idx, prob, flg


def vocabsharded_stats():
    """(tie rows resolved from lists, rows gathered whole) of the last
    sample_vocabsharded call on the current device."""
    a, b = ctypes.c_int64(), ctypes.c_int64()
    _check("mxs_vocabsharded_stats", load().mxs_vocabsharded_stats(ctypes.byref(a), ctypes.byref(b)))
    return a.value, b.value


def set_profile_events(start=None, stop=None):
    """Record torch.cuda.Event pair around the dominant (row-streaming) kernel of
    the next calls on the current device; None, None turns it off."""
    sp = None if start is None else ctypes.c_void_p(start.cuda_event)
    ep = None if stop is None else ctypes.c_void_p(stop.cuda_event)
    _check("mxs_set_profile_events", load().mxs_set_profile_events(sp, ep))


PATH_DEFAULT = 0
PATH_BLOCK = 2


def set_test_hooks(drop_tile=-1, replay_warp_min=1, path=PATH_DEFAULT):
    """Test hooks of this library's tests (mxs_set_test_hooks); the defaults
    turn every hook off."""
    _check("mxs_set_test_hooks", load().mxs_set_test_hooks(int(drop_tile), int(replay_warp_min), int(path)))


def get_status(clear=True):
    f = ctypes.c_uint32()
    _check("mxs_get_status", load().mxs_get_status(ctypes.byref(f), int(clear)))
    return f.value


def version():
    return load().mxs_version().decode()
