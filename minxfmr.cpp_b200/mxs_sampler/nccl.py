"""Minimal NCCL communicator handles for the C-ABI vocab-sharded call
(mxs_sample_vocabsharded takes an ncclComm_t).

Binds the libnccl.so.2 the process has already loaded (torch's, when torch is
imported) so that the communicator and the library's collective calls come
from the same NCCL; otherwise loads libnccl.so.2 from the loader's path.
Typical use, one process per GPU:
    uid = nccl.get_unique_id()            # on rank 0, then share the 128 bytes
    comm = nccl.comm_init_rank(world, uid, rank)
    ... mxs_sampler.sample_vocabsharded(shard, T, k, u, comm) ...
    nccl.comm_destroy(comm)
"""
import ctypes
import os


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]


_lib = None


def _nccl():
    global _lib
    if _lib is None:
        try:  # let torch load (and pin) its own NCCL first, so there is one NCCL in the process
            import torch
            torch.cuda.nccl.version()
        except Exception:
            pass
        try:
            lib = ctypes.CDLL("libnccl.so.2", mode=os.RTLD_NOLOAD | os.RTLD_NOW)
        except OSError:
            lib = ctypes.CDLL("libnccl.so.2")
        lib.ncclGetUniqueId.argtypes = [ctypes.POINTER(_UniqueId)]
        lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _UniqueId, ctypes.c_int]
        lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        lib.ncclCommInitAll.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        lib.ncclCommCount.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
        lib.ncclGetErrorString.argtypes = [ctypes.c_int]
        lib.ncclGetErrorString.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def _check(name, rc):
    if rc != 0:
        raise RuntimeError(f"{name}: {_nccl().ncclGetErrorString(rc).decode()}")


def get_unique_id():
    """128 bytes that every rank passes to comm_init_rank."""
    uid = _UniqueId()
    _check("ncclGetUniqueId", _nccl().ncclGetUniqueId(ctypes.byref(uid)))
    # all 128 bytes (reading the c_char field would stop at its first zero byte)
    return ctypes.string_at(ctypes.addressof(uid), 128)


def comm_init_rank(world, uid, rank):
    """A communicator of `world` ranks for the current CUDA device (an integer
    ncclComm_t)."""
    u = _UniqueId()
    ctypes.memmove(ctypes.addressof(u), uid, 128)
    comm = ctypes.c_void_p()
    _check("ncclCommInitRank", _nccl().ncclCommInitRank(ctypes.byref(comm), int(world), u, int(rank)))
    return comm.value


def comm_init_all(devices):
    """Communicators for several GPUs driven by one process (one per device,
    rank i on devices[i]): for hosts that run one thread per GPU."""
    n = len(devices)
    comms = (ctypes.c_void_p * n)()
    devs = (ctypes.c_int * n)(*devices)
    _check("ncclCommInitAll", _nccl().ncclCommInitAll(comms, n, devs))
    return [comms[i] for i in range(n)]


def comm_count(comm):
    n = ctypes.c_int()
    _check("ncclCommCount", _nccl().ncclCommCount(ctypes.c_void_p(comm), ctypes.byref(n)))
    return n.value


def comm_destroy(comm):
    _check("ncclCommDestroy", _nccl().ncclCommDestroy(ctypes.c_void_p(comm)))
