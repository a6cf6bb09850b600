"""A minimal NCCL communicator for jx_attn_step_sharded, through ctypes.

The library takes an ncclComm_t; this module makes one from the process's
libnccl.so.2 (the copy torch already loaded, else the system one):

    uid = NcclComm.unique_id()            # on one rank, shared with the others
    comm = NcclComm(world, rank, uid)     # on every rank, its device current
    jx.attn_step_sharded(..., comm=comm.handle, timeout_ms=5000)
    comm.destroy()                        # or comm.abort() after a failure

Creating the communicator is collective: every rank must construct it.
"""
from __future__ import annotations

import ctypes as C

_NCCL_UNIQUE_ID_BYTES = 128  # sizeof(ncclUniqueId)


class _UniqueId(C.Structure):
    _fields_ = [("internal", C.c_ubyte * _NCCL_UNIQUE_ID_BYTES)]


_lib = None


def _nccl() -> C.CDLL:
    global _lib
    if _lib is None:
        try:
            import torch  # noqa: F401  (loads torch's NCCL first when present)
        except ImportError:
            pass
        lib = C.CDLL("libnccl.so.2", mode=C.RTLD_GLOBAL)
        lib.ncclGetUniqueId.argtypes = [C.POINTER(_UniqueId)]
        lib.ncclCommInitRank.argtypes = [C.POINTER(C.c_void_p), C.c_int, _UniqueId, C.c_int]
        lib.ncclCommDestroy.argtypes = [C.c_void_p]
        lib.ncclCommAbort.argtypes = [C.c_void_p]
        lib.ncclGetErrorString.argtypes = [C.c_int]
        lib.ncclGetErrorString.restype = C.c_char_p
        for fn in (lib.ncclGetUniqueId, lib.ncclCommInitRank, lib.ncclCommDestroy,
                   lib.ncclCommAbort):
            fn.restype = C.c_int
        _lib = lib
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _nccl().ncclGetErrorString(rc)
        raise RuntimeError(f"{what}: {msg.decode() if msg else rc}")


class NcclComm:
    """An NCCL communicator of `world` ranks; `handle` is the ncclComm_t address."""

    @staticmethod
    def unique_id() -> bytes:
        uid = _UniqueId()
        _check(_nccl().ncclGetUniqueId(C.byref(uid)), "ncclGetUniqueId")
        return C.string_at(C.addressof(uid), _NCCL_UNIQUE_ID_BYTES)

    def __init__(self, world: int, rank: int, uid: bytes):
        if len(uid) != _NCCL_UNIQUE_ID_BYTES:
            raise ValueError("uid must be the 128 bytes of NcclComm.unique_id()")
        u = _UniqueId.from_buffer_copy(uid)
        comm = C.c_void_p()
        _check(_nccl().ncclCommInitRank(C.byref(comm), world, u, rank), "ncclCommInitRank")
        self.handle = comm.value
        self.world, self.rank = world, rank

    def destroy(self) -> None:
        if self.handle:
            _check(_nccl().ncclCommDestroy(C.c_void_p(self.handle)), "ncclCommDestroy")
            self.handle = None

    def abort(self) -> None:
        if self.handle:
            _nccl().ncclCommAbort(C.c_void_p(self.handle))
            self.handle = None

