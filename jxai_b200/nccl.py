"""A minimal NCCL communicator for jx_attn_step_sharded, through ctypes.

The library takes an ncclComm_t; this module makes one from the process's
libnccl.so.2 (the copy torch already loaded, else the system one):

    uid = NcclComm.unique_id()            # on one rank, shared with the others
    comm = NcclComm(world, rank, uid)     # on every rank, its device current
    jx.attn_step_sharded(..., comm=comm.handle, timeout_ms=5000)
    comm.destroy()                        # or comm.abort() after a failure

Creating the communicator is collective: every rank must construct it.  With
`timeout_s` the communicator is created non-blocking (ncclCommInitRankConfig,
blocking = 0) and the creation is polled against a host deadline: a rank that
never joins makes it raise NcclTimeout (after aborting the half-made
communicator) instead of waiting for ever.
"""
from __future__ import annotations

import ctypes as C
import time

_NCCL_UNIQUE_ID_BYTES = 128  # sizeof(ncclUniqueId)


_NCCL_IN_PROGRESS = 7
_NCCL_CONFIG_UNDEF_INT = -2147483648  # INT_MIN
_NCCL_CONFIG_MAGIC = 0xCAFEBEEF


class _UniqueId(C.Structure):
    _fields_ = [("internal", C.c_ubyte * _NCCL_UNIQUE_ID_BYTES)]


class _Config(C.Structure):
    """ncclConfig_t of NCCL 2.28 (ncclConfig_v22800), field for field."""
    _fields_ = [("size", C.c_size_t), ("magic", C.c_uint), ("version", C.c_uint),
                ("blocking", C.c_int), ("cgaClusterSize", C.c_int), ("minCTAs", C.c_int),
                ("maxCTAs", C.c_int), ("netName", C.c_char_p), ("splitShare", C.c_int),
                ("trafficClass", C.c_int), ("commName", C.c_char_p), ("collnetEnable", C.c_int),
                ("CTAPolicy", C.c_int), ("shrinkShare", C.c_int), ("nvlsCTAs", C.c_int),
                ("nChannelsPerNetPeer", C.c_int), ("nvlinkCentricSched", C.c_int)]

    @classmethod
    def initializer(cls, version: int) -> "_Config":
        """NCCL_CONFIG_INITIALIZER: every attribute undefined (NCCL's defaults)."""
        c = cls()
        c.size, c.magic, c.version = C.sizeof(cls), _NCCL_CONFIG_MAGIC, version
        for name, typ in cls._fields_[3:]:
            if typ is C.c_int:
                setattr(c, name, _NCCL_CONFIG_UNDEF_INT)
        return c


class NcclTimeout(RuntimeError):
    """A non-blocking NCCL operation did not finish before its host deadline."""


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
        lib.ncclGetVersion.argtypes = [C.POINTER(C.c_int)]
        lib.ncclCommInitRankConfig.argtypes = [C.POINTER(C.c_void_p), C.c_int, _UniqueId,
                                               C.c_int, C.POINTER(_Config)]
        lib.ncclCommGetAsyncError.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        for fn in (lib.ncclGetUniqueId, lib.ncclCommInitRank, lib.ncclCommDestroy,
                   lib.ncclCommAbort, lib.ncclGetVersion, lib.ncclCommInitRankConfig,
                   lib.ncclCommGetAsyncError):
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

    @staticmethod
    def version() -> int:
        v = C.c_int()
        _check(_nccl().ncclGetVersion(C.byref(v)), "ncclGetVersion")
        return v.value

    def __init__(self, world: int, rank: int, uid: bytes, timeout_s: float | None = None,
                 poll_s: float = 0.001):
        if len(uid) != _NCCL_UNIQUE_ID_BYTES:
            raise ValueError("uid must be the 128 bytes of NcclComm.unique_id()")
        u = _UniqueId.from_buffer_copy(uid)
        comm = C.c_void_p()
        self.world, self.rank = world, rank
        self.blocking = timeout_s is None
        if self.blocking:
            _check(_nccl().ncclCommInitRank(C.byref(comm), world, u, rank), "ncclCommInitRank")
            self.handle = comm.value
            return
        ver = self.version()
        if ver < 22800:
            raise RuntimeError(f"non-blocking init mirrors NCCL 2.28's config; this NCCL is {ver}")
        cfg = _Config.initializer(ver)
        cfg.blocking = 0
        rc = _nccl().ncclCommInitRankConfig(C.byref(comm), world, u, rank, C.byref(cfg))
        if rc not in (0, _NCCL_IN_PROGRESS):
            if comm.value:
                _nccl().ncclCommAbort(comm)
            _check(rc, "ncclCommInitRankConfig")
        self.handle = comm.value
        try:
            self.wait(timeout_s, "communicator creation", poll_s)
        except BaseException:
            self.abort()
            raise

    def async_state(self) -> int:
        """ncclCommGetAsyncError: 0 done, 7 (ncclInProgress) still working, else an error."""
        st = C.c_int(0)
        _check(_nccl().ncclCommGetAsyncError(C.c_void_p(self.handle), C.byref(st)),
               "ncclCommGetAsyncError")
        return st.value

    def wait(self, timeout_s: float, what: str = "operation", poll_s: float = 0.001) -> None:
        """Polls a non-blocking communicator until its pending work is done,
        raising NcclTimeout at the deadline (the communicator is left as it
        is: abort() is the caller's decision) or RuntimeError on an error."""
        deadline = time.monotonic() + timeout_s
        while True:
            st = self.async_state()
            if st == 0:
                return
            if st != _NCCL_IN_PROGRESS:
                _check(st, what)
            if time.monotonic() > deadline:
                raise NcclTimeout(f"NCCL {what} did not finish within {timeout_s} s "
                                  "(a rank that never joined?)")
            time.sleep(poll_s)

    def destroy(self) -> None:
        if self.handle:
            _check(_nccl().ncclCommDestroy(C.c_void_p(self.handle)), "ncclCommDestroy")
            self.handle = None

    def abort(self) -> None:
        if self.handle:
            _nccl().ncclCommAbort(C.c_void_p(self.handle))
            self.handle = None

