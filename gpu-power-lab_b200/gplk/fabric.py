"""Python host side of the fabric step (gplk_fabric_* in include/gplk.h):
an in-place BF16 sum allreduce over NVLink peer memory, one process per GPU.

    fab = Fabric(pg, nbytes)          # collective: every rank of `pg`
    buf = fab.tensor(count)           # this rank's buffer as a torch BF16 tensor
    fab.allreduce_bf16(count)         # in place, every rank, same order
    fab.close()

The CUDA IPC handles are exchanged with torch.distributed (all_gather_object
on `pg`, which may be a gloo or NCCL group). Errors raise gplk.GplkError;
a peer that never arrives shows up as a device-timeout status after the
kernel's bounded waits, read with gplk.status_read().
"""
from __future__ import annotations

import ctypes

import gplk

_p = ctypes.c_void_p


def _bind():
    L = gplk.lib()
    if getattr(L, "_fabric_bound", False):
        return L
    L.gplk_fabric_handle_bytes.restype = ctypes.c_size_t
    L.gplk_fabric_handle_bytes.argtypes = []
    L.gplk_fabric_create.restype = ctypes.c_int
    L.gplk_fabric_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(_p), _p]
    L.gplk_fabric_connect.restype = ctypes.c_int
    L.gplk_fabric_connect.argtypes = [_p, _p]
    L.gplk_fabric_data.restype = _p
    L.gplk_fabric_data.argtypes = [_p]
    L.gplk_fabric_allreduce_bf16.restype = ctypes.c_int
    L.gplk_fabric_allreduce_bf16.argtypes = [_p, ctypes.c_size_t, _p]
    L.gplk_fabric_destroy.restype = ctypes.c_int
    L.gplk_fabric_destroy.argtypes = [_p]
    L.gplk_fabric_allreduce_f32.restype = ctypes.c_int
    L.gplk_fabric_allreduce_f32.argtypes = [_p, ctypes.c_size_t, _p]
    L.gplk_fabric_create_local.restype = ctypes.c_int
    L.gplk_fabric_create_local.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_size_t,
                                           ctypes.POINTER(_p)]
    L._fabric_bound = True
    return L


class _CudaArray:
    """Minimal __cuda_array_interface__ holder so torch can view the buffer."""

    def __init__(self, ptr: int, count: int, typestr: str = "<i2"):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class LocalFabric:
    """One GPU's side of a single-process fabric (gplk_fabric_create_local):
    this process drives every GPU of the group, as the reference's NCCL rung
    does with ncclCommInitAll. Build the group with `local_group`."""

    def __init__(self, handle: ctypes.c_void_p, device: int, nbytes: int):
        self._f = handle
        self.device = device
        self.nbytes = nbytes

    def data_ptr(self) -> int:
        return int(_bind().gplk_fabric_data(self._f))

    def tensor(self, count: int, dtype=None):
        import torch

        dtype = dtype or torch.bfloat16
        es = 2 if dtype == torch.bfloat16 else 4
        assert count * es <= self.nbytes
        with torch.cuda.device(self.device):
            t = torch.as_tensor(_CudaArray(self.data_ptr(), count, "<i2" if es == 2 else "<f4"),
                                device=f"cuda:{self.device}")
        return t.view(torch.bfloat16) if es == 2 else t

    def allreduce(self, count: int, dtype=None, stream=None) -> None:
        import torch

        fn = "gplk_fabric_allreduce_f32" if dtype == torch.float32 else "gplk_fabric_allreduce_bf16"
        s = stream.cuda_stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        gplk._check(fn, getattr(_bind(), fn)(self._f, int(count), s))

    def close(self) -> None:
        if self._f:
            _bind().gplk_fabric_destroy(self._f)
            self._f = _p()


def local_group(devices, nbytes: int) -> list[LocalFabric]:
    """Fabrics over `devices` driven from this one process."""
    L = _bind()
    n = len(devices)
    devs = (ctypes.c_int * n)(*[int(d) for d in devices])
    outs = (_p * n)()
    gplk._check("gplk_fabric_create_local", L.gplk_fabric_create_local(n, devs, int(nbytes), outs))
    return [LocalFabric(_p(outs[i]), int(devices[i]), int(nbytes)) for i in range(n)]


class Fabric:
    def __init__(self, pg, nbytes: int, rank: int | None = None, world: int | None = None):
        """pg: a torch.distributed group (None with rank=0, world=1 for a
        single GPU, which needs no process group)."""
        import torch.distributed as dist

        L = _bind()
        self.rank = dist.get_rank(pg) if rank is None else rank
        self.world = dist.get_world_size(pg) if world is None else world
        self.nbytes = int(nbytes)
        hb = int(L.gplk_fabric_handle_bytes())
        handle = (ctypes.c_ubyte * hb)()
        f = _p()
        gplk._check("gplk_fabric_create", L.gplk_fabric_create(self.rank, self.world, self.nbytes, ctypes.byref(f),
                                                                 ctypes.addressof(handle)))
        self._f = f
        gathered: list = [None] * self.world
        if self.world == 1:
            gathered[0] = bytes(handle)
        else:
            dist.all_gather_object(gathered, bytes(handle), group=pg)
        allh = (ctypes.c_ubyte * (hb * self.world)).from_buffer_copy(b"".join(gathered))
        gplk._check("gplk_fabric_connect", L.gplk_fabric_connect(self._f, ctypes.addressof(allh)))

    def data_ptr(self) -> int:
        return int(_bind().gplk_fabric_data(self._f))

    def tensor(self, count: int):
        """The first `count` BF16 elements of this rank's buffer as a torch tensor."""
        import torch

        assert count * 2 <= self.nbytes
        t = torch.as_tensor(_CudaArray(self.data_ptr(), count), device="cuda")
        return t.view(torch.bfloat16)

    def allreduce_bf16(self, count: int, stream=None) -> None:
        gplk._check("gplk_fabric_allreduce_bf16",
                    _bind().gplk_fabric_allreduce_bf16(self._f, int(count), gplk._stream(stream)))

    def close(self) -> None:
        if self._f:
            _bind().gplk_fabric_destroy(self._f)
            self._f = _p()
