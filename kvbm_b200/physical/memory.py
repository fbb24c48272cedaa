"""Storage for the KV tiers: G1 device pools, G2 mapped pinned host pools,
CUDA IPC export/import of pools between the processes of one node.

Pools are allocated directly with the CUDA runtime (through
``libkvbm_cuda.so``) rather than through the PyTorch caching allocator so that

* an IPC handle maps exactly one pool (no allocator segment offsets), and
* G2 host memory is mapped into the device address space, letting SM kernels
  gather/scatter it directly.

The buffers expose ``__cuda_array_interface__`` (device) or the buffer
protocol (host) so they can be viewed as torch tensors without copies.

Parity: crates/kvbm-physical/src/layout/builder.rs (allocate_device /
allocate_pinned / external regions) and the NIXL registration step, which
on one node reduces to CUDA IPC here.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ..ops import _lib


class StorageKind:
    DEVICE = "device"      # G1
    PINNED = "pinned"      # G2
    DISK = "disk"          # G3
    OBJECT = "object"      # G4
    SYSTEM = "system"      # unpinned host


class DeviceBuffer:
    """A cudaMalloc'd region owned by this object (freed on close/GC)."""

    def __init__(self, nbytes: int, device: int | None = None, zero: bool = False):
        if device is not None:
            torch.cuda.set_device(device)
        self.device = torch.cuda.current_device()
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        _lib.check(_lib.load().kvbm_device_alloc(self.nbytes, C.byref(p)), "cudaMalloc")
        self.ptr = int(p.value or 0)
        self._owned = True
        if zero:
            _lib.check(_lib.load().kvbm_memset_async(self.ptr, 0, self.nbytes, None), "memset")
            torch.cuda.synchronize()

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.nbytes,), "typestr": "|u1", "data": (self.ptr, False), "version": 3,
                "strides": None, "stream": None}

    def tensor(self, dtype: torch.dtype = torch.uint8, shape: tuple | None = None) -> torch.Tensor:
        t = torch.as_tensor(self, device=f"cuda:{self.device}")
        if dtype != torch.uint8:
            t = t.view(dtype)
        if shape is not None:
            t = t.view(shape)
        return t

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        _lib.check(_lib.load().kvbm_ipc_get_handle(self.ptr, buf), "cudaIpcGetMemHandle")
        return bytes(buf.raw[:64])

    def close(self) -> None:
        if self._owned and self.ptr:
            _lib.load().kvbm_device_free(self.ptr)
        self.ptr = 0
        self._owned = False

    def __del__(self):  # pragma: no cover - GC timing
        try:
            self.close()
        except Exception:
            pass


class PeerBuffer:
    """A peer process's DeviceBuffer mapped into this process through CUDA IPC."""

    def __init__(self, handle: bytes, nbytes: int, device: int | None = None):
        if device is not None:
            torch.cuda.set_device(device)
        self.device = torch.cuda.current_device()
        p = C.c_void_p()
        _lib.check(_lib.load().kvbm_ipc_open_handle(bytes(handle), C.byref(p)), "cudaIpcOpenMemHandle")
        self.ptr = int(p.value or 0)
        self.nbytes = int(nbytes)

    def close(self) -> None:
        if self.ptr:
            _lib.load().kvbm_ipc_close(self.ptr)
        self.ptr = 0

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class PinnedBuffer:
    """Pinned host memory mapped into the device address space (G2)."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        _lib.check(_lib.load().kvbm_host_alloc_mapped(self.nbytes, C.byref(p)), "cudaHostAlloc")
        self.ptr = int(p.value or 0)
        d = C.c_void_p()
        _lib.check(_lib.load().kvbm_host_device_pointer(self.ptr, C.byref(d)), "cudaHostGetDevicePointer")
        self.device_ptr = int(d.value or 0)

    def tensor(self, dtype: torch.dtype = torch.uint8, shape: tuple | None = None) -> torch.Tensor:
        arr = (C.c_uint8 * self.nbytes).from_address(self.ptr)
        t = torch.frombuffer(arr, dtype=torch.uint8)
        if dtype != torch.uint8:
            t = t.view(dtype)
        if shape is not None:
            t = t.view(shape)
        return t

    def close(self) -> None:
        if self.ptr:
            _lib.load().kvbm_host_free(self.ptr)
        self.ptr = 0

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


# ---- NUMA placement of host pools ---------------------------------------------
# Linux x86-64 system call numbers and mempolicy constants (uapi/linux/mempolicy.h).
_SYS_MBIND, _SYS_GET_MEMPOLICY = 237, 239
_MPOL_PREFERRED, _MPOL_BIND = 1, 2
_MPOL_MF_MOVE = 1 << 1
_MPOL_F_NODE, _MPOL_F_ADDR = 1 << 0, 1 << 1


def gpu_numa_node(device: int | None = None) -> int:
    """NUMA node of the CPU socket nearest to a GPU (from its PCI device in sysfs), or -1."""
    try:
        props = torch.cuda.get_device_properties(torch.cuda.current_device() if device is None else device)
        path = f"/sys/bus/pci/devices/{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0/numa_node"
        with open(path) as f:
            return int(f.read().strip())
    except Exception:
        return -1


def bind_to_numa(ptr: int, nbytes: int, node: int, strict: bool = False) -> bool:
    """Set the memory policy of the page-aligned range [ptr, ptr + nbytes) to ``node``
    (MPOL_BIND when ``strict``, else MPOL_PREFERRED), moving pages already touched.
    Returns False when the kernel refuses (no such node, or a container without
    CAP_SYS_NICE); the range keeps the default first-touch policy then."""
    if node < 0 or nbytes <= 0:
        return False
    libc = C.CDLL(None, use_errno=True)
    mask = (C.c_ulong * 16)()
    if node >= 16 * 64:
        return False
    mask[node // 64] = 1 << (node % 64)
    rc = libc.syscall(_SYS_MBIND, C.c_void_p(ptr), C.c_ulong(nbytes), C.c_int(_MPOL_BIND if strict else _MPOL_PREFERRED),
                      mask, C.c_ulong(16 * 64 + 1), C.c_uint(_MPOL_MF_MOVE))
    return rc == 0


def numa_node_of(ptr: int) -> int:
    """NUMA node backing the (touched) page at ``ptr``, or -1."""
    libc = C.CDLL(None, use_errno=True)
    node = C.c_int(-1)
    rc = libc.syscall(_SYS_GET_MEMPOLICY, C.byref(node), None, C.c_ulong(0), C.c_void_p(ptr),
                      C.c_ulong(_MPOL_F_NODE | _MPOL_F_ADDR))
    return node.value if rc == 0 else -1


class NumaHostBuffer:
    """Anonymous host memory placed on one NUMA node (the per-NUMA pinned slab of a
    G2 pool): ``mmap`` (2 MiB huge pages when ``hugepages`` and the system has them),
    ``mbind`` to ``node`` (default: the node nearest to the current GPU), first touch,
    then - with CUDA present - page-locked and mapped for the GPU.

    ``numa_bound`` tells whether the policy was applied (containers often refuse
    ``mbind``; the memory is then placed by first touch from this thread)."""

    def __init__(self, nbytes: int, node: int | None = None, hugepages: bool = False, pin: bool | None = None):
        import mmap

        self.nbytes = int(nbytes)
        self.node = gpu_numa_node() if node is None and torch.cuda.is_available() else (-1 if node is None else node)
        flags = mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS
        self.hugepages: str | bool = False  # "hugetlb" (reserved 2 MiB pages), "thp" (transparent) or False
        mm = None
        if hugepages:
            size = (self.nbytes + (2 << 20) - 1) // (2 << 20) * (2 << 20)
            try:  # reserved huge pages (MAP_HUGETLB, Linux 0x40000)
                mm = mmap.mmap(-1, size, flags | getattr(mmap, "MAP_HUGETLB", 0x40000), mmap.PROT_READ | mmap.PROT_WRITE)
                self.hugepages = "hugetlb"
            except OSError:
                mm = mmap.mmap(-1, size, flags, mmap.PROT_READ | mmap.PROT_WRITE)
                if hasattr(mmap, "MADV_HUGEPAGE"):
                    try:  # transparent huge pages, before the first touch
                        mm.madvise(mmap.MADV_HUGEPAGE)
                        self.hugepages = "thp"
                    except OSError:
                        pass
        if mm is None:
            mm = mmap.mmap(-1, self.nbytes, flags, mmap.PROT_READ | mmap.PROT_WRITE)
        self._mm = mm
        buf = (C.c_uint8 * self.nbytes).from_buffer(mm)
        self.ptr = C.addressof(buf)
        del buf
        self.numa_bound = bind_to_numa(self.ptr, len(mm), self.node) if self.node >= 0 else False
        C.memset(self.ptr, 0, self.nbytes)  # first touch: pages are allocated under the policy
        self.pinned = torch.cuda.is_available() if pin is None else pin
        self.device_ptr = 0
        if self.pinned:
            _lib.check(_lib.load().kvbm_host_register(self.ptr, self.nbytes), "cudaHostRegister")
            d = C.c_void_p()
            _lib.check(_lib.load().kvbm_host_device_pointer(self.ptr, C.byref(d)), "cudaHostGetDevicePointer")
            self.device_ptr = int(d.value or 0)

    def tensor(self, dtype: torch.dtype = torch.uint8, shape: tuple | None = None) -> torch.Tensor:
        arr = (C.c_uint8 * self.nbytes).from_address(self.ptr)
        t = torch.frombuffer(arr, dtype=torch.uint8)
        if dtype != torch.uint8:
            t = t.view(dtype)
        return t.view(shape) if shape is not None else t

    def close(self) -> None:
        if self.ptr:
            if self.pinned:
                _lib.load().kvbm_host_unregister(self.ptr)
            self.ptr = 0
            try:
                self._mm.close()
            except BufferError:
                pass

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


@dataclass
class ExportedPool:
    """Everything a peer needs to map a pool: IPC handle, size, owner device."""

    handle: bytes
    nbytes: int
    device: int
    rank: int = 0


class SharedHostBuffer:
    """A named shared-memory file (``/dev/shm`` or a hugepage mount) mapped
    into this process. Another process on the node maps the same pool by
    path; :class:`SharedPinnedBuffer` additionally page-locks it for the GPU.
    """

    def __init__(self, name: str, nbytes: int, create: bool = True, directory: str = "/dev/shm"):
        import mmap
        import os

        self.name, self.nbytes = name, int(nbytes)
        self.path = os.path.join(directory, name)
        flags = os.O_RDWR | (os.O_CREAT if create else 0)
        fd = os.open(self.path, flags, 0o600)
        try:
            if create:
                os.ftruncate(fd, self.nbytes)
            self._mm = mmap.mmap(fd, self.nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(fd)
        self.owner = create
        if create:
            from ..utils import disk_cleanup

            disk_cleanup.register(self.path)  # unlinked if the process is told to stop
        buf = (C.c_uint8 * self.nbytes).from_buffer(self._mm)
        self.ptr = C.addressof(buf)
        del buf

    def tensor(self, dtype: torch.dtype = torch.uint8, shape: tuple | None = None) -> torch.Tensor:
        arr = (C.c_uint8 * self.nbytes).from_address(self.ptr)
        t = torch.frombuffer(arr, dtype=torch.uint8)
        if dtype != torch.uint8:
            t = t.view(dtype)
        return t.view(shape) if shape is not None else t

    def _release(self) -> None:
        pass

    def close(self) -> None:
        import os

        if self.ptr:
            self._release()
            self.ptr = 0
            try:
                self._mm.close()
            except BufferError:
                pass
            if self.owner:
                from ..utils import disk_cleanup

                disk_cleanup.deregister(self.path)
                try:
                    os.unlink(self.path)
                except FileNotFoundError:
                    pass

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class SharedPinnedBuffer(SharedHostBuffer):
    """A G2 pool in a named shared-memory file, page-locked and mapped into the
    device address space of every process that opens it.

    Any process on the node can map another instance's G2 pool by name, so a
    copy kernel can read a peer's pinned blocks directly (cross-instance
    prefix reuse without an intermediate hop). Hugepage-backed files
    (``/dev/hugepages``) work the same way.
    """

    def __init__(self, name: str, nbytes: int, create: bool = True, directory: str = "/dev/shm"):
        super().__init__(name, nbytes, create, directory)
        _lib.check(_lib.load().kvbm_host_register(self.ptr, self.nbytes), "cudaHostRegister")
        d = C.c_void_p()
        _lib.check(_lib.load().kvbm_host_device_pointer(self.ptr, C.byref(d)), "cudaHostGetDevicePointer")
        self.device_ptr = int(d.value or 0)

    def _release(self) -> None:
        _lib.load().kvbm_host_unregister(self.ptr)
