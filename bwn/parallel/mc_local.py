"""A one-GPU NVLS multicast buffer, for profiling the fused collectives in a
single process.

ncu profiles one process, and torch's symmetric memory creates no multicast
object for a one-rank group, so the ``multimem`` kernels (fused all-reduce,
sequence-parallel gather, gradient reduction) otherwise run only with every
rank of a multi-GPU group live.  This builds the object directly with the CUDA
driver API: physical memory on this GPU, a multicast object with this one
device bound to it, and two virtual mappings -- unicast (plain loads/stores,
flags) and multicast (``multimem.ld_reduce`` / ``multimem.st``).  A reduction
over a one-device object returns the local value, so the kernels run their
full code path with a world of one.  Used by ``bench/profile_fused.py
--local-mc`` only.
"""
from __future__ import annotations

import torch


def _check(res):
    err = res[0] if isinstance(res, tuple) else res
    if int(err) != 0:
        raise RuntimeError(f"CUDA driver call failed: {err}")
    return res[1] if isinstance(res, tuple) and len(res) == 2 else res


class LocalMulticastBuffer:
    def __init__(self, nbytes: int, device: torch.device):
        from cuda.bindings import driver as drv
        self._drv = drv
        torch.cuda.synchronize(device)  # the primary context is current
        ordinal = device.index if device.index is not None else torch.cuda.current_device()
        dev = _check(drv.cuDeviceGet(ordinal))
        if not _check(drv.cuDeviceGetAttribute(drv.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)):
            raise RuntimeError("this GPU has no NVLS multicast support")
        mprop = drv.CUmulticastObjectProp()
        mprop.numDevices = 1
        mprop.size = nbytes
        # a multicast object needs a shareable handle type even in one process
        # (zero is rejected as an invalid value); the bound memory requests the same
        htype = drv.CUmemAllocationHandleType.CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR
        mprop.handleTypes = htype
        gran = _check(drv.cuMulticastGetGranularity(
            mprop, drv.CUmulticastGranularity_flags.CU_MULTICAST_GRANULARITY_RECOMMENDED))
        aprop = drv.CUmemAllocationProp()
        aprop.type = drv.CUmemAllocationType.CU_MEM_ALLOCATION_TYPE_PINNED
        aprop.location.type = drv.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
        aprop.location.id = ordinal
        aprop.requestedHandleTypes = htype
        pgran = _check(drv.cuMemGetAllocationGranularity(
            aprop, drv.CUmemAllocationGranularity_flags.CU_MEM_ALLOC_GRANULARITY_RECOMMENDED))
        g = max(int(gran), int(pgran))
        size = (nbytes + g - 1) // g * g
        mprop.size = size
        self.size = size
        self.mc_handle = _check(drv.cuMulticastCreate(mprop))
        _check(drv.cuMulticastAddDevice(self.mc_handle, dev))
        self.phys = _check(drv.cuMemCreate(size, aprop, 0))
        _check(drv.cuMulticastBindMem(self.mc_handle, 0, self.phys, 0, size, 0))
        desc = drv.CUmemAccessDesc()
        desc.location.type = drv.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
        desc.location.id = ordinal
        desc.flags = drv.CUmemAccess_flags.CU_MEM_ACCESS_FLAGS_PROT_READWRITE
        self.uc = _check(drv.cuMemAddressReserve(size, g, 0, 0))
        _check(drv.cuMemMap(self.uc, size, 0, self.phys, 0))
        _check(drv.cuMemSetAccess(self.uc, size, [desc], 1))
        self.mc = _check(drv.cuMemAddressReserve(size, g, 0, 0))
        _check(drv.cuMemMap(self.mc, size, 0, self.mc_handle, 0))
        _check(drv.cuMemSetAccess(self.mc, size, [desc], 1))
        self.uc_ptr, self.mc_ptr = int(self.uc), int(self.mc)
        self.device = device
        self.tensor = torch.as_tensor(self, device=device)  # uint8 view of the unicast mapping
        self.tensor.zero_()
        torch.cuda.synchronize(device)

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.size,), "typestr": "|u1", "data": (self.uc_ptr, False), "version": 3,
                "strides": None}

    def close(self) -> None:
        drv = self._drv
        torch.cuda.synchronize(self.device)
        drv.cuMemUnmap(self.mc, self.size)
        drv.cuMemUnmap(self.uc, self.size)
        drv.cuMemAddressFree(self.mc, self.size)
        drv.cuMemAddressFree(self.uc, self.size)
        drv.cuMulticastUnbind(self.mc_handle, _check(drv.cuDeviceGet(self.device.index or 0)), 0, self.size)
        drv.cuMemRelease(self.phys)
        drv.cuMemRelease(self.mc_handle)
