"""KV cache codes reserved in virtual memory and backed block by block.

A layer's K or V codes are laid out [Hkv, C, words] (head-major, so that a
256-token block of one head is one contiguous run for the kernels' bulk
copies).  Growing C in place would move every head but the first, so the
reference appends separate 65,536-token bank blocks instead
(engine/src/rec_mlx/cache.py:47-84) and its kernel indexes the block of each
token.  Here the whole final capacity C is reserved as one virtual address
range (cuMemAddressReserve), and physical memory is created and mapped for
each head's rows one 32,768-token block at a time as the context grows
(cuMemCreate / cuMemMap / cuMemSetAccess).  The kernels keep their flat
[Hkv, C, words] addressing with C as the head stride, no row already written
moves or is copied, and memory is committed only for the blocks in use.
The library is told how many rows are backed (rec_set_kv_rows) and refuses
positions beyond them.

Only the codes are reserved this way (94 % of the cache at 8 bits, 89 % at
4 bits); the bf16 scales and biases (4 bytes per token and head each) are
ordinary allocations of the final capacity.
"""
from __future__ import annotations

import torch

BLOCK_TOKENS = 32768  # rows mapped per growth step (4 MB per head at 8 bits, 2 MB at 4 bits)


def _driver():
    from cuda.bindings import driver as cu

    return cu


def _ok(res, what: str):
    """Unpacks a cuda.bindings result tuple, raising on an error code."""
    cu = _driver()
    err = res[0] if isinstance(res, tuple) else res
    if err != cu.CUresult.CUDA_SUCCESS:
        raise RuntimeError(f"{what} failed: {err}")
    if isinstance(res, tuple):
        return res[1] if len(res) == 2 else res[1:]
    return None


class _View:
    """__cuda_array_interface__ of a strided int32 view (no ownership)."""

    def __init__(self, ptr: int, shape, strides_bytes):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i4", "data": (int(ptr), False),
                                         "version": 3, "strides": tuple(strides_bytes)}


class ReservedCodes:
    """One [heads, capacity, words] int32 tensor of KV codes whose rows are
    backed on demand.  `view()` covers the backed rows only (head stride =
    capacity), so nothing can touch unmapped memory through it."""

    def __init__(self, heads: int, capacity: int, words: int, device: torch.device):
        if capacity % BLOCK_TOKENS:
            raise ValueError(f"reserved capacity must be a multiple of {BLOCK_TOKENS}")
        cu = _driver()
        self.heads, self.capacity, self.words = heads, capacity, words
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.row_bytes = words * 4
        self.block_bytes = BLOCK_TOKENS * self.row_bytes
        torch.cuda.set_device(self.device)
        torch.zeros(1, device=self.device)  # the primary context is current on this thread
        prop = cu.CUmemAllocationProp()
        prop.type = cu.CUmemAllocationType.CU_MEM_ALLOCATION_TYPE_PINNED
        prop.location.type = cu.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
        prop.location.id = self.device.index
        self._prop = prop
        gran = int(_ok(cu.cuMemGetAllocationGranularity(
            prop, cu.CUmemAllocationGranularity_flags.CU_MEM_ALLOC_GRANULARITY_MINIMUM), "granularity"))
        if self.block_bytes % gran:
            raise ValueError(f"a block of {self.block_bytes} bytes is not a multiple of the granularity {gran}")
        self.total = heads * capacity * self.row_bytes
        self.base = int(_ok(cu.cuMemAddressReserve(self.total, gran, 0, 0), "cuMemAddressReserve"))
        self._handles = []  # (va, size, handle)
        self.rows = 0
        acc = cu.CUmemAccessDesc()
        acc.location = prop.location
        acc.flags = cu.CUmemAccess_flags.CU_MEM_ACCESS_FLAGS_PROT_READWRITE
        self._access = acc

    def grow(self, rows: int) -> None:
        """Backs rows [0, rows) (rounded up to whole blocks) of every head.
        New rows are not cleared: every row is written (quantize-on-append)
        before attention reads it, and the kernels mask the rows of a
        partly filled 4-row group by position, never by their contents."""
        cu = _driver()
        need = -(-rows // BLOCK_TOKENS) * BLOCK_TOKENS
        if need > self.capacity:
            raise ValueError(f"{rows} rows exceed the reserved capacity {self.capacity}")
        while self.rows < need:
            b = self.rows // BLOCK_TOKENS
            for h in range(self.heads):
                va = self.base + (h * self.capacity + b * BLOCK_TOKENS) * self.row_bytes
                handle = _ok(cu.cuMemCreate(self.block_bytes, self._prop, 0), "cuMemCreate")
                try:
                    _ok(cu.cuMemMap(va, self.block_bytes, 0, handle, 0), "cuMemMap")
                except Exception:
                    cu.cuMemRelease(handle)
                    raise
                self._handles.append((va, self.block_bytes, handle))
                _ok(cu.cuMemSetAccess(va, self.block_bytes, [self._access], 1), "cuMemSetAccess")
            self.rows += BLOCK_TOKENS

    def view(self) -> torch.Tensor:
        """int32 [heads, rows, words] over the backed rows (head stride =
        capacity rows)."""
        v = _View(self.base, (self.heads, self.rows, self.words),
                  (self.capacity * self.row_bytes, self.row_bytes, 4))
        t = torch.as_tensor(v, device=self.device)
        t._reserved_owner = self  # keeps the mapping alive as long as a view exists
        return t

    def release(self) -> None:
        cu = _driver()
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        for va, size, handle in self._handles:
            cu.cuMemUnmap(va, size)
            cu.cuMemRelease(handle)
        self._handles = []
        cu.cuMemAddressFree(self.base, self.total)
        self.base = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass
