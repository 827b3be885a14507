"""Host K/V slab: geometry, strict head-wise bookkeeping, pinned + mapped storage.

Geometry and bookkeeping follow SlabGeometry / SequentialCacheState
(hi/slab_cache.py:37-120): one flat slab [2 (K|V)][entries][max_len][D],
entry = layer * kv_heads + kv_head, entries updated in strict sequential order.
The storage is pinned host memory mapped into the device address space
(cudaHostAllocMapped), so kernels read selected rows straight over the host
link (the reference maps its pin_memory slab the same way for its zero-copy
path, hi/resident_zero_copy.py:15-29).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib


@dataclass(frozen=True)
class SlabGeometry:
    """Pure layout arithmetic (hi/slab_cache.py:37-74), CUDA-independent."""

    num_entries: int
    batch_size: int
    max_cache_len: int
    head_dim: int

    def __post_init__(self) -> None:
        for name, value in (("num_entries", self.num_entries), ("batch_size", self.batch_size),
                            ("max_cache_len", self.max_cache_len), ("head_dim", self.head_dim)):
            if value <= 0:
                raise ValueError(f"{name} must be positive, got {value}")

    @property
    def elements_per_entry(self) -> int:
        return self.batch_size * self.max_cache_len * self.head_dim

    @property
    def total_elements(self) -> int:
        return 2 * self.num_entries * self.elements_per_entry

    def bounds(self, kind: str, entry_idx: int) -> tuple[int, int]:
        if kind not in {"key", "value"}:
            raise ValueError(f"kind must be 'key' or 'value', got {kind!r}")
        if not 0 <= entry_idx < self.num_entries:
            raise IndexError(f"entry_idx {entry_idx} outside [0, {self.num_entries})")
        plane = 0 if kind == "key" else self.num_entries
        start = (plane + entry_idx) * self.elements_per_entry
        return start, start + self.elements_per_entry

    def tensor_shape(self) -> tuple[int, int, int, int]:
        return (self.batch_size, 1, self.max_cache_len, self.head_dim)


class SequentialCacheState:
    """Strict head-wise update order and logical lengths (hi/slab_cache.py:77-120)."""

    def __init__(self, num_entries: int, allocated_capacity: int) -> None:
        if num_entries <= 0 or allocated_capacity <= 0:
            raise ValueError("num_entries and allocated_capacity must be positive")
        self.num_entries = num_entries
        self.allocated_capacity = allocated_capacity
        self.logical_lengths = [0] * num_entries
        self.expected_next_entry = 0
        self.write_position = 0
        self.seen_tokens = 0

    def preview(self, entry_idx: int, append_length: int) -> tuple[int, int]:
        if entry_idx != self.expected_next_entry:
            raise ValueError("strict sequential head-wise update violated: "
                             f"expected {self.expected_next_entry}, got {entry_idx}")
        if append_length <= 0:
            raise ValueError("append_length must be positive")
        old_length = self.logical_lengths[entry_idx]
        new_length = old_length + append_length
        if new_length > self.allocated_capacity:
            raise RuntimeError(f"cache capacity exceeded: {old_length} + {append_length} > "
                               f"{self.allocated_capacity}")
        return old_length, new_length

    def advance(self, entry_idx: int, append_length: int) -> tuple[int, int]:
        old_length, new_length = self.preview(entry_idx, append_length)
        self.write_position = old_length
        self.logical_lengths[entry_idx] = new_length
        if entry_idx == 0:
            self.seen_tokens += append_length
        self.expected_next_entry = (entry_idx + 1) % self.num_entries
        return old_length, new_length

    def check_block(self, first: int, count: int) -> int:
        """The checks of advance(e, 1) for e = first .. first + count - 1 in order,
        for entries of one logical length; returns that old length."""
        if first != self.expected_next_entry:
            raise ValueError("strict sequential head-wise update violated: "
                             f"expected {self.expected_next_entry}, got {first}")
        lengths = self.logical_lengths
        old_length = lengths[first]
        if first + count > self.num_entries or lengths[first:first + count].count(old_length) != count:
            raise AssertionError("layer KV entries have unequal logical lengths")
        if old_length + 1 > self.allocated_capacity:
            raise RuntimeError(f"cache capacity exceeded: {old_length} + 1 > "
                               f"{self.allocated_capacity}")
        return old_length

    def commit_block(self, first: int, count: int, old_length: int) -> None:
        """The updates of advance(e, 1) for the block check_block accepted."""
        lengths = self.logical_lengths
        lengths[first:first + count] = [old_length + 1] * count
        self.write_position = old_length
        if first == 0:
            self.seen_tokens += 1
        self.expected_next_entry = (first + count) % self.num_entries

    def advance_block(self, first: int, count: int) -> int:
        old_length = self.check_block(first, count)
        self.commit_block(first, count, old_length)
        return old_length

    @property
    def uniform(self) -> bool:
        return len(set(self.logical_lengths)) == 1


class MappedHostSlab:
    """Pinned, device-mapped host allocation viewed as a torch CPU tensor.

    ``host`` is a CPU tensor over the pinned pages; ``device_ptr`` is the address
    kernels use.  Freed with ``close()`` (or when garbage collected)."""

    def __init__(self, geometry: SlabGeometry, dtype: torch.dtype,
                 numa_node: int | str | None = None) -> None:
        """numa_node: None = cudaHostAlloc's default placement; "auto" = the host
        NUMA node closest to the current GPU; an int = that node."""
        self.geometry = geometry
        self.dtype = dtype
        itemsize = torch.tensor([], dtype=dtype).element_size()
        self.nbytes = geometry.total_elements * itemsize
        lib = _lib.load()
        host = ctypes.c_void_p()
        dev = ctypes.c_void_p()
        self.numa_node: int | None = None
        if numa_node is None:
            _lib.check(lib.tw_host_alloc_mapped(self.nbytes, ctypes.byref(host), ctypes.byref(dev)),
                       "tw_host_alloc_mapped")
        else:
            want = -1 if numa_node == "auto" else int(numa_node)
            bound = ctypes.c_int32(-1)
            _lib.check(lib.tw_host_alloc_mapped_numa(self.nbytes, want, ctypes.byref(host),
                                                     ctypes.byref(dev), ctypes.byref(bound)),
                       "tw_host_alloc_mapped_numa")
            self.numa_node = bound.value if bound.value >= 0 else None
        self._host_ptr = host.value
        self.device_ptr = dev.value
        buf = (ctypes.c_uint8 * self.nbytes).from_address(self._host_ptr)
        self._buf = buf
        self.host = torch.frombuffer(buf, dtype=torch.uint8).view(dtype)
        self.rows = self.host.view(2, geometry.num_entries, geometry.max_cache_len,
                                   geometry.head_dim)

    def page_node(self, offset: int = 0) -> int | None:
        """Host NUMA node of the page holding byte `offset` of the slab, if known."""
        if not getattr(self, "_host_ptr", None):
            raise RuntimeError("the slab has been freed")
        node = ctypes.c_int32(-1)
        st = _lib.load().tw_host_numa_node(ctypes.c_void_p(self._host_ptr + offset), ctypes.byref(node))
        return node.value if st == _lib.TW_OK and node.value >= 0 else None

    @property
    def key_device_ptr(self) -> int:
        return self.device_ptr

    @property
    def value_device_ptr(self) -> int:
        half = self.nbytes // 2
        return self.device_ptr + half

    def entry(self, kind: str, entry: int) -> torch.Tensor:
        """[1, 1, max_len, D] host view of one entry (the reference's _host_tensor)."""
        start, end = self.geometry.bounds(kind, entry)
        return self.host[start:end].view(self.geometry.tensor_shape())

    def close(self) -> None:
        if getattr(self, "_host_ptr", None):
            self.host = None
            self.rows = None
            self._buf = None
            _lib.load().tw_host_free(self._host_ptr)
            self._host_ptr = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
