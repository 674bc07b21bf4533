"""Borrowed view of the reusable decode output (mirrors ``src/seoulkv4/result.py:12-38``)."""

from __future__ import annotations

import weakref

import torch

from seoulkv_b200 import _native


class _DeviceBuffer:
    """Exposes a raw device pointer to torch via ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape, stream: int):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": "<i2", "data": (ptr, False), "version": 3,
            "strides": None, "stream": stream or 1,
        }


class DecodeResult:
    """Output of one run, valid until the next run or close of its owner."""

    def __init__(self, owner, generation: int):
        self._owner_ref = weakref.ref(owner)
        self._generation = generation

    def _owner(self):
        owner = self._owner_ref()
        if owner is None or owner._closed or owner._generation != self._generation:
            raise RuntimeError("SeoulKV4 result is no longer live; read back before the next run or close")
        return owner

    @property
    def device_tensors(self) -> tuple:
        """Four borrowed CUDA BF16 tensors [1, 4, 256], one per KV group (query heads 4g..4g+3)."""
        owner = self._owner()
        eng = owner._require_initialized()
        base = torch.as_tensor(_DeviceBuffer(eng.output_device_ptr(), (16, 256), owner._stream()),
                               device=f"cuda:{owner._device_index}").view(torch.bfloat16)
        return tuple(base[4 * g:4 * g + 4].unsqueeze(0) for g in range(4))

    def to_torch(self) -> torch.Tensor:
        """Synchronise and copy the output into a CPU BF16 tensor [1, 1, 16, 256]
        (RuntimeError if a live count left its range, as ``synchronize``)."""
        owner = self._owner()
        eng = owner._require_initialized()
        # the engine writes its n_slots (one for SeoulKV4) outputs straight
        # into the returned tensor's storage
        y = torch.empty((eng.n_slots, 1, 16, 256), dtype=torch.bfloat16)
        try:
            eng.finish_to(y.data_ptr())  # wait, status check and output copy in one native call
        except _native.NativeError as exc:
            raise RuntimeError(str(exc)) from exc
        return y if eng.n_slots == 1 else y[:1]
