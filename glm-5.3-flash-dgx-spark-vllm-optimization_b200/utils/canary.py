"""Guard bands around scratch buffers: the memory half of the bounds-checked debug build.

With ``GLM53_BOUNDS=1`` every buffer allocated through :class:`Scratch` sits between two 256-byte guard bands
filled with a fixed byte (0xA5).  A kernel that writes past either end of its buffer changes a band;
:meth:`Scratch.check` compares the bands and names the buffers whose bands changed.  The kernels of that build
also check the indices they read from device data (``glm53_C_bounds``: ``bounds_status()``), so the two together
stand in for a memory checker on machines where none can run.  In the regular build the allocator returns plain
``torch.zeros`` tensors: no bands, no cost.

The bands keep the buffer 256-byte aligned (the caching allocator's blocks are 512-byte aligned), so kernels that
need 16-byte or 128-byte alignment of their operands see the same alignment as in the regular build.
"""

from __future__ import annotations

import math
import os
import weakref

import torch

GUARD = 256
FILL = 0xA5
ENABLED = os.environ.get("GLM53_BOUNDS", "0") == "1"

_live: "weakref.WeakSet[Scratch]" = weakref.WeakSet()


class Scratch:
    """Allocator of guarded scratch buffers for one owner (a Runtime).

    ``zeros(*shape, dtype=...)`` returns a zero-filled tensor; with guards enabled it is a view into a larger byte
    buffer whose first and last ``GUARD`` bytes hold ``FILL``.
    """

    def __init__(self, device, enabled: bool | None = None):
        self.device = torch.device(device)
        self.enabled = ENABLED if enabled is None else bool(enabled)
        self._bands: list[tuple[torch.Tensor, int, int]] = []   # raw bytes, payload bytes, payload data_ptr
        self._owner = None
        _live.add(self)

    def attach(self, owner) -> None:
        """Name buffers after the owner's attributes in reports (weakly: the owner is not kept alive)."""
        self._owner = weakref.ref(owner)

    def zeros(self, *shape, dtype: torch.dtype, device=None) -> torch.Tensor:
        if len(shape) == 1 and isinstance(shape[0], (tuple, list, torch.Size)):
            shape = tuple(shape[0])
        dev = self.device if device is None else torch.device(device)
        if not self.enabled:
            return torch.zeros(*shape, dtype=dtype, device=dev)
        nb = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        raw = torch.full((nb + 2 * GUARD,), FILL, dtype=torch.uint8, device=dev)
        body = raw[GUARD:GUARD + nb]
        body.zero_()
        out = body.view(dtype).view(shape)
        self._bands.append((raw, nb, out.data_ptr()))
        return out

    def __len__(self) -> int:
        return len(self._bands)

    def _names(self) -> dict[int, str]:
        owner = self._owner() if self._owner is not None else None
        names: dict[int, str] = {}
        if owner is None:
            return names
        for k, v in vars(owner).items():
            if isinstance(v, torch.Tensor):
                names.setdefault(v.data_ptr(), k)
            elif isinstance(v, (list, tuple)):
                for i, t in enumerate(v):
                    if isinstance(t, torch.Tensor):
                        names.setdefault(t.data_ptr(), f"{k}[{i}]")
        return names

    def check(self) -> list[str]:
        """Names of the buffers whose guard bands changed (empty: all intact, or guards disabled)."""
        if not self._bands:
            return []
        flags = torch.stack([(raw[:GUARD] != FILL).any() | (raw[GUARD + nb:] != FILL).any()
                             for raw, nb, _ in self._bands]).cpu()
        if not bool(flags.any()):
            return []
        names = self._names()
        return [names.get(ptr, f"buffer@{ptr:#x}") for (_, _, ptr), bad in zip(self._bands, flags.tolist()) if bad]


def check_all() -> list[str]:
    """Guard-band failures of every live Scratch allocator."""
    bad: list[str] = []
    for s in list(_live):
        bad += s.check()
    return bad
