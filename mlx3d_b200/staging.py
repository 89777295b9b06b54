"""Double-buffered host-to-device staging of per-step inputs.

The reference trains from host-resident arrays (MLX unified memory); on a
discrete GPU each step's inputs must cross PCIe.  ``HostStager`` keeps two
device copies of a set of tensors and fills one on a dedicated copy stream
while the compute stream works on the other, so the copy of step k+1 runs
under the kernels of step k.  Every step still copies all of its inputs:
nothing is cached across steps.

Ordering is carried by CUDA events only (no host synchronisation):
  * the compute stream waits for the copy that filled the slot it acquires;
  * a copy into a slot waits for the compute work that last read that slot
    (recorded by :meth:`release`).
"""

from __future__ import annotations

import torch

__all__ = ["HostStager"]


class HostStager:
    def __init__(self, like: dict[str, torch.Tensor], device, requires_grad: tuple[str, ...] = ()):
        """``like`` gives the names, shapes and dtypes of the staged tensors;
        names in ``requires_grad`` are made autograd leaves on the device."""
        self.device = torch.device(device)
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.slots = []
        for _ in range(2):
            slot = {k: torch.empty(v.shape, dtype=v.dtype, device=self.device) for k, v in like.items()}
            for k in requires_grad:
                slot[k].requires_grad_(True)
            self.slots.append(slot)
        self._filled = [None, None]
        self._released = [None, None]
        self._next = 0
        self._pending: list[int] = []

    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.slots[0].values())

    def prefetch(self, host: dict[str, torch.Tensor]) -> None:
        """Queue the copy of ``host`` (pinned tensors) into the next free slot."""
        if len(self._pending) >= 2:
            raise RuntimeError("HostStager: both slots are already filled; acquire() one first")
        for k, dst in self.slots[0].items():
            if not host[k].is_pinned():
                raise ValueError(f"HostStager: host tensor {k!r} must be in pinned memory")
        i = self._next
        self._next ^= 1
        with torch.cuda.stream(self.copy_stream):
            if self._released[i] is not None:
                self.copy_stream.wait_event(self._released[i])
            with torch.no_grad():
                for k, dst in self.slots[i].items():
                    dst.copy_(host[k], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        self._filled[i] = ev
        self._pending.append(i)

    def acquire(self) -> tuple[int, dict[str, torch.Tensor]]:
        """The oldest filled slot, ordered after its copy on the current stream."""
        if not self._pending:
            raise RuntimeError("HostStager: nothing prefetched")
        i = self._pending.pop(0)
        torch.cuda.current_stream(self.device).wait_event(self._filled[i])
        return i, self.slots[i]

    def release(self, i: int) -> None:
        """Mark the current stream's work on slot ``i`` as the point after which
        the next copy into it may start."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._released[i] = ev
