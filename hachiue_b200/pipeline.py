"""Host-fed steps with their copies overlapped: the serving-loop form of the
decode path.

A decode step of the reference reads its inputs from host memory and writes
its logits back (forwardSegment's one readback per call, src/engine.ts:1489,
:1520-1528); every step pays a host-to-device copy before its kernels and a
device-to-host copy after them.  ``HostPipeline`` runs such steps with two
buffer slots and three CUDA streams, ordered by events: the host-to-device
copies of step i+1 and the device-to-host copy of step i-1 run on their own
streams while step i's kernels run on the caller's current stream.  Per slot:

  * its input copy waits until the slot's previous step no longer reads them;
  * its kernels wait for its input copy and for the slot's previous output copy;
  * its output copy waits for its kernels.

Inputs must be pinned host tensors (otherwise the copies are synchronous).
The device buffers are allocated once, at construction.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    def __init__(self, device, inputs: Sequence[tuple[tuple[int, ...], torch.dtype]],
                 outputs: Sequence[tuple[tuple[int, ...], torch.dtype]], slots: int = 2):
        self.device = torch.device(device)
        self.slots = slots
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.dev_in = [[torch.empty(s, dtype=d, device=self.device) for s, d in inputs] for _ in range(slots)]
        self.dev_out = [[torch.empty(s, dtype=d, device=self.device) for s, d in outputs] for _ in range(slots)]
        self.ev_h2d = [torch.cuda.Event() for _ in range(slots)]
        self.ev_compute = [torch.cuda.Event() for _ in range(slots)]
        self.ev_d2h = [torch.cuda.Event() for _ in range(slots)]
        self.used = [False] * slots
        self.i = 0

    def begin(self) -> None:
        """Orders the copy streams after the work already queued on the current
        stream (e.g. a timing event), so the next steps' copies start after it."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.h2d.wait_event(ev)
        self.d2h.wait_event(ev)

    def submit(self, host_in: Sequence[torch.Tensor], host_out: Sequence[torch.Tensor],
               compute: Callable[[list, list], None]) -> None:
        """Enqueues one step: copy ``host_in`` into the slot's device inputs,
        ``compute(device_inputs, device_outputs)`` on the current stream, copy
        the device outputs into ``host_out``.  Returns without waiting."""
        j = self.i % self.slots
        cur = torch.cuda.current_stream(self.device)
        if self.used[j]:
            self.h2d.wait_event(self.ev_compute[j])
        with torch.cuda.stream(self.h2d):
            for d, h in zip(self.dev_in[j], host_in):
                d.copy_(h, non_blocking=True)
            self.ev_h2d[j].record(self.h2d)
        cur.wait_event(self.ev_h2d[j])
        if self.used[j]:
            cur.wait_event(self.ev_d2h[j])
        compute(self.dev_in[j], self.dev_out[j])
        self.ev_compute[j].record(cur)
        self.d2h.wait_event(self.ev_compute[j])
        with torch.cuda.stream(self.d2h):
            for h, d in zip(host_out, self.dev_out[j]):
                h.copy_(d, non_blocking=True)
            self.ev_d2h[j].record(self.d2h)
        self.used[j] = True
        self.i += 1

    def drain(self) -> None:
        """Makes the current stream wait for every output copy submitted so far."""
        cur = torch.cuda.current_stream(self.device)
        for j in range(self.slots):
            if self.used[j]:
                cur.wait_event(self.ev_d2h[j])
