"""Cross-rank device timeline of the wavefront (diagnostic; no counterpart in
the reference).

``Timeline.mark(label)`` enqueues ``wf_stamp`` on the current stream: a
one-thread kernel that writes the GPU's %globaltimer (ns) when the stream
reaches it.  The engine marks each tick's phases and the paged transport
marks every layer's entry and every remote flag wait, so the stamps show when
each rank's stream got where, with no profiler attached.  ``align()`` stamps
right after a world all_reduce: every rank leaves that collective within
microseconds, so subtracting each rank's own alignment stamp puts all ranks on
one time axis even if their timers are offset.
"""

from __future__ import annotations

import torch

from waveforcing_b200 import _lib as L


class Timeline:
    def __init__(self, device, capacity: int = 1 << 16) -> None:
        self.device = torch.device(device)
        self.buf = torch.zeros(capacity, dtype=torch.int64, device=self.device)
        self.labels: list[str] = []

    def mark(self, label: str) -> None:
        i = len(self.labels)
        if i >= self.buf.numel():
            return
        self.labels.append(label)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        L.check(L.lib().wf_stamp(self.buf.data_ptr() + 8 * i, stream), "wf_stamp")

    def align(self, group=None) -> None:
        """A world all_reduce, then a stamp labelled ``align`` on every rank."""
        import torch.distributed as dist

        x = torch.zeros(1, device=self.device)
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(x, group=group)
        self.mark("align")

    def rows(self) -> list[tuple[str, float]]:
        """(label, microseconds after this rank's last ``align`` stamp)."""
        torch.cuda.synchronize(self.device)
        ts = self.buf[: len(self.labels)].cpu().tolist()
        t0 = next((t for lab, t in zip(reversed(self.labels), reversed(ts)) if lab == "align"), ts[0] if ts else 0)
        return [(lab, (t - t0) / 1e3) for lab, t in zip(self.labels, ts)]
