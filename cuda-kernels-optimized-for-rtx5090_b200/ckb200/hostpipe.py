"""Host-resident batches through a row-wise op with the copies overlapped.

The rows of a pinned host batch are cut into chunks. Each chunk moves host -> device on one stream, runs the op on a
second and moves device -> host on a third, so the two copy directions (separate copy engines, full duplex over the
host link) and the kernels overlap across chunks and across calls. Every call still moves the whole input in and
the whole output back. The device buffers belong to the pipeline, one slot per chunk. A slot's input is refilled
only after the previous call's op on that slot has finished, and its output is rewritten only after the previous
call's copy-out has finished (events, no host synchronisation).

    pipe = RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), rows, cols, torch.bfloat16)
    pipe(hx, hy)          # asynchronous; hx, hy pinned host tensors [rows, cols]
    pipe.synchronize()    # hy now holds the result
"""

import torch


class RowPipeline:
    def __init__(self, op, rows, cols, dtype, out_dtype=None, chunks=8, device=None):
        """op(x_chunk, y_chunk) runs on the current stream and writes y_chunk from x_chunk (row-wise).

        rows, cols, dtype describe the input batch; out_dtype defaults to dtype; chunks is the number of row
        chunks (at most rows); device defaults to the current CUDA device.
        """
        if rows < 1 or cols < 1:
            raise ValueError(f"RowPipeline: shape ({rows}, {cols})")
        if chunks < 1:
            raise ValueError(f"RowPipeline: chunks {chunks}")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.op = op
        self.shape = (rows, cols)
        self.dtype = dtype
        self.out_dtype = dtype if out_dtype is None else out_dtype
        chunks = min(chunks, rows)
        step = (rows + chunks - 1) // chunks
        self.bounds = [(a, min(a + step, rows)) for a in range(0, rows, step)]
        with torch.cuda.device(self.device):
            self.x = torch.empty(rows, cols, dtype=dtype, device=self.device)
            self.y = torch.empty(rows, cols, dtype=self.out_dtype, device=self.device)
            self.h2d, self.comp, self.d2h = (torch.cuda.Stream(self.device) for _ in range(3))
        n = len(self.bounds)
        self.in_ready = [torch.cuda.Event() for _ in range(n)]
        self.op_done = [torch.cuda.Event() for _ in range(n)]
        self.out_done = [torch.cuda.Event() for _ in range(n)]

    def _check_host(self, t, dtype, what):
        if t.device.type != "cpu" or tuple(t.shape) != self.shape or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"RowPipeline: {what} must be a contiguous host tensor {self.shape} of {dtype}")
        if not t.is_pinned():
            raise ValueError(f"RowPipeline: {what} must be in pinned host memory")

    def __call__(self, hx, hy):
        """Queues hx -> op -> hy for every chunk; returns hy (valid after synchronize())."""
        self._check_host(hx, self.dtype, "input")
        self._check_host(hy, self.out_dtype, "output")
        with torch.cuda.device(self.device):
            for j, (a, b) in enumerate(self.bounds):
                with torch.cuda.stream(self.h2d):
                    self.h2d.wait_event(self.op_done[j])  # the previous call's op has read this input slot
                    self.x[a:b].copy_(hx[a:b], non_blocking=True)
                    self.in_ready[j].record(self.h2d)
                with torch.cuda.stream(self.comp):
                    self.comp.wait_event(self.in_ready[j])
                    self.comp.wait_event(self.out_done[j])  # the previous call's copy-out has read this output slot
                    self.op(self.x[a:b], self.y[a:b])
                    self.op_done[j].record(self.comp)
                with torch.cuda.stream(self.d2h):
                    self.d2h.wait_event(self.op_done[j])
                    hy[a:b].copy_(self.y[a:b], non_blocking=True)
                    self.out_done[j].record(self.d2h)
        return hy

    def record_start(self, event):
        """Records `event` on the copy-in stream after all queued work: a timing start for the next calls."""
        with torch.cuda.device(self.device):
            self.h2d.wait_stream(self.d2h)
            self.h2d.wait_stream(self.comp)
            event.record(self.h2d)

    def record_end(self, event):
        """Records `event` on the copy-out stream after every queued chunk (a timing end)."""
        with torch.cuda.device(self.device):
            self.d2h.wait_stream(self.comp)
            self.d2h.wait_stream(self.h2d)
            event.record(self.d2h)

    def synchronize(self):
        for s in (self.h2d, self.comp, self.d2h):
            s.synchronize()
