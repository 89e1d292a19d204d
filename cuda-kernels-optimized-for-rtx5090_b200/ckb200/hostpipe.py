"""Host-resident batches through a device op with the copies overlapped.

The batch's tensors share a leading dim (rows, tokens) and are cut along it into chunks. Each chunk moves host ->
device on one stream, runs the op on a second and moves device -> host on a third, so the two copy directions
(separate copy engines, full duplex over the host link) and the kernels overlap across chunks and across calls.
Every call still moves every input in and every output back. The device buffers belong to the pipeline, one slot
per chunk. A slot's inputs are refilled only after the previous call's op on that slot has finished, and its outputs
are rewritten only after the previous call's copy-out has finished (events, no host synchronisation).

    pipe = RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), rows, cols, torch.bfloat16)
    pipe(hx, hy)          # asynchronous; hx, hy pinned host tensors [rows, cols]
    pipe.synchronize()    # hy now holds the result

    pipe = Pipeline(op, [((tokens, 32, 128), torch.bfloat16), ((tokens,), torch.int64)],
                    [((tokens, 32, 128), torch.bfloat16)])
    pipe([hq, hids], [hq_out])   # op(ins, outs) gets the chunk's device views, in the order given

Work the caller queued on its current stream before a call (writes to tensors the op reads, say) is waited for. The
host outputs are valid only after synchronize(), or after an event recorded by record_end() has completed.
"""

import torch


class Pipeline:
    def __init__(self, op, inputs, outputs, chunks=8, device=None):
        """op(ins, outs) runs on the current stream and writes the device views `outs` (one per entry of `outputs`)
        from `ins` (one per entry of `inputs`), chunk by chunk along the leading dim.

        inputs, outputs: lists of (shape, dtype); every shape has the same leading dim n >= 1. chunks is the number
        of chunks (at most n); device defaults to the current CUDA device.
        """
        if not inputs or not outputs:
            raise ValueError("Pipeline: needs at least one input and one output")
        lead = {tuple(s)[0] if len(s) else None for s, _ in list(inputs) + list(outputs)}
        if len(lead) != 1 or None in lead or min(lead) < 1:
            raise ValueError(f"Pipeline: shapes must share a leading dim >= 1, got {inputs} -> {outputs}")
        if chunks < 1:
            raise ValueError(f"Pipeline: chunks {chunks}")
        n = lead.pop()
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.op = op
        self.in_specs = [(tuple(s), d) for s, d in inputs]
        self.out_specs = [(tuple(s), d) for s, d in outputs]
        chunks = min(chunks, n)
        step = (n + chunks - 1) // chunks
        self.bounds = [(a, min(a + step, n)) for a in range(0, n, step)]
        with torch.cuda.device(self.device):
            self.ins = [torch.empty(s, dtype=d, device=self.device) for s, d in self.in_specs]
            self.outs = [torch.empty(s, dtype=d, device=self.device) for s, d in self.out_specs]
            self.h2d, self.comp, self.d2h = (torch.cuda.Stream(self.device) for _ in range(3))
        k = len(self.bounds)
        self.in_ready = [torch.cuda.Event() for _ in range(k)]
        self.op_done = [torch.cuda.Event() for _ in range(k)]
        self.out_done = [torch.cuda.Event() for _ in range(k)]

    @staticmethod
    def _check_host(ts, specs, what):
        if len(ts) != len(specs):
            raise ValueError(f"Pipeline: {len(specs)} {what} tensors expected, got {len(ts)}")
        for t, (shape, dtype) in zip(ts, specs):
            if t.device.type != "cpu" or tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous():
                raise ValueError(f"Pipeline: {what} must be contiguous host tensors {shape} of {dtype}")
            if not t.is_pinned():
                raise ValueError(f"Pipeline: {what} must be in pinned host memory")

    def __call__(self, host_ins, host_outs):
        """Queues host_ins -> op -> host_outs for every chunk; returns host_outs (valid after synchronize())."""
        self._check_host(host_ins, self.in_specs, "input")
        self._check_host(host_outs, self.out_specs, "output")
        with torch.cuda.device(self.device):
            caller = torch.cuda.current_stream(self.device)
            self.h2d.wait_stream(caller)
            self.comp.wait_stream(caller)
            for j, (a, b) in enumerate(self.bounds):
                with torch.cuda.stream(self.h2d):
                    self.h2d.wait_event(self.op_done[j])  # the previous call's op has read this input slot
                    for dev, host in zip(self.ins, host_ins):
                        dev[a:b].copy_(host[a:b], non_blocking=True)
                    self.in_ready[j].record(self.h2d)
                with torch.cuda.stream(self.comp):
                    self.comp.wait_event(self.in_ready[j])
                    self.comp.wait_event(self.out_done[j])  # the previous call's copy-out has read this output slot
                    self.op([t[a:b] for t in self.ins], [t[a:b] for t in self.outs])
                    self.op_done[j].record(self.comp)
                with torch.cuda.stream(self.d2h):
                    self.d2h.wait_event(self.op_done[j])
                    for dev, host in zip(self.outs, host_outs):
                        host[a:b].copy_(dev[a:b], non_blocking=True)
                    self.out_done[j].record(self.d2h)
        return host_outs

    def bytes_per_call(self):
        """(host -> device, device -> host) bytes one call copies."""
        size = lambda specs: sum(torch.empty(0, dtype=d).element_size() * _numel(s) for s, d in specs)  # noqa: E731
        return size(self.in_specs), size(self.out_specs)

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


def _numel(shape):
    n = 1
    for d in shape:
        n *= d
    return n


class RowPipeline(Pipeline):
    """A Pipeline of one [rows, cols] input and one [rows, cols] output: op(x_chunk, y_chunk)."""

    def __init__(self, op, rows, cols, dtype, out_dtype=None, chunks=8, device=None):
        if rows < 1 or cols < 1:
            raise ValueError(f"RowPipeline: shape ({rows}, {cols})")
        out_dtype = dtype if out_dtype is None else out_dtype
        super().__init__(lambda ins, outs: op(ins[0], outs[0]), [((rows, cols), dtype)],
                         [((rows, cols), out_dtype)], chunks=chunks, device=device)
        self.shape = (rows, cols)
        self.dtype, self.out_dtype = dtype, out_dtype
        self.x, self.y = self.ins[0], self.outs[0]

    def __call__(self, hx, hy):
        """Queues hx -> op -> hy for every chunk; returns hy (valid after synchronize()). hx and hy may also be
        given as one-element lists, as Pipeline takes them."""
        if isinstance(hx, (list, tuple)):
            return super().__call__(list(hx), list(hy))
        super().__call__([hx], [hy])
        return hy
