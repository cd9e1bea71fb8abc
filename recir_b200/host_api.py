"""Forward+backward for callers whose tensors live in (pinned) host memory.

Sequences never interact, so a jagged batch can be streamed: the token rows are copied in as
chunks of equal size, every sequence is computed as soon as its last row has arrived, and results
leave in chunks of the same size, trailing the inputs by at most one sequence.  PCIe is full
duplex, so the two copy directions overlap with each other and with the kernels.  Three CUDA
streams (copy-in, compute, copy-out) over device buffers that hold the whole batch.

The copy chunks are cut by token count, not at sequence ends: with chunks of whole sequences the
sizes differ by the length of a sequence, and copies of unequal sizes running in both directions
at once move about a tenth less per second on PCIe than equal ones (measured: 7.97 against 7.14 ms
for 2 x 320 MB in 16 chunks).

Enqueueing the pipeline from Python costs a few hundred microseconds per chunk, which on a slow or
busy host can exceed the copy time.  So the first ``run`` on a given set of host buffers records the
whole multi-stream schedule (copies, kernels, cross-stream dependencies) into one CUDA graph, and
later calls with the same buffers replay it with a single launch; the device time is then bounded
by the PCIe copies, not by the host.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops


class HostPipeline:
    """Streams one jagged attention problem (fixed offsets / targets) through the GPU.

    ``seq_offsets`` / ``num_targets`` are host tensors.  ``run`` takes pinned host tensors
    ``q, k, v, dout`` of shape ``[T, H, D]`` and pinned host outputs ``o, dq, dk, dv``.
    """

    def __init__(self, seq_offsets: torch.Tensor, num_targets: torch.Tensor | None, heads: int, dqk: int,
                 dv: int, dtype: torch.dtype, max_seq_len: int, alpha: float, causal: bool = True,
                 contextual_seq_len: int = 0, max_attn_len: int = 0, full_attn_size: int = 0,
                 n_chunks: int = 6, device: torch.device | str = "cuda", use_graph: bool = True):
        self.device = torch.device(device)
        self.cfg = (int(max_seq_len), float(alpha), bool(causal), int(contextual_seq_len), int(max_attn_len),
                    int(full_attn_size))
        offs = seq_offsets.to(torch.int64).cpu().numpy()
        B = len(offs) - 1
        total = int(offs[-1])
        n_chunks = max(1, min(n_chunks, total))
        self.steps = plan_steps(offs, n_chunks)
        # per step: the group of whole sequences whose last row arrives with the step's rows
        self.groups = []
        for st in self.steps:
            b0, b1 = st["seqs"]
            if b1 > b0:
                local = torch.from_numpy(offs[b0:b1 + 1] - offs[b0]).to(self.device)
                nt = None if num_targets is None else num_targets[b0:b1].to(self.device)
                self.groups.append((int(offs[b0]), int(offs[b1]), local, nt))
            else:
                self.groups.append(None)
        mk = lambda d: torch.empty(total, heads, d, dtype=dtype, device=self.device)
        self.dev = dict(q=mk(dqk), k=mk(dqk), v=mk(dv), do=mk(dv), o=mk(dv), dq=mk(dqk), dk=mk(dqk), dv=mk(dv))
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream(self.device) for _ in range(3))
        self.bytes_in = total * heads * (2 * dqk + 2 * dv) * torch.empty((), dtype=dtype).element_size()
        self.bytes_out = self.bytes_in
        self.use_graph = bool(use_graph)
        self._graphs = {}  # (data pointers of the eight host tensors) -> captured schedule

    def run(self, q, k, v, dout, o, dq, dk, dv) -> None:
        """Enqueues the whole pipeline; returns once everything is queued.  The caller's current
        stream is ordered before the first copy and after the last one.  With ``use_graph`` the
        schedule is captured on the first call for a given set of host buffers (which must stay
        allocated and pinned) and replayed afterwards."""
        if not self.use_graph:
            return self._enqueue(q, k, v, dout, o, dq, dk, dv)
        key = tuple(t.data_ptr() for t in (q, k, v, dout, o, dq, dk, dv))
        g = self._graphs.get(key)
        if g is None:
            # one eager pass first: everything that initialises lazily (function attributes, the
            # allocator's pools, the context of the side streams) happens outside the capture
            self._enqueue(q, k, v, dout, o, dq, dk, dv)
            torch.cuda.current_stream(self.device).synchronize()
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(self.device)
            cap.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.graph(g, stream=cap):
                self._enqueue(q, k, v, dout, o, dq, dk, dv)
            torch.cuda.current_stream(self.device).wait_stream(cap)
            if len(self._graphs) >= 4:  # bounded: each graph keeps its workspaces alive
                self._graphs.pop(next(iter(self._graphs)))
            self._graphs[key] = g
        g.replay()

    def _enqueue(self, q, k, v, dout, o, dq, dk, dv) -> None:
        cur = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(cur)
        for st in (self.s_in, self.s_comp, self.s_out):
            st.wait_event(start)
        max_seq_len, alpha, causal, ctx, win, full = self.cfg
        d = self.dev
        for st, grp in zip(self.steps, self.groups):
            t0, t1 = st["rows_in"]
            with torch.cuda.stream(self.s_in):
                if t1 > t0:
                    for name, src in (("q", q), ("k", k), ("v", v), ("do", dout)):
                        d[name][t0:t1].copy_(src[t0:t1], non_blocking=True)
                in_done = torch.cuda.Event()
                in_done.record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(in_done)
                if grp is not None:
                    g0, g1, local, nt = grp
                    a = (local, max_seq_len, alpha, causal, nt, ctx, win, None, full)
                    ops._fwd_cuda(d["q"][g0:g1], d["k"][g0:g1], d["v"][g0:g1], *a, out=d["o"][g0:g1])
                    ops._bwd_cuda(d["do"][g0:g1], d["q"][g0:g1], d["k"][g0:g1], d["v"][g0:g1], *a,
                                  grads=(d["dq"][g0:g1], d["dk"][g0:g1], d["dv"][g0:g1]))
                comp_done = torch.cuda.Event()
                comp_done.record(self.s_comp)
            r0, r1 = st["rows_out"]
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(comp_done)
                if r1 > r0:
                    for dst, name in ((o, "o"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
                        dst[r0:r1].copy_(d[name][r0:r1], non_blocking=True)
        cur.wait_stream(self.s_out)
        cur.wait_stream(self.s_comp)
        cur.wait_stream(self.s_in)


def plan_steps(offs: np.ndarray, n_chunks: int) -> list[dict]:
    """The pipeline's schedule for sequence offsets ``offs`` (``[B + 1]``, starting at 0): a list of steps,
    each ``{"rows_in": (t0, t1), "seqs": (b0, b1), "rows_out": (r0, r1)}``.  Step ``c`` copies in rows
    ``[t0, t1)`` (``n_chunks`` pieces of equal size), computes the sequences ``[b0, b1)`` that are complete
    with those rows, and copies out rows ``[r0, r1)``.  The copy-out pieces are the copy-in pieces shifted back
    by ``lag`` rows, the largest number of rows any step leaves uncomputed behind its cut (at most the longest
    sequence): equal sizes again, except a shorter first and a longer last one, and the results trail the
    inputs by ``lag`` rows instead of a whole piece."""
    total = int(offs[-1])
    B = len(offs) - 1
    cuts = [total * c // n_chunks for c in range(n_chunks + 1)]
    ends, b_prev = [], 0
    for c in range(n_chunks):
        # sequences whose end is at or before the cut (empty sequences at the very end are swept up by the last step)
        b1 = int(np.searchsorted(offs, cuts[c + 1], side="right")) - 1
        b1 = B if c == n_chunks - 1 else max(b_prev, min(b1, B))
        ends.append(b1)
        b_prev = b1
    lag = max((cuts[c + 1] - int(offs[ends[c]]) for c in range(n_chunks - 1)), default=0)
    steps, b_prev, r_prev = [], 0, 0
    for c in range(n_chunks):
        r1 = total if c == n_chunks - 1 else max(r_prev, cuts[c + 1] - lag)
        steps.append({"rows_in": (cuts[c], cuts[c + 1]), "seqs": (b_prev, ends[c]), "rows_out": (r_prev, r1)})
        b_prev, r_prev = ends[c], r1
    return steps
