"""Forward+backward for callers whose tensors live in (pinned) host memory.

Sequences never interact, so a jagged batch can be cut into chunks of whole sequences and
streamed: while chunk ``c`` is computed, chunk ``c+1`` is copied in and the results of
chunk ``c-1`` are copied out.  PCIe is full duplex, so the two copy directions overlap as
well.  Three CUDA streams (copy-in, compute, copy-out) and two device buffer slots.

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
        n_chunks = max(1, min(n_chunks, B))
        # contiguous groups of whole sequences with about equal token counts
        bounds = [0]
        for c in range(1, n_chunks):
            target = total * c / n_chunks
            b = int(np.searchsorted(offs, target, side="left"))
            bounds.append(min(max(b, bounds[-1] + 1), B - (n_chunks - c)))
        bounds.append(B)
        self.chunks = []
        max_tokens = 0
        for c in range(n_chunks):
            b0, b1 = bounds[c], bounds[c + 1]
            t0, t1 = int(offs[b0]), int(offs[b1])
            local = torch.from_numpy(offs[b0:b1 + 1] - offs[b0]).to(self.device)
            nt = None if num_targets is None else num_targets[b0:b1].to(self.device)
            self.chunks.append((t0, t1, local, nt))
            max_tokens = max(max_tokens, t1 - t0)
        mk = lambda d: torch.empty(max_tokens, heads, d, dtype=dtype, device=self.device)
        self.slots = [dict(q=mk(dqk), k=mk(dqk), v=mk(dv), do=mk(dv)) for _ in range(2)]
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
            return self._enqueue(q, k, v, dout, o, dq, dk, dv, record_streams=True)
        key = tuple(t.data_ptr() for t in (q, k, v, dout, o, dq, dk, dv))
        g = self._graphs.get(key)
        if g is None:
            # one eager pass first: everything that initialises lazily (function attributes, the
            # allocator's pools, the context of the side streams) happens outside the capture
            self._enqueue(q, k, v, dout, o, dq, dk, dv, record_streams=True)
            torch.cuda.current_stream(self.device).synchronize()
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(self.device)
            cap.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.graph(g, stream=cap):
                self._enqueue(q, k, v, dout, o, dq, dk, dv, record_streams=False)
            torch.cuda.current_stream(self.device).wait_stream(cap)
            if len(self._graphs) >= 4:  # bounded: each graph keeps its own output buffers alive
                self._graphs.pop(next(iter(self._graphs)))
            self._graphs[key] = g
        g.replay()

    def _enqueue(self, q, k, v, dout, o, dq, dk, dv, record_streams: bool) -> None:
        cur = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(cur)
        for st in (self.s_in, self.s_comp, self.s_out):
            st.wait_event(start)
        max_seq_len, alpha, causal, ctx, win, full = self.cfg
        slot_free = [None, None]
        for c, (t0, t1, local, nt) in enumerate(self.chunks):
            slot = self.slots[c % 2]
            n = t1 - t0
            with torch.cuda.stream(self.s_in):
                if slot_free[c % 2] is not None:
                    self.s_in.wait_event(slot_free[c % 2])
                for name, src in (("q", q), ("k", k), ("v", v), ("do", dout)):
                    slot[name][:n].copy_(src[t0:t1], non_blocking=True)
                in_done = torch.cuda.Event()
                in_done.record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(in_done)
                a = (local, max_seq_len, alpha, causal, nt, ctx, win, None, full)
                oc = torch.ops.recir.b200_hstu_attention_fwd(slot["q"][:n], slot["k"][:n], slot["v"][:n], *a)
                gq, gk, gv = torch.ops.recir.b200_hstu_attention_bwd(slot["do"][:n], slot["q"][:n], slot["k"][:n],
                                                                     slot["v"][:n], *a)
                comp_done = torch.cuda.Event()
                comp_done.record(self.s_comp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(comp_done)
                for dst, src in ((o, oc), (dq, gq), (dk, gk), (dv, gv)):
                    dst[t0:t1].copy_(src, non_blocking=True)
                    if record_streams:  # (a captured schedule owns its buffers for its whole life)
                        src.record_stream(self.s_out)
                done = torch.cuda.Event()
                done.record(self.s_out)
            # the inputs of this slot may be overwritten once its compute has finished
            slot_free[c % 2] = comp_done
        cur.wait_event(done)
        cur.wait_stream(self.s_comp)
