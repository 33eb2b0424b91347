"""Expert parallelism for the MoE / QMoE layer: one process per GPU, experts sharded.

Rank r of W owns experts [r*E/W, (r+1)*E/W) and routes its own T tokens (data-parallel
routing).  One layer call:

  1. dispatch  (device)  route over all E experts, gather routed rows in expert order:
                         the rows for rank d form one contiguous block of ``send``;
  2. counts    (NCCL)    all-to-all of the per-expert row counts, [W, E/W] ints;
  3. rows      (NCCL)    all-to-all of the routed rows (variable split sizes);
  4. experts   (device)  expert FFN of the received rows, each with its local expert id
                         (rows arrive grouped by source, then by expert);
  5. rows back (NCCL)    all-to-all of the FFN rows along the reverse splits;
  6. combine   (device)  out[t] = sum_j w[t,j] * rows[pos[t,j]].

Optionally the tokens go through in chunks whose row all-to-alls run on NCCL's stream while
another chunk's experts compute (off by default; see :meth:`ExpertParallelMoE.forward`).

Transport "p2p" (the default for fp16/bf16 MoE and fp16 QMoE) replaces steps 2-6 by the device-side
exchange of the library (``moe_b200_ep_forward``): counts, rows and returned rows move by
peer stores between IPC-shared regions, ordered by flags with bounded waits, so a layer
call has no host synchronisation; the fc2 epilogue writes straight into the sender's
return buffer.

The reference plugin has no parallelism at all (one EP instance drives one device,
``musa/ep/src/ep_factory.cc:466-470``); the design follows the plan for the MoE path:
the split sizes of the variable all-to-all need the counts on the host, which costs one
small device-to-host copy per layer call.

The device steps go through a backend object so the exchange logic can be tested on CPU
ranks (gloo) with a NumPy backend; :class:`CudaBackend` is the product path.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist


class CudaBackend:
    """Device steps through the C ABI of libmoe_b200."""

    def __init__(self, pkg):
        self.pkg = pkg

    def dispatch(self, problem, x, router_probs):
        return self.pkg.ep_dispatch(problem, router_probs, x)

    def expert_ffn(self, problem, rows, row_expert, weights):
        out = torch.empty_like(rows)
        tensors = dict(weights, input=rows, output=out)
        self.pkg.expert_ffn(problem, tensors, row_expert)
        return out

    def combine(self, rows, pos, w, out):
        return self.pkg.ep_combine(rows, pos, w, out)


class ExpertParallelMoE:
    """One MoE (or QMoE) layer sharded by expert over the ranks of ``group``.

    ``local_weights`` holds this rank's experts only (leading dimension E/W) under the
    names of :class:`Tensors` fields (fc1_weights, fc1_scales, fc1_bias, ...).
    ``attrs`` are the node attributes (activation_type, k, normalize_routing_weights,
    expert_weight_bits, block_size, ...).
    """

    def __init__(self, pkg, *, num_experts: int, hidden_size: int, inter_size: int,
                 dtype: int, has_fc3: bool, local_weights: dict[str, Any], group=None,
                 backend=None, transport: str = "auto", max_rows: int | None = None,
                 **attrs):
        self.pkg = pkg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E, self.H, self.I = num_experts, hidden_size, inter_size
        self.E_local = num_experts // self.world
        self.dtype, self.has_fc3 = dtype, has_fc3
        self.attrs = dict(attrs)
        self.k = int(attrs.get("k", 1))
        self.weights = local_weights
        self.backend = backend if backend is not None else CudaBackend(pkg)
        # "p2p": device-side exchange over peer memory (moe_b200_ep_*: no host sync, no
        # collective on the data path); "collective": NCCL all-to-all around the device
        # steps.  "auto" takes p2p for fp16/bf16 MoE and fp16 QMoE on CUDA ranks with the
        # CUDA backend.
        bits = int(attrs.get("expert_weight_bits", 0))
        p2p_ok = (backend is None and self.world <= 8 and torch.cuda.is_available()
                  and (dtype in (pkg.FLOAT16, pkg.BFLOAT16) if bits == 0
                       else dtype == pkg.FLOAT16))
        if transport == "auto":
            transport = "p2p" if p2p_ok else "collective"
        if transport == "p2p" and not p2p_ok:
            raise ValueError("the p2p transport needs fp16/bf16 MoE or fp16 QMoE on CUDA ranks")
        if transport not in ("p2p", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.max_rows = max_rows
        self._comm = None
        self._ws = None

    def _problem(self, rows: int, experts: int, k: int):
        a = dict(self.attrs, k=k)
        return self.pkg.make_problem(rows, self.H, self.I, experts, self.dtype,
                                     has_fc3=self.has_fc3, **a)

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        if self.world == 1:
            out.copy_(inp)
            return out
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    # ------------------------------------------------------------- p2p transport
    def agree_max_rows(self, T: int) -> int:
        """The exchange region's row capacity, the same on every rank: the max_rows given
        to the constructor (which must then be equal on all ranks; peers write at offsets
        computed from it), else the largest first call's T over the ranks."""
        mine = (int(self.max_rows) if self.max_rows is not None else int(T),
                self.max_rows is not None)
        vals = [mine]
        if self.world > 1:
            vals = [None] * self.world
            dist.all_gather_object(vals, mine, group=self.group)
        given = {v for v, g in vals if g}
        if given and (len(given) > 1 or not all(g for _, g in vals)):
            raise ValueError(f"ranks were constructed with different max_rows "
                             f"{[v if g else None for v, g in vals]}: the exchange "
                             "regions must have the same layout on every rank")
        return max(1, max(v for v, _ in vals))

    def _connect(self, T: int, device) -> None:
        """Creates this rank's exchange region (same size on every rank: the largest call,
        agreed by an all-reduce) and opens the other ranks' regions (IPC handles)."""
        max_rows = self.agree_max_rows(T)
        self.max_rows = max_rows
        comm = self.pkg.EpComm(self.rank, self.world, max_rows, self.k, self.H, self.E,
                               self.dtype)
        mine = comm.handle()
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, mine, group=self.group)
        else:
            handles = [mine]
        comm.connect(handles)
        self._comm = comm

    def _forward_p2p(self, x, router_probs, events=None):
        T = x.shape[0]
        if self._comm is None:
            self._connect(T, x.device)
        if T > self.max_rows:
            raise ValueError(f"{T} rows exceed the exchange's max_rows={self.max_rows}; "
                             "construct the layer with a larger max_rows")
        prob = self._problem(T, self.E_local, self.k)
        out = torch.empty_like(x)
        nbytes = self._comm.workspace_size(prob)
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        tensors = dict(self.weights, input=x, router_probs=router_probs, output=out)
        if events is not None:
            self._comm.forward_staged(prob, tensors, self._ws, events)
        else:
            self._comm.forward(prob, tensors, self._ws)
        return out

    def close(self) -> None:
        if self._comm is not None:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)  # no rank frees its region while peers use it
            self._comm.close()
            self._comm = None

    def forward(self, x, router_probs, chunks: int | None = None, events=None):
        """``events`` (p2p transport only): len(EP_PHASES) + 1 timing events recorded at the
        phase boundaries of the call (``EpComm.forward_staged``)."""
        if self.transport == "p2p":
            return self._forward_p2p(x, router_probs, events)
        if events is not None:
            raise ValueError("phase events need the p2p transport")
        return self._forward_collective(x, router_probs, chunks)

    def _forward_collective(self, x, router_probs, chunks: int | None = None):
        """x [T, H], router_probs [T, E] -> output [T, H] for this rank's tokens.

        With ``chunks`` > 1 the tokens are processed in chunks whose row exchanges run
        asynchronously on NCCL's stream while the previous chunk's experts compute; the
        count exchange of all chunks costs one host round trip.  The default is one chunk:
        the persistent expert GEMM holds every SM, so the exchange kernels cannot run beside
        it, and smaller chunks only lower the rows per expert (measured on two B200s at
        4096 tokens per rank: 2.92 ms with 1 chunk, 3.37 ms with 2, 4.38 ms with 4)."""
        T = x.shape[0]
        W, El = self.world, self.E_local
        if chunks is None:
            chunks = 1
        bounds = [T * c // chunks for c in range(chunks + 1)]
        parts = []
        for c in range(chunks):
            xs, ls = x[bounds[c]:bounds[c + 1]], router_probs[bounds[c]:bounds[c + 1]]
            send, offsets, pos, w = self.backend.dispatch(
                self._problem(xs.shape[0], self.E, self.k), xs, ls)
            parts.append(dict(send=send, offsets=offsets, pos=pos, w=w))
        counts = torch.stack([(p["offsets"][1:] - p["offsets"][:-1]).to(torch.int64).view(W, El)
                              for p in parts])                      # [chunks, W, El]
        # Per destination rank: the counts of every chunk, as one even all-to-all.
        send_c = counts.permute(1, 0, 2).reshape(-1).contiguous()  # [W, chunks, El]
        recv_c = self._a2a(torch.empty_like(send_c), send_c).view(W, chunks, El)
        send_splits = counts.sum(2).tolist()                       # the one host round trip
        recv_splits = recv_c.sum(2).t().tolist()                   # [chunks][W]
        for c, p in enumerate(parts):
            p["send_splits"], p["recv_splits"] = send_splits[c], recv_splits[c]
            p["recv_counts"] = recv_c[:, c, :]
            p["recv"] = p["send"].new_empty((sum(recv_splits[c]), self.H))
            p["h"] = self._a2a_async(p["recv"], p["send"], p["recv_splits"], p["send_splits"])
        for c, p in enumerate(parts):
            self._wait(p["h"])
            local_ids = torch.arange(El, device=p["recv"].device, dtype=torch.int32).repeat(W)
            row_expert = torch.repeat_interleave(local_ids, p["recv_counts"].reshape(-1).to(
                p["recv"].device), output_size=p["recv"].shape[0])
            y_recv = self.backend.expert_ffn(self._problem(p["recv"].shape[0], El, 1), p["recv"],
                                             row_expert.to(torch.int32).contiguous(), self.weights)
            p["y_send"] = torch.empty_like(p["send"])
            p["hb"] = self._a2a_async(p["y_send"], y_recv, p["send_splits"], p["recv_splits"])
        out = torch.empty_like(x)
        for c, p in enumerate(parts):
            self._wait(p["hb"])
            self.backend.combine(p["y_send"], p["pos"], p["w"], out[bounds[c]:bounds[c + 1]])
        return out

    def _a2a_async(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return None
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group,
                                      async_op=True)

    @staticmethod
    def _wait(handle):
        if handle is not None:
            handle.wait()


class HostPipeline:
    """Calls of an expert-parallel layer on pinned host tensors: the H2D copy of call i+1
    and the D2H copy of call i-1 run on their own streams while call i computes on the
    current stream (the multi-GPU counterpart of ``moe_b200_pipeline_*``).  Host tensors
    must stay alive until :meth:`synchronize`."""

    def __init__(self, layer: ExpertParallelMoE, max_rows: int, dtype, device, depth: int = 2):
        self.layer = layer
        self.device = device
        self.cin = torch.cuda.Stream(device)
        self.cout = torch.cuda.Stream(device)
        self.slots = [dict(x=torch.empty(max_rows, layer.H, dtype=dtype, device=device),
                           lg=torch.empty(max_rows, layer.E, dtype=dtype, device=device),
                           in_done=torch.cuda.Event(), comp_done=torch.cuda.Event(),
                           out_done=torch.cuda.Event(), out=None)
                      for _ in range(depth)]
        self.calls = 0

    def submit(self, host_x, host_logits, host_out) -> None:
        s = self.slots[self.calls % len(self.slots)]
        reuse = self.calls >= len(self.slots)
        n = host_x.shape[0]
        comp = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.cin):
            if reuse:
                self.cin.wait_event(s["comp_done"])
            s["x"][:n].copy_(host_x, non_blocking=True)
            s["lg"][:n].copy_(host_logits, non_blocking=True)
            s["in_done"].record(self.cin)
        comp.wait_event(s["in_done"])
        if reuse:
            comp.wait_event(s["out_done"])
        out = self.layer.forward(s["x"][:n], s["lg"][:n])
        s["comp_done"].record(comp)
        with torch.cuda.stream(self.cout):
            self.cout.wait_event(s["comp_done"])
            host_out.copy_(out, non_blocking=True)
            s["out_done"].record(self.cout)
        out.record_stream(self.cout)
        s["out"] = out
        self.calls += 1

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)


def shard_experts(tensors: dict[str, Any], rank: int, world: int) -> dict[str, Any]:
    """The slice of each per-expert tensor (leading dimension E) owned by ``rank``."""
    out = {}
    for name, t in tensors.items():
        if t is None:
            out[name] = None
            continue
        el = t.shape[0] // world
        out[name] = t[rank * el:(rank + 1) * el].contiguous()
    return out
