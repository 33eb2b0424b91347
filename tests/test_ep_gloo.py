"""Expert-parallel host logic on CPU ranks (gloo, world size 1, 2 and 4).

The device steps are replaced by a NumPy backend built on the oracle; what is tested is
the exchange itself: count all-to-all, variable-split row all-to-alls, the local expert
ids of received rows and the routing-weighted combine.  Each rank's output must equal the
single-device layer on its own tokens with all experts.
"""

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class OracleBackend:
    def __init__(self, orc, attrs):
        self.orc = orc
        self.attrs = attrs

    def dispatch(self, problem, x, router_probs):
        k, E = problem.attrs.k, problem.num_experts
        idx, w = self.orc.route(router_probs.numpy(), k, self.attrs["normalize_routing_weights"])
        offsets, pos, src = self.orc.permutation(idx, E)
        send = x[torch.from_numpy(src.astype(np.int64) // k)]
        return (send, torch.from_numpy(offsets), torch.from_numpy(pos.astype(np.int64)),
                torch.from_numpy(w))

    def expert_ffn(self, problem, rows, row_expert, weights):
        out = torch.zeros(rows.shape, dtype=torch.float64)
        ffn_attrs = {a: v for a, v in self.attrs.items() if a in ("activation_type",)}
        sel = lambda n, e: None if weights.get(n) is None else weights[n][e].numpy()
        for e in range(problem.num_experts):
            m = (row_expert == e).nonzero().flatten()
            if m.numel() == 0:
                continue
            y = self.orc.expert_ffn(rows[m].numpy(), sel("fc1_weights", e), sel("fc1_bias", e),
                                    sel("fc2_weights", e), sel("fc2_bias", e),
                                    sel("fc3_weights", e), sel("fc3_bias", e), **ffn_attrs)
            out[m] = torch.from_numpy(y)
        return out

    def combine(self, rows, pos, w, out):
        res = (torch.from_numpy(w.numpy().astype(np.float64))[..., None] * rows[pos]).sum(1)
        out.copy_(res.to(out.dtype))
        return out


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q, chunks=None):
    import __graft_entry__ as ge
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg, orc = ge.load_package(), ge.load_oracle()
        from onnxruntime_musa_b200 import ep
        E, H, I, k, T = 8, 32, 24, 2, 13 + rank  # ragged token counts per rank
        attrs = dict(activation_type="silu", k=k, normalize_routing_weights=1)
        full = orc.make_moe_inputs(T=64, H=H, I=I, E=E, k=k, act="silu", gated=True,
                                   dtype="float64", bias=True, seed=5)
        x = full["x"][rank * 20:rank * 20 + T]
        lg = full["router_probs"][rank * 20:rank * 20 + T]
        weights = dict(fc1_weights=full["fc1_w"], fc1_bias=full["fc1_b"],
                       fc2_weights=full["fc2_w"], fc2_bias=full["fc2_b"],
                       fc3_weights=full["fc3_w"], fc3_bias=full["fc3_b"])
        local = ep.shard_experts({n: torch.from_numpy(v) for n, v in weights.items()}, rank, world)
        layer = ep.ExpertParallelMoE(pkg, num_experts=E, hidden_size=H, inter_size=I,
                                     dtype=pkg.FLOAT, has_fc3=True, local_weights=local,
                                     backend=OracleBackend(orc, attrs), **attrs)
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(lg), chunks=chunks).numpy()
        ref = orc.moe(x, lg, full["fc1_w"], full["fc1_b"], full["fc2_w"], full["fc2_b"],
                      full["fc3_w"], full["fc3_b"], **attrs)
        result_q.put((rank, float(np.abs(out - ref).max())))
    except Exception as exc:  # report, never hang the parent
        result_q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunks", [(1, None), (2, None), (4, None), (2, 3), (4, 2)])
def test_expert_parallel_exchange_matches_single_device(world, chunks):
    """chunks > 1 pipelines the token chunks through asynchronous row exchanges."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, chunks)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(results[r], str), results[r]
        assert results[r] < 1e-10, f"rank {r}: max |ep - ref| = {results[r]}"


def _dead_peer_worker(rank, world, port, result_q):
    import datetime
    import __graft_entry__ as ge
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    if rank == 1:  # this rank leaves between layer calls, before its next collective
        result_q.put((rank, "left"))
        return
    pkg, orc = ge.load_package(), ge.load_oracle()
    from onnxruntime_musa_b200 import ep
    attrs = dict(activation_type="silu", k=2, normalize_routing_weights=1)
    full = orc.make_moe_inputs(T=16, H=16, I=8, E=4, k=2, act="silu", gated=True,
                               dtype="float64", seed=1)
    w = dict(fc1_weights=full["fc1_w"], fc2_weights=full["fc2_w"], fc3_weights=full["fc3_w"])
    local = ep.shard_experts({n: torch.from_numpy(v) for n, v in w.items()}, rank, world)
    layer = ep.ExpertParallelMoE(pkg, num_experts=4, hidden_size=16, inter_size=8,
                                 dtype=pkg.FLOAT, has_fc3=True, local_weights=local,
                                 backend=OracleBackend(orc, attrs), **attrs)
    t0 = time.time()
    try:
        layer.forward(torch.from_numpy(full["x"]), torch.from_numpy(full["router_probs"]))
        result_q.put((rank, "no error"))
    except Exception as exc:
        result_q.put((rank, ("raised", type(exc).__name__, time.time() - t0)))


def test_expert_parallel_dead_peer_raises():
    """A rank that stops taking part makes the survivor's next collective fail with an
    error (connection loss or the process-group timeout), never a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert isinstance(res[0], tuple) and res[0][0] == "raised", res[0]
    assert res[0][2] < 60


def _max_rows_worker(rank, world, port, result_q, given):
    import __graft_entry__ as ge
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg, orc = ge.load_package(), ge.load_oracle()
        from onnxruntime_musa_b200 import ep
        attrs = dict(activation_type="silu", k=2, normalize_routing_weights=1)
        layer = ep.ExpertParallelMoE(pkg, num_experts=4, hidden_size=16, inter_size=8,
                                     dtype=pkg.FLOAT, has_fc3=False, local_weights={},
                                     backend=OracleBackend(orc, attrs), max_rows=given[rank],
                                     **attrs)
        try:
            result_q.put((rank, ("ok", layer.agree_max_rows(10 + rank))))
        except ValueError as exc:
            result_q.put((rank, ("rejected", str(exc))))
    except Exception as exc:
        result_q.put((rank, ("error", repr(exc))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("given,expect", [((None, None), ("ok", 11)), ((64, 64), ("ok", 64)),
                                          ((64, 128), ("rejected",)), ((64, None), ("rejected",))])
def test_exchange_region_capacity_agreed_or_rejected(given, expect):
    """The p2p exchange regions must have the same layout on every rank (peers store at
    offsets computed from their own max_rows): ranks given different max_rows fail on
    every rank before any region is opened."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_max_rows_worker, args=(r, 2, port, q, given)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert res[r][:len(expect)] == expect, res[r]
