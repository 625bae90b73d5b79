"""Expert-parallel exchange logic (turbomoe.ep) on CPU: world-size 2 and 4
gloo groups in spawned processes.  Routing, expert compute and the combine
are the oracle's (injected), so these tests check the dispatch / combine
plumbing: every rank's output equals the single-process layer output for its
tokens, for ragged token counts, skewed routing and ranks that receive no
rows at all."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O

SHAPE = dict(hidden=256, inter=128, experts=8, top_k=2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_functions(layer, E, k, rank, E_loc, skew=False):
    from turbomoe.ep import Routing

    def route_fn(x):
        idx, w = O.compute_routing(x, layer.router, k)
        if skew:  # every token to experts 0 and 1 (both on rank 0)
            idx = torch.tensor([[0, 1]] * x.shape[0], dtype=torch.int64)
        grp = O.routing_groups(idx, E)
        slot_token = grp["tokens"].long()
        slot_pair = slot_token * k + grp["kpos"].long()
        P = slot_pair.numel()
        pair_slot = torch.empty(P, dtype=torch.int64)
        pair_slot[slot_pair] = torch.arange(P)
        counts = grp["counts"].long()
        return Routing(idx=idx, w=w, slot_token=slot_token, slot_expert=torch.repeat_interleave(torch.arange(E), counts),
                       pair_slot=pair_slot, counts=counts)

    def expert_fn(rows, eid):
        gid = eid.long().view(-1, 1) + rank * E_loc
        return O.execute_layer(layer, rows, gid, torch.ones(rows.shape[0], 1, dtype=rows.dtype))

    def combine_fn(y_slots, r, residual):
        T, kk = r.w.shape
        ys = y_slots[r.pair_slot.view(T, kk)]
        out = (r.w.float().unsqueeze(-1) * ys.float()).sum(1)
        if residual is not None:
            out = out + residual.float()
        return out.to(y_slots.dtype)

    return route_fn, expert_fn, combine_fn


def _worker(rank, world, port, skew, q):
    try:
        from turbomoe import synth
        from turbomoe.ep import ExpertParallelMoE
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        H, I, E, k = SHAPE["hidden"], SHAPE["inter"], SHAPE["experts"], SHAPE["top_k"]
        lw = synth.make_layer(synth.MoEShape(H, I, E, k, 0), 77, 0)  # same weights on every rank
        layer = O.OracleLayer(lw, torch.float32)
        T = 5 + 3 * rank  # ragged token counts
        x = synth.make_hidden(T, H, 1000 + rank, dtype=torch.float32)
        res = torch.randn(T, H, generator=torch.Generator().manual_seed(rank))
        ep = ExpertParallelMoE(E, k, *oracle_functions(layer, E, k, rank, E // world, skew))
        outs = [ep.forward(x), ep.forward(x, residual=res)]
        # reference: the whole layer on this rank's tokens, same routing
        idx, w = O.compute_routing(x, layer.router, k)
        if skew:
            idx = torch.tensor([[0, 1]] * T, dtype=torch.int64)
        ref = O.execute_layer(layer, x, idx, w)
        errs = [(outs[0] - ref).abs().max().item(), (outs[1] - (ref + res)).abs().max().item()]
        q.put((rank, errs, ep.last_counts, list(ep.local_experts())))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None))


def _run(world, skew=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, skew, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(results, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 4])
def test_ep_matches_single_process_layer(world):
    for rank, errs, counts, experts in _run(world):
        assert not isinstance(errs, str), errs
        assert max(errs) < 1e-5, (rank, errs)
        assert len(experts) == SHAPE["experts"] // world
        sc, rc = counts
        assert sum(sc) == (5 + 3 * rank) * SHAPE["top_k"]


def test_ep_skewed_routing_and_idle_ranks():
    res = _run(2, skew=True)
    for rank, errs, counts, _ in res:
        assert not isinstance(errs, str), errs
        assert max(errs) < 1e-5, (rank, errs)
    # every row goes to rank 0; rank 1 receives none
    assert sum(res[1][2][1]) == 0
    assert sum(res[0][2][1]) == sum(sum(r[2][0]) for r in res)


def test_zipf_routing_bias_skews_owner_load():
    """The skewed-routing workload (bench.py --workload ep --ep-zipf 1.2): the
    bias is log p_e with p_e ~ rank^-1.2 over a seeded permutation (hottest 0),
    carried exactly by one coordinate, and it concentrates the routed pairs on
    few experts; s = 0 keeps the routing balanced."""
    import torch
    from turbomoe import synth
    from oracle import moe_oracle as O
    E, H, k, G = 64, 512, 8, 8
    b = synth.zipf_expert_bias(E, 3, 1.2)
    assert b.max().item() == 0.0
    ranks = torch.exp(-b / 1.2).round()
    assert sorted(ranks.tolist()) == list(range(1, E + 1))
    assert torch.equal(b, synth.zipf_expert_bias(E, 3, 1.2))      # seeded
    shape = synth.MoEShape(H, 256, E, k, 0)
    lw = synth.make_layer(shape, 11, 0)
    x = synth.make_hidden(512, H, 4, rms_normalise=True)
    w = synth.router_with_bias(lw.router, b)
    xb = synth.tokens_for_bias(x)
    # the bias is carried exactly: logits = W x (coordinate H-1 excluded) + bias
    ref = x.float()[:, :-1] @ lw.router.float()[:, :-1].T + b.to(torch.bfloat16).float()
    assert torch.allclose(xb.float() @ w.float().T, ref, atol=1e-4)
    loads = {}
    for s in (0.0, 1.2):
        wb = synth.router_with_bias(lw.router, synth.zipf_expert_bias(E, 3, s))
        idx, _ = O.compute_routing(xb, wb, k)
        per_owner = torch.bincount(idx.reshape(-1) // (E // G), minlength=G).float()
        loads[s] = (per_owner.max() / per_owner.mean()).item()
    assert loads[0.0] < 1.25 and loads[1.2] > 1.5
