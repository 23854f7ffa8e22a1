"""Expert-parallel MoE layer: the partition of experts over ranks, the roles
of each rank, and the sum of the ranks' partial outputs.

The CPU tests run two gloo ranks, each computing its partial layer output
with the oracle (its experts only: the other experts' down rows are zero, so
they add exactly nothing), and check that the all-reduced sum is the whole
layer.  The GPU test runs two ranks on two GPUs through the library, with the
partial outputs summed inside the combine kernel over peer memory."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llambda_b200 import configs as CF
from llambda_b200 import ep
from oracle import oracle as O
from tests.helpers import host_layer, max_rel, oracle_layer

SMALL = dataclasses.replace(CF.CONFIG3, name="ep_small", hidden=512, experts=16, top_k=4,
                            inter=256, inter_sh=256)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_expert_ranges_partition_the_experts(world):
    for experts in (16, 128, 512, 7):
        ranges = [ep.expert_range(r, world, experts) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == experts
        for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
            assert e0 == b1 and b0 <= e0
    with pytest.raises(ValueError):
        ep.expert_range(2, 2, 16)


def test_layer_roles():
    roles = [ep.layer_roles(r, 4, 512, peer_reduction=False) for r in range(4)]
    assert [r["shared_here"] for r in roles] == [True, False, False, False]
    assert [r["add_residual"] for r in roles] == [True, False, False, False]  # x added once
    peer = [ep.layer_roles(r, 4, 512, peer_reduction=True) for r in range(4)]
    assert all(r["add_residual"] for r in peer)  # every rank sums all partials itself
    assert all(r["shared_here"] for r in peer)  # each for its part of the tokens


def _rank_tensors(cfg, tensors, rank, world):
    """The layer as rank `rank` sees it: other experts' (and, off the shared
    rank, the shared expert's) down rows zero."""
    roles = ep.layer_roles(rank, world, cfg.experts, peer_reduction=False)
    eb, ee = roles["expert_range"]
    out = dict(tensors)
    t, ne0, ne1, ne2, arr = tensors["ffn_down_exps"]
    per = arr.size // ne2
    down = arr.copy()
    for e in range(ne2):
        if not eb <= e < ee:
            down[e * per:(e + 1) * per] = 0
    out["ffn_down_exps"] = (t, ne0, ne1, ne2, down)
    if not roles["shared_here"]:
        t, ne0, ne1, ne2, arr = tensors["ffn_down_shexp"]
        out["ffn_down_shexp"] = (t, ne0, ne1, ne2, np.zeros_like(arr))
    return out, roles


def _gloo_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tensors = host_layer(SMALL, seed=3)
        norm = np.ones(SMALL.hidden, np.float32)
        x = O.synth_f32(3, CF.S_ACT, 0, 5 * SMALL.hidden, 1.0).reshape(5, SMALL.hidden)
        mine, roles = _rank_tensors(SMALL, tensors, rank, world)
        part, _, _ = O.moe_forward(oracle_layer(SMALL, mine, input_norm=norm,
                                                residual=roles["add_residual"]), x, 5,
                                   SMALL.top_k)
        t = torch.from_numpy(np.ascontiguousarray(part))
        ep.allreduce_partial(t)
        if rank == 0:
            full, _, _ = O.moe_forward(oracle_layer(SMALL, tensors, input_norm=norm,
                                                    residual=True), x, 5, SMALL.top_k)
            result.put(max_rel(t.numpy(), full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_partials_sum_to_the_layer(world):
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert result.get(timeout=5) < 1e-5


def _peer_worker(rank, world, port, result):
    import llambda_b200 as LB
    from tests.helpers import gpu_tensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        tensors = host_layer(SMALL, seed=4)
        norm = np.ones(SMALL.hidden, np.float32)
        T = 6
        x = O.synth_f32(4, CF.S_ACT, 0, T * SMALL.hidden, 1.0).reshape(T, SMALL.hidden)
        roles = ep.layer_roles(rank, world, SMALL.experts, peer_reduction=True)
        s = LB.MoeSession.create(SMALL.arch, SMALL.hidden, SMALL.top_k, gpu_tensors(tensors),
                                 weight_scale=SMALL.weight_scale,
                                 weights_norm=SMALL.weights_norm, max_tokens=8,
                                 expert_range=roles["expert_range"],
                                 shared_here=roles["shared_here"],
                                 input_norm=norm, norm_epsilon=1e-6,
                                 add_residual=roles["add_residual"])
        keep = ep.attach_peer_reduction([s])
        xs = torch.from_numpy(x).cuda()
        outs = []
        for _ in range(3):  # successive calls reuse both parities of the slots
            y = torch.empty_like(xs)
            s.run_device(xs, y, T)
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy())
        status = s.status()
        full, _, _ = O.moe_forward(oracle_layer(SMALL, tensors, input_norm=norm, residual=True),
                                   x, T, SMALL.top_k)
        result.put((rank, status, max(max_rel(o, full) for o in outs)))
        dist.barrier()
        s.close()
        del keep
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_reduction_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    got = sorted(result.get(timeout=5) for _ in range(world))
    for rank, status, err in got:
        assert status == 0, (rank, status)
        assert err < 1e-5, (rank, err)


@pytest.mark.gpu
def test_peer_wait_gives_up_when_a_peer_never_arrives():
    """Rank 0 of a world of two whose peer never runs (its "peer" buffer is a
    second buffer on the same GPU that nothing writes flags into): the
    combine's bounded wait gives up after two seconds, the session reports
    status bit 4, and the device stays usable."""
    import time

    import llambda_b200 as LB
    from tests.helpers import gpu_tensors

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    tensors = host_layer(SMALL, seed=4)
    T = 4
    roles = ep.layer_roles(0, 2, SMALL.experts, peer_reduction=True)
    s = LB.MoeSession.create(SMALL.arch, SMALL.hidden, SMALL.top_k, gpu_tensors(tensors),
                             weight_scale=SMALL.weight_scale, weights_norm=SMALL.weights_norm,
                             max_tokens=T, expert_range=roles["expert_range"],
                             shared_here=roles["shared_here"],
                             add_residual=roles["add_residual"])
    try:
        nbytes = s.peer_bytes(2)
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
        s.attach_peers(0, 2, [b.data_ptr() for b in bufs], nbytes)
        x = O.synth_f32(4, CF.S_ACT, 0, T * SMALL.hidden, 1.0).reshape(T, SMALL.hidden)
        xs = torch.from_numpy(x).cuda()
        y = torch.empty_like(xs)
        t0 = time.time()
        s.run_device(xs, y, T)
        torch.cuda.synchronize()
        assert time.time() - t0 < 60
        assert s.status() & 4
        z = torch.arange(8, device="cuda", dtype=torch.float32)
        assert float(z.sum().item()) == 28.0
    finally:
        s.close()


# ------------------------------------------------------------ token dispatch

@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_token_slices_partition_the_tokens(world):
    for tokens in (1, 7, 256, 2048):
        sl = [ep.token_slice(r, world, tokens) for r in range(world)]
        assert sl[0][0] == 0 and sl[-1][1] == tokens
        assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
        assert max(e - b for b, e in sl) - min(e - b for b, e in sl) <= 1


def _dispatch_worker(rank, world, port, result):
    import llambda_b200 as LB
    from tests.helpers import gpu_tensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        tensors = host_layer(SMALL, seed=8)
        norm = O.synth_f32(8, 30, 0, SMALL.hidden, 1.0)
        T = 256  # 128 tokens per rank: the prefill path on every rank
        x = O.synth_f32(8, CF.S_ACT, 0, T * SMALL.hidden, 1.0).reshape(T, SMALL.hidden)
        t0, t1 = ep.token_slice(rank, world, T)
        roles = ep.layer_roles(rank, world, SMALL.experts, peer_reduction=True)
        kw = dict(weight_scale=SMALL.weight_scale, weights_norm=SMALL.weights_norm,
                  max_tokens=T, input_norm=norm, norm_epsilon=1e-6, add_residual=True)
        s = LB.MoeSession.create(SMALL.arch, SMALL.hidden, SMALL.top_k, gpu_tensors(tensors),
                                 expert_range=roles["expert_range"], shared_here=True, **kw)
        keep = ep.attach_token_dispatch([s], max_local_tokens=(T + world - 1) // world)
        xs = torch.from_numpy(np.ascontiguousarray(x[t0:t1])).cuda()
        sel = torch.empty(t1 - t0, SMALL.top_k, dtype=torch.int32, device="cuda")
        outs = []
        for _ in range(3):  # successive calls reuse the landing zones and flags
            y = torch.empty_like(xs)
            s.run_device(xs, y, t1 - t0, sel_dev=sel)
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy())
        status = s.status()
        # the same layer on one device (every expert), same kernels and bytes
        one = LB.MoeSession.create(SMALL.arch, SMALL.hidden, SMALL.top_k, gpu_tensors(tensors),
                                   **kw)
        xa = torch.from_numpy(x).cuda()
        ya = torch.empty_like(xa)
        one.run_device(xa, ya, T)
        torch.cuda.synchronize()
        single = ya.cpu().numpy()[t0:t1]
        one.close()
        full, sel_ref, _ = O.moe_forward(oracle_layer(SMALL, tensors, input_norm=norm,
                                                      residual=True), x, T, SMALL.top_k)
        same = np.all(sel.cpu().numpy() == sel_ref[t0:t1], axis=1)
        result.put((rank, status, float(same.mean()),
                    max(max_rel(o[same], full[t0:t1][same]) for o in outs),
                    max(max_rel(o, single) for o in outs),
                    all(np.array_equal(o, outs[0]) for o in outs)))
        dist.barrier()
        s.close()
        del keep
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_token_dispatch_two_gpus():
    """Two ranks, each with half of a 256-token prefill batch and half of the
    experts: each token's row travels to its experts' owner and the results
    come back over peer memory; every rank's output matches the oracle within
    the bf16 prefill bar and the same layer on one device to float rounding."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dispatch_worker, args=(r, world, port, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    got = sorted(result.get(timeout=5) for _ in range(world))
    for rank, status, match, err_oracle, err_single, repeat in got:
        assert status == 0, (rank, status)
        assert match > 0.9, (rank, match)
        assert err_oracle < 2e-2, (rank, err_oracle)
        assert err_single < 1e-5, (rank, err_single)
        assert repeat, rank


@pytest.mark.gpu
def test_dispatch_wait_gives_up_when_a_peer_never_arrives():
    """Rank 0 of a world of two whose peer never runs (the "peer" buffer is a
    second buffer on the same GPU that nothing else writes): both bounded
    waits (the peer's rows, its done flag) give up after two seconds each,
    the session reports status bit 4, and the device stays usable."""
    import time

    import llambda_b200 as LB
    from tests.helpers import gpu_tensors

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    tensors = host_layer(SMALL, seed=4)
    T = 128
    s = LB.MoeSession.create(SMALL.arch, SMALL.hidden, SMALL.top_k, gpu_tensors(tensors),
                             weight_scale=SMALL.weight_scale, weights_norm=SMALL.weights_norm,
                             max_tokens=2 * T, expert_range=ep.expert_range(0, 2, SMALL.experts),
                             shared_here=True, add_residual=True)
    try:
        nbytes = s.dispatch_bytes(2, T)
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
        s.attach_dispatch(0, 2, [b.data_ptr() for b in bufs], nbytes, T)
        x = O.synth_f32(4, CF.S_ACT, 0, T * SMALL.hidden, 1.0).reshape(T, SMALL.hidden)
        xs = torch.from_numpy(x).cuda()
        y = torch.empty_like(xs)
        t0 = time.time()
        s.run_device(xs, y, T)
        torch.cuda.synchronize()
        assert time.time() - t0 < 60
        assert s.status() & 4
        z = torch.arange(8, device="cuda", dtype=torch.float32)
        assert float(z.sum().item()) == 28.0
    finally:
        s.close()
