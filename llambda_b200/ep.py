"""Expert-parallel plumbing of the MoE layer over torch.distributed.

Experts are independent, so rank r of `world` owns experts
[r*E/world, (r+1)*E/world) of every layer (the weights of the others never
reach it), every rank holds the replicated activations and computes the
router and top-k itself, and the ranks' partial layer outputs are summed once
per layer.  Two ways to sum them:

  * peer memory (`attach_peer_reduction`): one symmetric device buffer, mapped
    into every rank through torch's symmetric memory; each layer's combine
    kernel pushes its partial into every rank's copy over NVLink and sums all
    ranks' partials in rank order, so no collective call follows the layer
    (llambda_cuda_moe_session_attach_peers);
  * a collective (`allreduce_partial`): an all-reduce of the partial outputs
    (NCCL on GPUs, gloo on CPUs), with the residual on one rank only.

Prefill batches can instead be split by token (`attach_token_dispatch`): each
rank passes its own slice of the tokens, and every layer call sends each
token's row to the ranks owning its selected experts and brings the expert
outputs back over peer memory (llambda_cuda_moe_session_attach_dispatch).

llambda itself runs on one device; this module has no counterpart there.
"""
from __future__ import annotations


def expert_range(rank: int, world: int, experts: int) -> tuple[int, int]:
    """[begin, end) of the experts rank `rank` of `world` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    return rank * experts // world, (rank + 1) * experts // world


def shared_rank(world: int) -> int:
    """The rank that computes the shared expert (once per layer)."""
    return 0


def layer_roles(rank: int, world: int, experts: int, peer_reduction: bool) -> dict:
    """Session arguments of one rank: its expert range, whether it holds the
    shared expert, and whether its output carries the residual.  With the
    peer-memory reduction every rank holds the shared expert and computes it
    for its part of the tokens (the rank sum reunites them), and every rank
    adds the residual to the sum of all partials it forms itself; with an
    all-reduce one rank computes the shared expert and adds x, so both count
    once."""
    if peer_reduction:
        return {"expert_range": expert_range(rank, world, experts), "shared_here": True,
                "add_residual": True}
    return {"expert_range": expert_range(rank, world, experts),
            "shared_here": rank == shared_rank(world),
            "add_residual": rank == shared_rank(world)}


def attach_peer_reduction(sessions, group=None):
    """Allocates one zero-filled symmetric buffer large enough for every
    session, exchanges the peer mappings and attaches it to every session.
    Returns the buffer and its handle; keep them alive while the sessions
    run."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    group = group or dist.group.WORLD
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nbytes = max(s.peer_bytes(world) for s in sessions)
    if nbytes == 0:
        raise ValueError("the sessions cannot reduce over %d ranks" % world)
    buf = symm_mem.empty(nbytes, dtype=torch.uint8, device="cuda")
    buf.zero_()
    handle = symm_mem.rendezvous(buf, group)
    torch.cuda.synchronize()
    dist.barrier(group)
    ptrs = list(handle.buffer_ptrs)
    for s in sessions:
        s.attach_peers(rank, world, ptrs, nbytes)
    return buf, handle


def allreduce_partial(out, group=None) -> None:
    """Sums the ranks' partial layer outputs in place (the collective form)."""
    import torch.distributed as dist

    dist.all_reduce(out, group=group)


def token_slice(rank: int, world: int, tokens: int) -> tuple[int, int]:
    """[begin, end) of the tokens rank `rank` of `world` holds under the token
    dispatch (contiguous, as even as the count allows)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    return rank * tokens // world, (rank + 1) * tokens // world


def attach_token_dispatch(sessions, max_local_tokens: int, group=None):
    """One zero-filled symmetric buffer for the token dispatch of every
    session (the sessions of a stack run one at a time and share it).
    Returns the buffer and its handle; keep them alive while the sessions
    run."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    group = group or dist.group.WORLD
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nbytes = max(s.dispatch_bytes(world, max_local_tokens) for s in sessions)
    if nbytes == 0:
        raise ValueError("the sessions cannot dispatch over %d ranks" % world)
    buf = symm_mem.empty(nbytes, dtype=torch.uint8, device="cuda")
    buf.zero_()
    handle = symm_mem.rendezvous(buf, group)
    torch.cuda.synchronize()
    dist.barrier(group)
    ptrs = list(handle.buffer_ptrs)
    for s in sessions:
        s.attach_dispatch(rank, world, ptrs, nbytes, max_local_tokens)
    return buf, handle
