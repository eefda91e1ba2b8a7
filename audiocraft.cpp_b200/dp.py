"""Host-side coordination of data-parallel ranks (one process per GPU) around libactrain.so.

The reference trains on one device; data parallelism is this build's addition.  The device side
is the library's own NCCL communicator (act_nccl_init, act_set_grad_sync, act_set_timeout).  What
lives here is what the ranks' host threads need to agree on, over a CPU (gloo) process group, so
that a failed rank is noticed on the host before the others launch their next collective:

* share_nccl_id  -- rank 0 creates the NCCL unique id and every rank receives it; a rank 0 that
                    never gets there makes the others fail after the group's timeout.
* check_peers    -- a bounded barrier (gloo's monitored barrier) between steps: a rank that
                    stalled, died or raised makes the others raise PeerFailure naming it,
                    instead of entering an all-reduce that would never complete.
"""
from __future__ import annotations

from datetime import timedelta

import torch.distributed as dist


class PeerFailure(RuntimeError):
    """Another rank did not reach a coordination point in time (stalled, died or raised)."""


def host_group(timeout_s: float):
    """A gloo group over all ranks for host-side coordination, with its own timeout."""
    return dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))


def share_nccl_id(group, rank: int, make_id) -> bytes:
    """Rank 0 calls make_id() (act_nccl_get_unique_id); every rank returns its bytes."""
    box = [make_id() if rank == 0 else None]
    try:
        dist.broadcast_object_list(box, src=0, group=group)
    except RuntimeError as e:  # gloo raises on timeout or on a closed peer connection
        raise PeerFailure(f"rank {rank}: no NCCL id from rank 0 ({e})") from e
    return box[0]


def check_peers(group, timeout_s: float, what: str = "step") -> None:
    """Bounded barrier over the host group; raises PeerFailure when a rank does not arrive."""
    try:
        dist.monitored_barrier(group=group, timeout=timedelta(seconds=timeout_s), wait_all_ranks=True)
    except RuntimeError as e:
        raise PeerFailure(f"peer check before {what} failed: {e}") from e
