"""Multi-process checks of the data-parallel gradient exchange (gloo, CPU).

Two ranks hold different gradients for the same MoCE parameters; after
``allreduce_moce_grads`` both hold the mean.  A second test makes one rank
fail before the collective and checks that the other rank's collective ends
with an error (short process-group timeout) instead of waiting forever.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from datetime import timedelta
    from moce_thesis_b200 import MoCE
    from moce_thesis_b200.dist import allreduce_moce_grads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # generous: on a cold container a spawned rank may take tens of seconds to import torch
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    torch.manual_seed(0)
    net = torch.nn.Sequential(MoCE(in_channels=16, sampling_factor=2, k=4), MoCE(in_channels=8, sampling_factor=2, k=2))
    for i, p in enumerate(net.parameters()):
        p.grad = torch.full_like(p, float(rank + 1) * (i + 1))
    net[1].gate.bias.grad = None if rank == 0 else net[1].gate.bias.grad
    n = allreduce_moce_grads(net)
    # numpy arrays travel by value: a torch tensor in the queue is shared
    # through a file descriptor that dies with this process
    out = {name: p.grad.detach().numpy().copy() for name, p in net.named_parameters()}
    q.put((rank, n, out))
    dist.destroy_process_group()


def test_allreduce_averages_across_two_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict()
    for _ in range(world):
        rank, n, out = q.get(timeout=120)
        res[rank] = (n, out)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n0, g0 = res[0]
    n1, g1 = res[1]
    g0 = {name: torch.from_numpy(v) for name, v in g0.items()}
    g1 = {name: torch.from_numpy(v) for name, v in g1.items()}
    assert n0 == n1 == (7 * 16 + 4 + 1) + (3 * 8 + 2 + 1)
    names = list(g0)
    for i, name in enumerate(names):
        assert torch.equal(g0[name], g1[name])
        if name == "1.gate.bias":
            # rank 0 had no gradient (counts as zero), rank 1 had 2 * (i + 1)
            assert torch.allclose(g0[name], torch.full_like(g0[name], (2.0 * (i + 1)) / 2))
        else:
            assert torch.allclose(g0[name], torch.full_like(g0[name], 1.5 * (i + 1)))


def _failing_worker(rank, world, port, q):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # rendezvous with room for slow process start-up (a cold container pages
    # torch in for tens of seconds); the step that fails runs in a group
    # whose collectives time out after 3 s
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    short = dist.new_group(list(range(world)), timeout=timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t, group=short)  # one completed step: connections are up
    if rank == 1:
        # leaves between steps, before its collective: the host-side failure
        q.put((rank, "left"))
        q.close()
        q.join_thread()              # flush the message before the hard exit
        os._exit(0)
    try:
        t = torch.ones(4)
        dist.all_reduce(t, group=short)
        q.put((rank, "completed"))
    except Exception as exc:  # the peer never joins: the collective must error out
        q.put((rank, "error:" + type(exc).__name__))


def test_peer_failure_ends_collective_with_error():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error:"), got[0]
