"""Host-side failure detection with gloo CPU ranks (no GPU is faulted or hung):
a rank that raises and leaves, and a rank that stops beating, are both detected by the
survivors at a step boundary; a NaN loss stops training."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from burn_dragon_b200.parallel.fault import Heartbeat, NonFiniteGuard, NonFiniteLoss, PeerFailure


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    hb = Heartbeat(interval=0.1, timeout=1.0)
    hb.wait_for_peers(5.0)
    dist.barrier()
    try:
        for step in range(50):
            hb.check()
            if rank == 1 and step == 3:
                if mode == "raise":
                    hb.announce_exit("RuntimeError: injected at step 3")
                    out[rank] = "left"
                    return
                hb.stop()  # "hang": stop beating, stay silent
                time.sleep(3.0)
                out[rank] = "silent"
                return
            time.sleep(0.1)
        out[rank] = "finished"
    except PeerFailure as e:
        out[rank] = f"detected: {e}"
    finally:
        hb.stop()


@pytest.mark.parametrize("mode", ["raise", "silent"])
def test_survivor_detects_failed_peer(mode):
    out = mp.Manager().dict()
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode is not None
    assert out[0].startswith("detected"), out[0]
    assert ("left" in out[0]) == (mode == "raise")


def test_non_finite_guard():
    g = NonFiniteGuard()
    g.check(0, torch.tensor(1.0))
    with pytest.raises(NonFiniteLoss):
        g.check(1, torch.tensor(float("nan")))


def _timeout_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank), BDH_PG_TIMEOUT_S="3")
    from burn_dragon_b200.train.trainer import init_distributed

    init_distributed()
    dist.all_reduce(torch.ones(1))  # one good step together
    if rank == 1:
        out[rank] = "silent"  # stays alive between steps but never joins the next collective
        time.sleep(8.0)
        return
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(1))
        out[rank] = "completed"
    except Exception as e:  # the process group's timeout ends the collective
        out[rank] = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"


def test_process_group_timeout_ends_a_collective_with_a_missing_peer():
    out = mp.Manager().dict()
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=_timeout_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode is not None
    assert out[1] == "silent"
    assert out[0].startswith("error after"), out[0]
    assert 2.0 < float(out[0].split()[2].rstrip("s:")) < 8.0  # the 3 s process-group timeout
