"""Failure detection on CPU ranks (gloo): a rank that exits, one that raises, one that never joins;
the watchdog; the device-error check with a host-side fake."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from predicitivecoding_b200.parallel.health import Heartbeat, PeerFailure, Watchdog, check_device_error


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    hb = Heartbeat(store, rank, world, interval=0.1, timeout=1.0).start()
    result = "ok"
    try:
        for step in range(6):
            if rank == world - 1 and step == 2:
                if mode == "exit":
                    os._exit(0)                     # dies between steps, nothing in flight
                if mode == "raise":
                    raise RuntimeError("injected failure in a training hook")
            hb.check()                              # host-side detection before the next collective
            t = torch.ones(4) * rank
            dist.all_reduce(t)
            time.sleep(0.5)
        result = "finished"
    except PeerFailure as e:
        result = f"detected {e.ranks}"
    except RuntimeError as e:
        if "injected" in str(e):
            result = f"raised {str(e)[:40]}"
        else:                                       # the collective ended with an error: attribute it
            dead = hb.attribute()
            result = f"detected {dead}" if dead else f"raised {str(e)[:40]}"
    finally:
        hb.stop()
    q.put((rank, result))
    q.close()
    q.join_thread()                                 # flush the result before leaving
    os._exit(0)                                     # skip destroy: a peer is gone


@pytest.mark.parametrize("mode", ["exit", "raise"])
def test_survivors_detect_a_dead_rank_between_steps(mode):
    world, port = 3, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 90
    while len(got) < world and time.time() < deadline:
        try:
            r, res = q.get(timeout=5)
            got[r] = res
        except Exception:
            if mode == "exit" and len(got) == world - 1:
                break
    for p in procs:
        p.join(30)
    for r in range(world - 1):
        assert got[r] == f"detected [{world - 1}]", got
    if mode == "raise":
        assert got[world - 1].startswith("raised injected failure")


def _lonely(rank, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
        q.put("joined")
    except Exception as e:
        q.put(f"timeout after {time.time() - t0:.1f}s: {type(e).__name__}")
    q.close()
    q.join_thread()


def test_rank_that_never_joins_ends_rendezvous_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(0, _free_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(30)
    assert res.startswith("timeout after")


def test_watchdog_fires_on_a_stalled_step_and_not_on_progress():
    fired = []
    with Watchdog(0.3, fired.append, poll=0.02) as wd:
        for _ in range(10):
            time.sleep(0.05)
            wd.kick()
        assert not fired
        time.sleep(0.6)
    assert fired and fired[0] > 0.3


def test_heartbeat_flags_a_rank_that_never_beat():
    store = torch.distributed.HashStore()
    hb = Heartbeat(store, 0, 2, interval=0.05, timeout=0.2).start()
    assert hb.dead_ranks() == []
    time.sleep(0.4)
    assert hb.dead_ranks() == [1]
    store.set("hb/1", repr(time.time()))
    assert hb.dead_ranks() == []
    hb.stop()
    with pytest.raises(PeerFailure):
        time.sleep(0.3)
        hb.check()


def test_device_error_word_is_reported():
    check_device_error(torch.zeros(1, dtype=torch.int32))
    with pytest.raises(PeerFailure, match="peer flag never arrived"):
        check_device_error(torch.tensor([5], dtype=torch.int32))
