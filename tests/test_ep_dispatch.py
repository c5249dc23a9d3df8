"""Expert-parallel setup (osm_b200.ep) on gloo ranks on the CPU: the IPC
handles of the ranks' EP blocks are gathered in rank order together with the
rank geometry; ranks that disagree on the geometry (a rank that would send a
different number of pairs than its peers expect) all fail with ValueError,
and a rank that never joins makes the others fail with a RuntimeError after
the exchange's timeout instead of hanging."""
import datetime
import os
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "orbi-streammoe_b200"))


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker(rank, world, port, mode, q, done):
    from osm_b200 import ep

    _init(rank, world, port)
    try:
        handle = bytes([rank]) * ep.IPC_HANDLE_BYTES
        geometry = (world, 512, 10, 2048, 64, 1)
        if mode == "mismatch" and rank == 1:
            geometry = (world, 256, 10, 2048, 64, 1)   # fewer tokens: fewer pairs than expected
        if mode == "absent" and rank == 1:
            done.wait(60)                              # never joins the exchange
            q.put((rank, "absent"))
            return
        try:
            hs = ep.exchange_handles(handle, geometry,
                                     timeout=datetime.timedelta(seconds=2) if mode == "absent" else None)
            q.put((rank, [h[0] for h in hs]))
        except ValueError:
            q.put((rank, "ValueError"))
        except RuntimeError:
            q.put((rank, "RuntimeError"))
        finally:
            if mode == "absent":
                done.set()
    finally:
        if mode != "absent":
            dist.destroy_process_group()


def _run(mode, world=2):
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    done = ctxm.Event()
    port = 29300 + (os.getpid() % 400) + {"ok": 0, "mismatch": 1, "absent": 2}[mode]
    procs = [ctxm.Process(target=_worker, args=(r, world, port, mode, q, done)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    return res


def test_handles_gathered_in_rank_order():
    res = _run("ok")
    assert res == [(0, [0, 1]), (1, [0, 1])]


def test_geometry_mismatch_fails_on_every_rank():
    res = _run("mismatch")
    assert res == [(0, "ValueError"), (1, "ValueError")]


def test_absent_rank_times_out_with_an_error():
    res = _run("absent")
    assert res == [(0, "RuntimeError"), (1, "absent")]


def test_context_rows():
    from osm_b200 import ep

    assert ep.context_rows(8, 512, 10) == 9 * 5120
    assert ep.context_rows(1, 4096, 10) == 2 * 40960


def test_handle_size_checked():
    from osm_b200 import ep

    with pytest.raises(ValueError):
        ep.exchange_handles(b"x", (1,))
