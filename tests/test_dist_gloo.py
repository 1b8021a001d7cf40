"""Multi-process host logic of the whole-cloud sharding (ns_fps_b200.dist),
run as world_size-2 gloo process groups on the CPU: the shard map, the
max/sum over ranks that bench.py uses for whole-job timing, and the failure
path where one rank leaves before a collective."""
import multiprocessing as mp
import os
import socket
import traceback

import pytest

from ns_fps_b200 import dist as D


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          LOCAL_RANK=str(rank), WORLD_SIZE=str(world))
        D.init("gloo", timeout_s=10 if mode == "ok" else 4)
        if mode == "ok":
            mine = D.shard_indices(256, rank, world)
            mx = D.max_over_ranks([10.0 * (rank + 1), -rank])
            sm = D.sum_over_ranks([len(mine), 1.0])
            D.barrier()
            q.put((rank, "ok", mine[:3], mx, sm))
        else:  # rank 1 leaves without joining the collective
            if rank == 1:
                q.put((rank, "left", None, None, None))
                q.close()
                q.join_thread()  # flush the queue before leaving abruptly
                os._exit(0)
            try:
                D.max_over_ranks([1.0])
                q.put((rank, "no-error", None, None, None))
            except Exception as e:  # noqa: BLE001
                q.put((rank, "error", type(e).__name__, None, None))
            # the group lost a member: leave without tearing it down
            q.close()
            q.join_thread()
            os._exit(0)
        D.finalize()
    except Exception:  # noqa: BLE001
        q.put((rank, "crash", traceback.format_exc(), None, None))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=60)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def test_shard_indices_cover_every_cloud_once():
    for world in (1, 2, 3, 8):
        seen = sorted(i for r in range(world) for i in D.shard_indices(256, r, world))
        assert seen == list(range(256))
    with pytest.raises(ValueError):
        D.shard_indices(4, 2, 2)


def test_two_rank_gloo_aggregation():
    res = _run("ok")
    assert res[0][1] == "ok", res[0][2]
    assert res[1][1] == "ok", res[1][2]
    assert res[0][2] == [0, 2, 4] and res[1][2] == [1, 3, 5]
    assert res[0][3] == [20.0, 0.0] and res[1][3] == [20.0, 0.0]
    assert res[0][4] == [256.0, 2.0]


def test_rank_leaving_surfaces_as_error_not_hang():
    res = _run("leave")
    assert res[1][1] == "left"
    assert res[0][1] == "error", res[0]
