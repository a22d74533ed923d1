"""Request sharding and the final output gather with world_size 2 on gloo (CPU), including a
rank that fails on the host and the error reaching the other rank instead of a hang."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, fail_rank, q):
    import datetime

    import torch.distributed as dist

    from thesis_b200.shard import gather_outputs, shard_requests

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        mine = shard_requests(n, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected host-side failure")
        outs = {i: [i] * (i % 4 + 1) for i in mine}          # ragged per-request outputs
        allo = gather_outputs(outs, n, world)
        q.put((rank, "ok", allo))
    except Exception as e:                                       # noqa: BLE001 - reported to the test
        q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, n, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return sorted(res)


def test_shard_partition():
    from thesis_b200.shard import shard_requests

    parts = [shard_requests(11, r, 4) for r in range(4)]
    assert sorted(sum(parts, [])) == list(range(11))
    with pytest.raises(ValueError):
        shard_requests(3, 4, 4)


@pytest.mark.parametrize("n", [7, 1])
def test_two_rank_gather_reassembles_every_request(n):
    """Ragged outputs, and a rank that owns no request (n = 1)."""
    res = _run(2, n)
    for rank, status, allo in res:
        assert status == "ok"
        assert allo == {i: [i] * (i % 4 + 1) for i in range(n)}


def test_failed_rank_surfaces_as_an_error_on_the_other_rank():
    res = _run(2, 6, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    assert res[0][1] == "error"                    # the collective ended with an error, not a hang
