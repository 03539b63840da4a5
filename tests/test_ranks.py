"""Failure detection among CPU ranks (gloo, world size 2): a rank that leaves between steps,
announced or silently, is found on the host by the ranks that stay, by name, at their next
step, with nothing in flight (`lollm_b200.ranks.PeerGuard`)."""

import json
import os
import socket

import pytest
import torch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    import datetime
    import torch.distributed as dist
    from lollm_b200.ranks import PeerGuard, RankFailure
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    guard = PeerGuard(store, rank, world, timeout_s=2.0)
    result = {"rank": rank, "steps": 0, "error": None}
    try:
        for step in range(4):
            if rank == 1 and step == 2:
                if mode == "announced":
                    guard.leave(step - 1)
                break                     # rank 1 stops between steps 1 and 2
            guard.checkpoint(step)
            t = torch.ones(4) * (rank + 1)
            dist.all_reduce(t)            # the step's only collective (the max-over-ranks timing)
            assert float(t[0]) == 3.0
            result["steps"] = step + 1
    except RankFailure as e:
        result["error"] = str(e)
        result["missing"] = e.missing
        result["left"] = {str(k): v for k, v in e.left.items()}
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump(result, f)
    os._exit(0)   # skip destroy_process_group: a peer is gone


@pytest.mark.parametrize("mode", ["announced", "silent"])
def test_rank_leaving_between_steps_is_detected(tmp_path, mode):
    ctx = torch.multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    r0 = json.load(open(tmp_path / "r0.json"))
    r1 = json.load(open(tmp_path / "r1.json"))
    assert r1["steps"] == 2 and r1["error"] is None
    assert r0["steps"] == 2, r0
    assert r0["missing"] == [1], r0
    if mode == "announced":
        assert r0["left"] == {"1": 1} and "rank 1 left after step 1" in r0["error"]
    else:
        assert r0["left"] == {} and "did not reach step 2" in r0["error"]
