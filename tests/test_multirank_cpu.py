"""Multi-rank host logic on CPU with gloo (world size 2): groups are split
without overlap, each rank's reward shard allgathers into the global order,
and every rank computes the same advantages as a single process.  Also
exercises failure detection on the host: a rank that never joins the
collective makes the others fail with a timeout instead of hanging."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q, mode):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import __graft_entry__ as ge
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5 if mode == "dead_peer" else 60))
    pkg, orc = ge.load_package(), ge.load_oracle()
    groups, G = 512, 16
    g0, ng = pkg.shard_groups(groups, world, rank)
    reqs = pkg.grpo_requests(g0, ng, G, 256, 32)
    lo = (reqs["request_id"] & np.uint64(0xFFFFFFFF)).astype(np.int64)
    rewards = torch.tensor([orc.reward_u01(5, int(x)) for x in lo], dtype=torch.float32)
    out = torch.zeros(groups * G, dtype=torch.float32)
    try:
        if mode == "dead_peer" and rank == 1:
            q.put((rank, "skipped"))
            return  # this rank never reaches the collective
        dist.all_gather_into_tensor(out, rewards)
        adv = orc.grpo_advantages(out.numpy(), G)
        q.put((rank, out.numpy().tobytes(), adv.tobytes(), lo.tolist(),
               (reqs["request_id"] >> np.uint64(32)).tolist()))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def run(world, mode, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    return sorted(res, key=lambda x: x[0])


def test_two_rank_reward_exchange_matches_single_process(orc):
    res = run(2, "ok", 29611)
    (r0, out0, adv0, ids0, pf0), (r1, out1, adv1, ids1, pf1) = res
    assert out0 == out1 and adv0 == adv1
    full = np.array([orc.reward_u01(5, i + 1) for i in range(512 * 16)], np.float32)
    assert out0 == full.tobytes()
    assert adv0 == orc.grpo_advantages(full, 16).tobytes()
    assert sorted(ids0 + ids1) == list(range(1, 512 * 16 + 1))
    assert set(pf0) == set(range(1, 257)) and set(pf1) == set(range(1, 257))


def test_dead_peer_times_out_instead_of_hanging():
    res = run(2, "dead_peer", 29613)
    assert res[1][1] == "skipped"
    assert res[0][1] == "error"


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_groups_partition(pkg, world):
    spans = [pkg.shard_groups(512, world, r) for r in range(world)]
    covered = [g for g0, n in spans for g in range(g0, g0 + n)]
    assert covered == list(range(512))
