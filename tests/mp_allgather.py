"""Worker for test_reward_gpu.test_nccl_reward_allgather_two_gpus (run under
torch.distributed.run): NCCL allgather of per-rank rewards through the C ABI,
checked against the oracle on every rank."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    pkg, orc = ge.load_package(), ge.load_oracle()
    groups = 512
    g0, ng = pkg.shard_groups(groups, world, rank)
    local = np.array([orc.reward_u01(5, g0 * 16 + i + 1) for i in range(ng * 16)], np.float32)

    def exchange(b):
        obj = [b]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]
    nc = pkg.NcclRewards(rank, world, exchange)
    send = torch.from_numpy(local).to(dev)
    recv = torch.zeros(groups * 16, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream()
    nc.allgather(send, recv, stream=s)
    nc.wait(stream=s, timeout_ms=30000)
    adv = pkg.grpo_advantages(recv, 16).cpu().numpy()
    full = np.array([orc.reward_u01(5, i + 1) for i in range(groups * 16)], np.float32)
    assert recv.cpu().numpy().tobytes() == full.tobytes()
    assert adv.tobytes() == orc.grpo_advantages(full, 16).tobytes()
    print(f"rank {rank} allgather ok", flush=True)
    nc.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
