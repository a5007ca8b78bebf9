"""Rewards, GRPO advantages and the NCCL reward allgather on the GPU."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_advantages_bit_exact_vs_oracle(pkg, orc, cuda):
    rng = np.random.default_rng(2)
    for G, n in [(16, 8192), (4, 64), (1, 7), (3, 3 * 33)]:
        r = rng.random(n).astype(np.float32)
        r[: G] = 0.5  # one constant group: std 0 -> eps guards the division
        got = pkg.grpo_advantages(torch.from_numpy(r).to(cuda), G).cpu().numpy()
        want = orc.grpo_advantages(r, G)
        assert got.tobytes() == want.tobytes()


def test_reward_score_kernel_matches_reference_formula(pkg, cuda):
    """reference cu/reward.cu:4-15: (token_count & 0xFF) / 255."""
    n = 600
    d = np.zeros(n, dtype=[("rollout_id", "<u4"), ("token_start", "<u4"), ("token_count", "<u4"),
                           ("reward_model_id", "<u4"), ("reward", "<f4"), ("flags", "<u4")])
    d["token_count"] = np.arange(n) * 7
    dd = torch.from_numpy(d.view(np.uint8).copy()).to(cuda)
    scores = torch.zeros(n, dtype=torch.float32, device=cuda)
    pkg.check(pkg.lib().rt_reward_score(dd.data_ptr(), n, scores.data_ptr(), None), "reward")
    torch.cuda.synchronize()
    want = ((d["token_count"] & 0xFF).astype(np.float32) / np.float32(255.0))
    assert np.array_equal(scores.cpu().numpy(), want)
    back = dd.cpu().numpy().view(d.dtype)
    assert np.array_equal(back["reward"], want)


def test_loop_rewards_follow_philox_twin(pkg, orc, cuda):
    """The loop's RT_REWARD_PHILOX rewards (by consume row) equal the oracle
    twin, and the group advantages computed from them equal the oracle's."""
    eng = pkg.RolloutEngine(dict(max_slots=64, max_admit=64, drop_when_full=0, decode_mode=0,
                                 reward_mode=1, reward_seed=5, max_passes=1 << 20,
                                 idle_timeout_ms=2000))
    n = 128
    reqs = pkg.grpo_requests(0, n // 16, 16, 5, 1)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(72 * 256 + 32, dtype=torch.uint8, device=cuda)
    dones = torch.zeros(n * 24, dtype=torch.uint8, device=cuda)
    eng.launch(requests=req_d, n_requests=n, state=state, dones=dones, n_rows=n)
    st = eng.wait()
    d = dones.cpu().numpy().view(orc.DONE_DTYPE)[: st["done"]]
    assert st["done"] == n
    by_req = {int(x["request_id"]): float(x["reward"]) for x in d}
    want = np.array([orc.reward_u01(5, i + 1) for i in range(n)], dtype=np.float32)
    got = np.array([by_req[i + 1] for i in range(n)], dtype=np.float32)
    assert np.array_equal(got, want)
    adv = pkg.grpo_advantages(torch.from_numpy(got).to(cuda), 16).cpu().numpy()
    assert adv.tobytes() == orc.grpo_advantages(want, 16).tobytes()
    eng.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_reward_allgather_two_gpus():
    """Two ranks (processes), each owning 256 groups' rewards, allgather over
    NCCL (rt_reward_allgather) and compute identical advantages."""
    script = os.path.join(ROOT, "tests", "mp_allgather.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1", MASTER_PORT="29517")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517",
                        script], capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("allgather ok") == 2
