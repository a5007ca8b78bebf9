"""Device-side trace of the GPU-resident loop (rt_rollout_set_trace,
rt_trace_read): the schedule kernel's records against the loop's own
counters and the requests."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STATE_BYTES = 72 * 256 + 32


def cfg(pkg):
    return dict(num_q_heads=32, num_kv_heads=8, vocab=2048, max_slots=16, max_context=256,
                max_new_tokens=24, max_admit=256, drop_when_full=0,
                decode_mode=pkg.RT_ROLLOUT_DECODE_FULL, reward_mode=0, logit_std=2.0,
                max_prefixes=1, max_prefix_pages=1, max_passes=1 << 20, idle_timeout_ms=2000)


def requests(orc, n, seed):
    rng = np.random.default_rng(seed)
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    r["request_id"] = np.arange(1, n + 1, dtype=np.uint64)
    r["max_tokens"] = rng.integers(1, 24, n)
    r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 3
    return r


def run(pkg, eng, cuda, reqs):
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    eng.launch(requests=req_d, n_requests=len(reqs), state=state)
    return eng.wait()


def test_trace_records_match_the_loop(pkg, orc, cuda):
    eng = pkg.RolloutEngine(cfg(pkg), pkg.DeviceArena(256))
    tr = pkg.DeviceTrace(1 << 14)
    eng.set_trace(tr)
    reqs = requests(orc, 40, 1)
    st = run(pkg, eng, cuda, reqs)
    rec, total = tr.read()
    assert total == len(rec) and st["error"] == 0
    by = {t: rec[rec["type"] == t] for t in set(rec["type"].tolist())}
    n = len(reqs)
    for t in (pkg.TRACE_ROLLOUT_ALLOC, pkg.TRACE_DESC_CONSUMED, pkg.TRACE_REWARD_POSTED,
              pkg.TRACE_TRAJECTORY_DONE, pkg.TRACE_ROLLOUT_FREE):
        assert len(by[t]) == n, t
    batches = by[pkg.TRACE_DECODE_BATCH]
    assert len(batches) == st["passes"]
    assert np.array_equal(batches["seq"], np.arange(st["passes"]))
    assert (np.diff(batches["tsc"].astype(np.int64)) >= 0).all()
    assert batches["rollout_id"].max() == 16          # all slots busy at some pass
    done = by[pkg.TRACE_TRAJECTORY_DONE]
    want = {int(r["request_id"]): int(r["max_tokens"]) for r in reqs}
    assert {int(d["rollout_id"]): int(d["seq"]) for d in done} == want
    alloc = {int(a["rollout_id"]): int(a["tsc"]) for a in by[pkg.TRACE_ROLLOUT_ALLOC]}
    assert all(int(d["tsc"]) >= alloc[int(d["rollout_id"])] for d in done)
    consumed = by[pkg.TRACE_DESC_CONSUMED]
    assert sorted(consumed["seq"].tolist()) == list(range(n))
    # detached: another run appends nothing
    eng.set_trace(None)
    run(pkg, eng, cuda, reqs)
    assert tr.read(16)[1] == total
    eng.close()


def test_trace_ring_wraps_keeping_the_newest(pkg, orc, cuda):
    eng = pkg.RolloutEngine(cfg(pkg), pkg.DeviceArena(256))
    tr = pkg.DeviceTrace(64)
    eng.set_trace(tr)
    st = run(pkg, eng, cuda, requests(orc, 40, 2))
    rec, total = tr.read()
    assert total > 64 and len(rec) == 64
    b = rec[rec["type"] == pkg.TRACE_DECODE_BATCH]["seq"]
    assert (np.diff(b.astype(np.int64)) == 1).all() and b[-1] == st["passes"] - 1
    eng.close()
