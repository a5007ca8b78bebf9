"""The reference's own scheduler, reward and prefix-resolve kernels, compiled
unmodified for sm_100a into oracle/_ref/libref_cuda.so and run on the B200,
as pins of this runtime's replacements:

- rollout_worker (reference cu/gpu_scheduler.cu:26-83) against
  rt_launch_rollout_worker (the drop-in persistent worker) and the graph
  loop rt_rollout_launch in the reference's pacing (one admission per pass,
  drop when full), on the same RequestRing contents: done stream, final
  GpuRolloutState bytes and step counter equal byte for byte;
- reward_score_kernel (cu/reward.cu:4-15) against rt_reward_score;
- kv_branch_resolve (cu/kv_prefix.cu:4-23) against rt_kv_branch_resolve.

The reference worker only stops at the stop sentinel and spins without bound
on a full DoneRing, so it runs only on rings filled before its launch, with
fewer requests than DoneRing slots (the harness checks this on the host)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STATE_BYTES = 72 * 256 + 32
REQ_SLOTS_OFF, DONE_SLOTS_OFF = 128, 256  # slot arrays in RequestRing / DoneRing
RING = 1024


@pytest.fixture(scope="module")
def refcu(orc):
    try:
        return orc.RefCuda()
    except OSError as e:
        pytest.skip(str(e))


def _requests(orc, n, max_tokens, seed):
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    r["request_id"] = np.arange(1, n + 1, dtype=np.uint64) * np.uint64(7) + np.uint64(3)
    r["max_tokens"] = max_tokens
    r["kv_blocks"] = np.arange(n) % 9
    r["temperature"] = 0.8
    r["top_k"] = 50
    r["top_p"] = 0.9
    r["rng_seed"] = np.uint64(seed) + np.arange(n, dtype=np.uint64) * np.uint64(0x9E3779B9)
    return r


def _filled_request_ring(orc, refcu, reqs, cuda):
    """A RequestRing in device memory holding reqs followed by the stop
    sentinel (cons.head 0, prod.tail n + 1)."""
    n = len(reqs)
    assert n + 1 < RING
    size = refcu.sizeof(0)
    raw = np.zeros(size, dtype=np.uint8)
    sent = np.zeros(1, dtype=orc.REQUEST_DTYPE)
    sent["request_id"] = np.iinfo(np.uint64).max
    recs = np.concatenate([reqs, sent]).view(np.uint8)
    raw[REQ_SLOTS_OFF:REQ_SLOTS_OFF + recs.size] = recs
    raw[64:68] = np.frombuffer(np.uint32(n + 1).tobytes(), dtype=np.uint8)
    return torch.from_numpy(raw).to(cuda)


def _done_records(orc, done_ring):
    raw = done_ring.cpu().numpy()
    head = int(raw[0:4].view(np.uint32)[0])
    tail = int(raw[64:68].view(np.uint32)[0])
    overflow = int(raw[128:132].view(np.uint32)[0])
    recs = raw[DONE_SLOTS_OFF:DONE_SLOTS_OFF + tail * 24].view(orc.DONE_DTYPE)
    return head, tail, overflow, recs


CASES = [
    # (n requests, max_tokens range, seed): few, many (256 slots full, drops),
    # zero-token and one-token requests
    (40, (0, 30), 1),
    (300, (1, 40), 2),
    (900, (0, 400), 3),
    (1000, (200, 260), 4),
]


@pytest.mark.parametrize("n,tok,seed", CASES)
def test_rollout_worker_matches_reference_kernel(pkg, orc, refcu, cuda, n, tok, seed):
    rng = np.random.default_rng(seed)
    reqs = _requests(orc, n, rng.integers(tok[0], tok[1] + 1, size=n), seed)

    # the reference kernel
    rq_ref = _filled_request_ring(orc, refcu, reqs, cuda)
    dn_ref = torch.zeros(refcu.sizeof(1), dtype=torch.uint8, device=cuda)
    st_ref = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps_ref = torch.zeros(1, dtype=torch.int64, device=cuda)
    refcu.rollout_worker(rq_ref, dn_ref, st_ref, steps_ref)
    h_ref, t_ref, ov_ref, recs_ref = _done_records(orc, dn_ref)

    # this runtime's drop-in worker on the same ring contents
    rq = _filled_request_ring(orc, refcu, reqs, cuda)
    dn = torch.zeros(refcu.sizeof(1), dtype=torch.uint8, device=cuda)
    st = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps = torch.zeros(1, dtype=torch.int64, device=cuda)
    s = torch.cuda.current_stream()
    pkg.check(pkg.lib().rt_launch_rollout_worker(rq.data_ptr(), dn.data_ptr(), st.data_ptr(),
                                                  steps.data_ptr(), 5000, pkg._stream_ptr(s)),
              "rt_launch_rollout_worker")
    torch.cuda.synchronize()
    stats = pkg.rt_rollout_stats_t()
    pkg.check(pkg.lib().rt_rollout_worker_stats(pkg._stream_ptr(s), ctypes.byref(stats)),
              "rt_rollout_worker_stats")
    assert stats.error == 0 and stats.stopped_by_sentinel == 1
    h, t, ov, recs = _done_records(orc, dn)

    assert t == t_ref and h == h_ref == 0 and ov == ov_ref == 0
    assert recs.tobytes() == recs_ref.tobytes()
    assert st.cpu().numpy().tobytes() == st_ref.cpu().numpy().tobytes()
    assert int(steps.item()) == int(steps_ref.item()) == t
    # the ring was consumed to the sentinel by both
    assert rq.cpu().numpy()[0:4].tobytes() == rq_ref.cpu().numpy()[0:4].tobytes()
    # and the CPU restatement agrees with the reference kernel too, given the
    # same records (the stop sentinel ends the run with rollouts still active)
    sent = np.zeros(1, dtype=orc.REQUEST_DTYPE)
    sent["request_id"] = np.iinfo(np.uint64).max
    od, _, ostate, _ = orc.scheduler_run(np.concatenate([reqs, sent]), max_admit=1,
                                         drop_when_full=True)
    assert od.tobytes() == recs_ref.tobytes()
    assert ostate.tobytes() == st_ref.cpu().numpy().tobytes()


@pytest.mark.parametrize("n,tok,seed", CASES[:3])
def test_graph_loop_matches_reference_kernel(pkg, orc, refcu, cuda, n, tok, seed):
    """The CUDA-graph loop (rt_rollout_launch, counter decode) with the
    reference's pacing, fed from the same pre-filled RequestRing."""
    rng = np.random.default_rng(seed)
    reqs = _requests(orc, n, rng.integers(tok[0], tok[1] + 1, size=n), seed)
    rq_ref = _filled_request_ring(orc, refcu, reqs, cuda)
    dn_ref = torch.zeros(refcu.sizeof(1), dtype=torch.uint8, device=cuda)
    st_ref = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps_ref = torch.zeros(1, dtype=torch.int64, device=cuda)
    refcu.rollout_worker(rq_ref, dn_ref, st_ref, steps_ref)
    _, t_ref, _, recs_ref = _done_records(orc, dn_ref)

    eng = pkg.RolloutEngine(dict(max_slots=256, max_admit=1, drop_when_full=1, decode_mode=0,
                                 reward_mode=0, max_passes=1 << 30, idle_timeout_ms=2000))
    rq = _filled_request_ring(orc, refcu, reqs, cuda)
    dn = torch.zeros(refcu.sizeof(1), dtype=torch.uint8, device=cuda)
    st = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps = torch.zeros(1, dtype=torch.int64, device=cuda)
    eng.launch(ring=rq.data_ptr(), done_ring=dn.data_ptr(), state=st, step_count=steps)
    stats = eng.wait()
    assert stats["stopped_by_sentinel"] == 1
    _, t, _, recs = _done_records(orc, dn)
    assert t == t_ref
    assert recs.tobytes() == recs_ref.tobytes()
    assert st.cpu().numpy().tobytes() == st_ref.cpu().numpy().tobytes()
    assert int(steps.item()) == int(steps_ref.item())
    eng.close()


def test_reward_score_matches_reference_kernel(pkg, refcu, cuda):
    n = 5000
    rng = np.random.default_rng(17)
    raw = rng.integers(0, 256, size=n * 24, dtype=np.uint8)
    # keep the reward field a finite float so byte comparison is meaningful
    words = raw.view(np.uint32).reshape(n, 6)
    words[:, 4] = np.float32(0.25).view(np.uint32)
    d_ref = torch.from_numpy(raw.copy()).to(cuda)
    d_mine = torch.from_numpy(raw.copy()).to(cuda)
    s_ref = torch.full((n,), -1.0, dtype=torch.float32, device=cuda)
    s_mine = torch.full((n,), -1.0, dtype=torch.float32, device=cuda)
    refcu.reward_score(d_ref, s_ref)
    pkg.check(pkg.lib().rt_reward_score(d_mine.data_ptr(), n, s_mine.data_ptr(), None),
              "rt_reward_score")
    torch.cuda.synchronize()
    assert d_mine.cpu().numpy().tobytes() == d_ref.cpu().numpy().tobytes()
    assert s_mine.cpu().numpy().tobytes() == s_ref.cpu().numpy().tobytes()


def _prefix_table(pkg, refcu):
    """A KVPrefixTable built by the host API (kv_prefix.h) and then widened
    with edge states: released prefixes (refcnt 0), branches naming
    out-of-range prefix ids, random offsets."""
    size = refcu.sizeof(3)
    buf = (ctypes.c_uint8 * size)()
    L = pkg.lib()
    L.kv_prefix_table_init(buf)
    L.kv_prefix_register.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint32,
                                     ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32)]
    L.kv_branch_alloc.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                  ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint32,
                                  ctypes.POINTER(ctypes.c_uint32)]
    L.kv_prefix_release.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
    rng = np.random.default_rng(23)
    pid = ctypes.c_uint32()
    bid = ctypes.c_uint32()
    for i in range(40):
        assert L.kv_prefix_register(buf, 4096 * i + 17, 1024 + i, 64, ctypes.byref(pid)) == 0
    for i in range(600):
        p = int(rng.integers(0, 45)) if i % 7 else 513 + i  # some prefix ids out of range
        L.kv_branch_alloc(buf, i, p, int(rng.integers(-5, 1 << 40)), 16, 1, ctypes.byref(bid))
    for p in range(0, 40, 3):  # drop every reference of some prefixes
        while L.kv_prefix_release(buf, p) == 0:
            pass
    return np.frombuffer(buf, dtype=np.uint8).copy()


def test_kv_branch_resolve_matches_reference_kernel(pkg, refcu, cuda):
    tab = _prefix_table(pkg, refcu)
    ids = np.concatenate([np.arange(700), np.array([16383, 16384, 20000, 0xFFFFFFFF]),
                          np.random.default_rng(3).integers(0, 17000, size=2000)]).astype(np.uint32)
    t_ref = torch.from_numpy(tab.copy()).to(cuda)
    t_mine = torch.from_numpy(tab.copy()).to(cuda)
    ids_d = torch.from_numpy(ids.view(np.int32)).to(cuda)
    o_ref = torch.zeros(len(ids), dtype=torch.int64, device=cuda)
    o_mine = torch.full((len(ids),), 7, dtype=torch.int64, device=cuda)
    refcu.kv_branch_resolve(t_ref, ids_d, o_ref)
    pkg.check(pkg.lib().rt_kv_branch_resolve(t_mine.data_ptr(), ids_d.data_ptr(),
                                              o_mine.data_ptr(), len(ids), None),
              "rt_kv_branch_resolve")
    torch.cuda.synchronize()
    got, want = o_mine.cpu().numpy(), o_ref.cpu().numpy()
    assert np.array_equal(got, want)
    # the cases the test means to reach are all present
    assert (want == -1).any()
    assert len(set(want.tolist())) > 100


def test_reference_record_sizes_match(refcu):
    """The reference build's ring, state, table and reward record sizes equal
    this runtime's (include/request.h, kv_prefix.h, reward.h compiled here:
    34,944 / 24,832 / 18,464 / 606,280 / 24 bytes)."""
    assert [refcu.sizeof(i) for i in range(5)] == [34944, 24832, STATE_BYTES, 606280, 24]
