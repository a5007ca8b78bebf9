"""GPU-resident rollout loop (rt_rollout_*, rt_launch_rollout_worker) against
the oracle's restatement of the reference pass loop (cu/gpu_scheduler.cu:26-83)
and, for full decode, against a token-by-token replay of the loop's logits
through the standalone sampler."""
import threading

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STATE_BYTES = 72 * 256 + 32


def make_requests(orc, n, max_tokens, seed=42, prefix_plus_one=None, temperature=0.8,
                  top_k=50, top_p=0.9):
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    ids = np.arange(1, n + 1, dtype=np.uint64)
    if prefix_plus_one is not None:
        ids = ids | (np.asarray(prefix_plus_one, dtype=np.uint64) << np.uint64(32))
    r["request_id"] = ids
    r["max_tokens"] = max_tokens
    r["kv_blocks"] = 4
    r["temperature"] = temperature
    r["top_k"] = top_k
    r["top_p"] = top_p
    r["rng_seed"] = seed
    return r


def run_array(pkg, cuda, eng, reqs, max_new=1, traj=False):
    n = len(reqs)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    dones = torch.zeros(n * 24, dtype=torch.uint8, device=cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps = torch.zeros(1, dtype=torch.int64, device=cuda)
    tr = torch.full((n, max_new), -1, dtype=torch.int32, device=cuda) if traj else None
    rw = torch.zeros(n, dtype=torch.float32, device=cuda) if traj else None
    eng.launch(requests=req_d, n_requests=n, dones=dones, state=state, step_count=steps,
               trajectories=tr, rewards=rw, n_rows=n)
    st = eng.wait()
    return st, dones.cpu().numpy(), state.cpu().numpy(), int(steps.item()), tr, rw


def mock_cfg(max_admit=1, drop=1, max_slots=256):
    return dict(max_slots=max_slots, max_admit=max_admit, drop_when_full=drop,
                decode_mode=0, reward_mode=0, max_passes=1 << 30, idle_timeout_ms=2000)


@pytest.mark.parametrize("max_admit,drop,n,tok_hi", [(1, 1, 200, 40), (256, 0, 300, 60),
                                                      (256, 1, 300, 60), (7, 0, 600, 9)])
def test_counter_decode_matches_reference_pass_loop(pkg, orc, cuda, max_admit, drop, n, tok_hi):
    rng = np.random.default_rng(n + max_admit)
    reqs = make_requests(orc, n, rng.integers(0, tok_hi + 1, size=n))
    eng = pkg.RolloutEngine(mock_cfg(max_admit, drop))
    st, dones, state, steps, _, _ = run_array(pkg, cuda, eng, reqs)
    od, _, ostate, opasses = orc.scheduler_run(reqs, max_admit=max_admit, drop_when_full=bool(drop))
    got = dones[: st["done"] * 24].view(orc.DONE_DTYPE)
    assert st["done"] == len(od) == steps
    assert got.tobytes() == od.tobytes()
    assert state.tobytes() == ostate.tobytes()
    assert st["passes"] == opasses
    assert st["dropped"] == (n - len(od) if drop else 0)
    eng.close()


def test_dropin_rollout_worker_over_mapped_rings(pkg, orc, cuda):
    """The reference bench's flow (bench/bench_gpu_scheduler.cu:41-112): mapped
    rings, the worker launched once, requests pushed by the host, dones
    drained, sentinel, sync."""
    n, tokens = 3000, 128
    reqs = make_requests(orc, n, tokens)
    rings = pkg.HostRings()
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    steps = torch.zeros(1, dtype=torch.int64, device=cuda)
    s = torch.cuda.Stream()
    pkg.check(pkg.lib().rt_launch_rollout_worker(rings.req, rings.done, state.data_ptr(),
                                                  steps.data_ptr(), 5000,
                                                  pkg._stream_ptr(s)), "rt_launch_rollout_worker")
    got_n, raw = rings.pump(reqs.view(np.uint8), n, send_sentinel=True, timeout_ms=60000)
    s.synchronize()
    assert got_n == n
    d = raw[: n * 24].view(orc.DONE_DTYPE)
    assert sorted(d["request_id"].tolist()) == list(range(1, n + 1))
    assert np.all(d["tokens_generated"] == tokens)
    assert np.allclose(d["reward"], (tokens & 0xFF) / 255.0)
    assert int(steps.item()) == n
    rings.close()


def full_cfg(max_slots=64, max_admit=256, vocab=2048, max_new=24, max_context=512,
             n_prefix=4, prefix_pages=64):
    return dict(num_q_heads=32, num_kv_heads=8, vocab=vocab, max_slots=max_slots,
                max_context=max_context, max_new_tokens=max_new, max_admit=max_admit,
                drop_when_full=0, decode_mode=1, reward_mode=0, logit_std=2.0,
                max_prefixes=n_prefix, max_prefix_pages=prefix_pages, max_passes=1 << 20,
                idle_timeout_ms=2000)


def setup_prefixes(pkg, arena, eng, lens, seed=9):
    ids = []
    for pid, L in enumerate(lens):
        pages = arena.acquire((L + 15) // 16)
        arena.fill_pages(pages, seed=seed, stream_id=1000 * pid)
        eng.set_prefix(pid, pages, L)
        ids.append(pid)
    return ids


def replay_tokens(pkg, cuda, reqs, dones, traj, vocab, logit_std=2.0):
    """Expected token stream of every finished request: the loop's logits for
    (seed, request low 32, token index) regenerated with rt_logits_synth and
    sampled with rt_sample_rows using the request's parameters."""
    rows, meta = [], []
    by_id = {int(r["request_id"]) & 0xFFFFFFFF: (i, r) for i, r in enumerate(reqs)}
    for d in dones:
        i, r = by_id[int(d["request_id"])]
        for t in range(int(d["tokens_generated"])):
            meta.append((i, t))
            rows.append((float(r["temperature"]), int(r["top_k"]), float(r["top_p"]),
                         int(r["request_id"]) & 0xFFFFFFFF, t, int(r["rng_seed"])))
    R = len(rows)
    logits = torch.empty(R, vocab, dtype=torch.float32, device=cuda)
    for k, row in enumerate(rows):
        pkg.logits_synth(logits[k], vocab, row[5], row[3], row[4], logit_std)
    tab = pkg.sample_row_table(*[np.array([row[j] for row in rows]) for j in range(6)])
    tok = pkg.sample_rows(logits, torch.from_numpy(tab.view(np.uint8)).to(cuda), vocab)
    tok = tok.cpu().numpy()
    tr = traj.cpu().numpy()
    return [(i, t, int(tok[k]), int(tr[i, t])) for k, (i, t) in enumerate(meta)]


def test_full_decode_tokens_and_schedule(pkg, orc, cuda):
    """Full decode: 2 GRPO groups x 16 rollouts sharing 40- and 64-token
    prefixes (the 40-token one has a partial last page: copy-on-write),
    plus 8 rollouts without a prefix; max_admit 256, backpressure."""
    arena = pkg.DeviceArena(2048)
    eng = pkg.RolloutEngine(full_cfg(), arena)
    setup_prefixes(pkg, arena, eng, [40, 64])
    rng = np.random.default_rng(5)
    n = 40
    pfx = np.array([1] * 16 + [2] * 16 + [0] * 8)
    reqs = make_requests(orc, n, rng.integers(1, 25, size=n), seed=1234, prefix_plus_one=pfx)
    st, dones, state, steps, traj, rew = run_array(pkg, cuda, eng, reqs, max_new=24, traj=True)
    assert st["error"] == 0 and st["attn_error"] == 0
    od, _, ostate, opasses = orc.scheduler_run(reqs, max_admit=256, drop_when_full=False)
    got = dones[: st["done"] * 24].view(orc.DONE_DTYPE)
    assert got.tobytes() == od.tobytes()
    assert state.tobytes() == ostate.tobytes()
    assert st["tokens"] == int(reqs["max_tokens"].sum())
    checks = replay_tokens(pkg, cuda, reqs, got, traj, 2048)
    bad = [c for c in checks if c[2] != c[3]]
    assert not bad, f"{len(bad)}/{len(checks)} tokens differ, first {bad[:3]}"
    eng.close()


def test_full_decode_ring_fed_matches_array(pkg, orc, cuda):
    """The same requests through mapped rings with the C host pump give the
    same token streams (by request) as the device-array source."""
    cfg = full_cfg(max_slots=32)
    arena = pkg.DeviceArena(2048)
    eng = pkg.RolloutEngine(cfg, arena)
    setup_prefixes(pkg, arena, eng, [33])
    n = 48
    reqs = make_requests(orc, n, np.random.default_rng(8).integers(1, 20, size=n), seed=77,
                         prefix_plus_one=np.array([1] * 32 + [0] * 16))
    _, adones, _, _, atraj, _ = run_array(pkg, cuda, eng, reqs, max_new=24, traj=True)
    rings = pkg.HostRings()
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    tr = torch.full((n, 24), -1, dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream()
    eng.launch(ring=rings.req, done_ring=rings.done, state=state, trajectories=tr, n_rows=n,
               stream=s)
    got_n, raw = rings.pump(reqs.view(np.uint8), n, send_sentinel=True, timeout_ms=60000)
    st = eng.wait(stream=s)
    assert got_n == n and st["stopped_by_sentinel"] == 1
    # rows are consume order == push order in both runs
    a = atraj.cpu().numpy()
    b = tr.cpu().numpy()
    assert np.array_equal(a, b)
    rings.close()
    eng.close()


def test_loop_reports_context_overflow(pkg, orc, cuda):
    """A prefix + max_tokens longer than max_context is reported (RT_EDEVICE),
    not written out of bounds."""
    arena = pkg.DeviceArena(1024)
    eng = pkg.RolloutEngine(full_cfg(max_context=64, max_new=40, max_slots=4), arena)
    setup_prefixes(pkg, arena, eng, [48])
    reqs = make_requests(orc, 2, 30, prefix_plus_one=np.array([1, 1]))
    n = len(reqs)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    eng.launch(requests=req_d, n_requests=n, state=state)
    st = eng.wait(check_errors=False)
    assert st["error"] == pkg.RT_EDEVICE
    eng.close()


class _DevView:
    """A raw device pointer seen as a torch tensor (no copy, no ownership)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def _dev(ptr, shape, typestr, cuda):
    return torch.as_tensor(_DevView(ptr, shape, typestr), device=cuda)


def _check_pass(pkg, orc, cuda, eng, arena, S, maxp, want_groups):
    b = eng.buffers()
    lens = _dev(b.seq_lens, (S,), "<i4", cuda).cpu().numpy()
    pt = _dev(b.page_table, (S, maxp), "<i4", cuda).cpu().numpy()
    q = _dev(b.q, (S, 32, 128), "<i2", cuda).cpu().numpy().view(np.uint16)
    out = _dev(b.attn_out, (S, 32, 128), "<f4", cuda).cpu().numpy()
    act = lens > 0
    assert act.any()
    kv = arena.buf.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = orc.paged_gqa_attention(q, kv, np.where(act[:, None], pt, 0), lens, 32, 8, 128 ** -0.5)
    err = np.abs(out - ref) * act[:, None, None]
    bad = err > 2e-3 + 1e-2 * np.abs(ref)
    if bad.any():
        s_, h_, d_ = np.argwhere(bad)[0]
        raise AssertionError(
            f"{bad.sum()} bad in slots {sorted(set(np.argwhere(bad)[:, 0].tolist()))}; first "
            f"slot {s_} head {h_} dim {d_}: got {out[s_, h_, d_]:.5f} ref {ref[s_, h_, d_]:.5f} "
            f"len {lens[s_]} row0 {pt[s_, :4].tolist()}")
    if not want_groups:
        assert not b.groups
        return 0
    ng = int(_dev(b.n_groups, (1,), "<i4", cuda).cpu().numpy()[0])
    recs = _dev(b.groups, (b.max_groups, 18), "<i4", cuda).cpu().numpy()[:ng]
    skip = _dev(b.skip_pages, (S,), "<i4", cuda).cpu().numpy()
    seen = set()
    for n_mem, shared, *members in recs:
        mem = members[:n_mem]
        assert 2 <= n_mem <= 16 and shared >= 1
        assert list(mem) == sorted(mem) and not seen & set(mem)
        seen |= set(mem)
        for m in mem:
            assert act[m] and skip[m] == shared and lens[m] >= 16 * shared
            assert np.array_equal(pt[m, :shared], pt[mem[0], :shared])
    assert all(skip[s] == 0 for s in range(S) if s not in seen)
    return ng


@pytest.mark.parametrize("mode", ["grouped", "per_sequence"])
def test_loop_attention_matches_oracle(pkg, orc, cuda, mode):
    """Pass by pass (host-stepped), the loop's attention output equals the
    oracle on that pass's q, KV arena, page tables and lengths.  Grouped mode
    also checks the shared-prefix group table the schedule kernel builds:
    20 + 17 + 3 slots on three prefixes (2, 4 and 18 full pages; the 40- and
    300-token ones end in a copy-on-write page), 1 on a fourth, 8 without."""
    S = 64
    cfg = full_cfg(max_slots=S)
    cfg["prefix_attention"] = (pkg.RT_PREFIX_ATTN_GROUPED if mode == "grouped"
                               else pkg.RT_PREFIX_ATTN_PER_SEQUENCE)
    arena = pkg.DeviceArena(1024)
    eng = pkg.RolloutEngine(cfg, arena)
    setup_prefixes(pkg, arena, eng, [40, 64, 300, 32])
    pfx = np.array([1] * 20 + [2] * 17 + [3] * 3 + [4] + [0] * 8)
    np.random.default_rng(3).shuffle(pfx)
    n = len(pfx)
    reqs = make_requests(orc, n, np.random.default_rng(4).integers(2, 25, size=n), seed=99,
                         prefix_plus_one=pfx)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    checked = []

    def hook(p):
        if p in (0, 1, 7, 15):
            checked.append(_check_pass(pkg, orc, cuda, eng, arena, S, 32, mode == "grouped"))
        return p >= 15

    eng.step(hook, requests=req_d, n_requests=n, state=state)
    assert len(checked) == 4
    if mode == "grouped":
        assert checked[0] == 2 + 1 + 1  # 20 -> 16 + 4; 17 -> 16 + a lone (ungrouped) one; 3
    eng.close()


@pytest.mark.parametrize("vocab", [2048, 2001])
def test_loop_logits_equal_synth(pkg, orc, cuda, vocab):
    """Pass by pass (host-stepped), every decoded slot's logits row is, bit for
    bit, rt_logits_synth's row for that slot's (seed, request low 32, token
    index), so the token replays above sample the loop's own logits.  Vocab
    2001 leaves rows unaligned and a partial last group; seeds above 2^32
    reach both key words."""
    S = 64
    cfg = full_cfg(max_slots=S, vocab=vocab)
    arena = pkg.DeviceArena(1024)
    eng = pkg.RolloutEngine(cfg, arena)
    setup_prefixes(pkg, arena, eng, [40, 64])
    n = 48
    pfx = np.array([1] * 16 + [2] * 16 + [0] * 16)
    reqs = make_requests(orc, n, np.random.default_rng(8).integers(4, 25, size=n),
                         seed=0x9E3779B97F4A7C15, prefix_plus_one=pfx)
    reqs["rng_seed"] = np.random.default_rng(9).integers(0, 2 ** 63, size=n, dtype=np.int64)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    row_dt = np.dtype([("temperature", "<f4"), ("top_k", "<u4"), ("top_p", "<f4"),
                       ("rollout_id", "<u4"), ("step", "<u8"), ("seed", "<u8")])
    assert row_dt.itemsize == pkg.SAMPLE_ROW_BYTES
    checked = []

    def hook(p):
        if p in (0, 1, 5, 11):
            b = eng.buffers()
            en = _dev(b.enable, (S,), "<u4", cuda).cpu().numpy()
            rows = _dev(b.sample_rows, (S * row_dt.itemsize,), "|u1", cuda).cpu().numpy()
            rows = rows.view(row_dt)
            lg = _dev(b.logits, (S * vocab,), "<i4", cuda).clone().view(S, vocab)
            ref = torch.empty(vocab, dtype=torch.float32, device=cuda)
            live = np.flatnonzero(en)
            assert len(live)
            for s in live:
                r = rows[s]
                pkg.logits_synth(ref, vocab, int(r["seed"]), int(r["rollout_id"]), int(r["step"]),
                                 2.0)
                diff = torch.nonzero(lg[s] != ref.view(torch.int32))
                assert diff.numel() == 0, f"pass {p} slot {s}: {diff.numel()} logits differ"
            checked.append(len(live))
        return p >= 11

    eng.step(hook, requests=req_d, n_requests=n, state=state)
    assert len(checked) == 4 and min(checked) > 0
    eng.close()
