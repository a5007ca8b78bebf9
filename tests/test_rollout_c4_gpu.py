"""The rollout loop at the shapes it is benchmarked on.

BASELINE config 4 (continuous batching): GRPO groups of 16 whose contexts
start with one shared 1,024-token copy-on-write prefix followed by a
per-group prompt of U[64, 1024] tokens (so a group's context usually ends
mid-page), max_new U[32, 512] per rollout, Poisson arrivals, config-2
attention shape and config-3 sampling.  Here 128 rollouts (8 groups) with
arrivals gated by pass index (deterministic), checked against the oracle's
restatement of the reference pass loop (cu/gpu_scheduler.cu:33-82, with the
same arrival gate), token by token against a replay of the loop's logits
through the standalone sampler, and - host-stepped - the attention output
of selected passes against the fp64 oracle and every copy-on-write page
against the prefix page it was copied from.

Config-5 shape: 256 slots, 512 rollouts (32 groups x 16) over two waves, a
512-token prompt per group, 256 new tokens each."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STATE_BYTES = 72 * 256 + 32
VOCAB = 32000
HKV, HQ = 8, 32
PAGE_ELEMS = HKV * 2 * 16 * 128  # bf16 elements per 16-token page (all kv heads)


def c4_inputs(orc, n_groups, seed=4, mean_gap_passes=1.25):
    rng = np.random.default_rng(seed)
    n = n_groups * 16
    prompt = rng.integers(64, 1025, size=n_groups)          # per group
    max_new = rng.integers(32, 513, size=n)                 # per rollout
    gaps = rng.exponential(mean_gap_passes, size=n)
    arrival = np.floor(np.cumsum(gaps) - gaps[0]).astype(np.uint32)
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    gid = np.arange(n) // 16
    r["request_id"] = np.arange(1, n + 1, dtype=np.uint64) | \
        ((gid.astype(np.uint64) + np.uint64(1)) << np.uint64(32))
    r["max_tokens"] = max_new
    r["kv_blocks"] = (1024 + prompt[gid] + 15) // 16
    r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 1234
    return r, prompt, arrival


def c4_engine(pkg, n_groups, prompt, max_slots=256, mode=None, seed=9):
    """Engine and arena with the shared 1,024-token base prefix and one
    registered prefix per group (base pages + the group's prompt pages)."""
    base_pages = 64
    grp_pages = [(int(p) + 15) // 16 for p in prompt]
    priv = max_slots * ((512 + 16 + 15) // 16)
    arena = pkg.DeviceArena(base_pages + sum(grp_pages) + priv + 16)
    cfg = dict(num_q_heads=HQ, num_kv_heads=HKV, vocab=VOCAB, max_slots=max_slots,
               max_context=1024 + 1024 + 512, max_new_tokens=512, max_admit=256,
               drop_when_full=0, decode_mode=1, reward_mode=0, logit_std=2.0,
               max_prefixes=n_groups, max_prefix_pages=n_groups * (base_pages + 64),
               max_passes=1 << 22, idle_timeout_ms=5000)
    if mode is not None:
        cfg["prefix_attention"] = mode
    eng = pkg.RolloutEngine(cfg, arena)
    base = arena.acquire(base_pages)
    arena.fill_pages(base, seed=seed, stream_id=0)
    pages = []
    for g in range(n_groups):
        own = arena.acquire(grp_pages[g])
        arena.fill_pages(own, seed=seed, stream_id=100000 * (g + 1))
        pages.append(list(base) + list(own))
        eng.set_prefix(g, pages[-1], 1024 + int(prompt[g]))
    return eng, arena, pages


def replay(pkg, cuda, reqs, traj_rows, max_new, rows_to_check, chunk=2048):
    """(row, token index) pairs whose trajectory token differs from the
    loop's logits (regenerated with rt_logits_synth for (seed, request low
    32, token index)) sampled by rt_sample_rows with the request's
    parameters."""
    meta = [(i, t) for i in rows_to_check for t in range(int(max_new[i]))]
    bad = []
    for c0 in range(0, len(meta), chunk):
        part = meta[c0:c0 + chunk]
        logits = torch.empty(len(part), VOCAB, dtype=torch.float32, device=cuda)
        for k, (i, t) in enumerate(part):
            rq = int(reqs["request_id"][i]) & 0xFFFFFFFF
            pkg.logits_synth(logits[k], VOCAB, int(reqs["rng_seed"][i]), rq, t, 2.0)
        tab = pkg.sample_row_table(
            np.array([float(reqs["temperature"][i]) for i, _ in part]),
            np.array([int(reqs["top_k"][i]) for i, _ in part]),
            np.array([float(reqs["top_p"][i]) for i, _ in part]),
            np.array([int(reqs["request_id"][i]) & 0xFFFFFFFF for i, _ in part], dtype=np.uint32),
            np.array([t for _, t in part]), np.array([int(reqs["rng_seed"][i]) for i, _ in part]))
        tok = pkg.sample_rows(logits, torch.from_numpy(tab.view(np.uint8)).to(cuda), VOCAB)
        tok = tok.cpu().numpy()
        for k, (i, t) in enumerate(part):
            if int(tok[k]) != int(traj_rows[i, t]):
                bad.append((i, t, int(tok[k]), int(traj_rows[i, t])))
    return bad, len(meta)


@pytest.mark.parametrize("max_slots", [256, 48])
def test_c4_continuous_batching_matches_oracle_and_replay(pkg, orc, cuda, max_slots):
    n_groups = 8
    reqs, prompt, arrival = c4_inputs(orc, n_groups)
    n = len(reqs)
    assert np.any((1024 + prompt) % 16 != 0)  # some prefixes end mid-page (copy-on-write)
    eng, _, _ = c4_engine(pkg, n_groups, prompt, max_slots)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    arr_d = torch.from_numpy(arrival.astype(np.int64)).to(cuda)
    dones = torch.zeros(n * 24, dtype=torch.uint8, device=cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    traj = torch.full((n, 512), -1, dtype=torch.int32, device=cuda)
    eng.launch(requests=req_d, n_requests=n, dones=dones, state=state, trajectories=traj,
               n_rows=n, arrivals=arr_d, arrival_unit=pkg.RT_ARRIVAL_PASS)
    st = eng.wait()
    assert st["error"] == 0 and st["attn_error"] == 0
    od, dpass, ostate, opasses, admit = orc.scheduler_run(
        reqs, arrival_pass=arrival, max_admit=256, drop_when_full=False, with_admit=True,
        max_slots=max_slots)
    got = dones[: st["done"] * 24].cpu().numpy().view(orc.DONE_DTYPE)
    assert got.tobytes() == od.tobytes()
    assert state.cpu().numpy().tobytes() == ostate.tobytes()
    assert st["passes"] == opasses
    # continuous batching really happened: some pass both retired and admitted
    assert set(dpass.tolist()) & set(admit.tolist())
    if max_slots < 128:
        # ... and with fewer slots than rollouts, arrivals waited for a slot
        assert st["max_active"] == max_slots and np.any(admit > arrival)
    assert st["tokens"] == int(reqs["max_tokens"].sum())
    bad, total = replay(pkg, cuda, reqs, traj.cpu().numpy(), reqs["max_tokens"], range(n))
    assert not bad, f"{len(bad)}/{total} tokens differ, first {bad[:3]}"
    eng.close()


def _dev(ptr, shape, typestr, cuda):
    class V:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                    "data": (int(ptr), False), "version": 3}
    return torch.as_tensor(V(), device=cuda)


def test_c4_attention_and_copy_on_write_pages(pkg, orc, cuda):
    """Host-stepped: at selected passes, the loop's attention output equals
    the fp64 oracle over that pass's q, arena, page tables and lengths, and
    every slot whose prefix ends mid-page holds, in its first private page,
    the prefix's partial page rows (all heads, K and V)."""
    n_groups = 4
    reqs, prompt, arrival = c4_inputs(orc, n_groups, seed=14)
    n = len(reqs)
    S = 64
    eng, arena, pf_pages = c4_engine(pkg, n_groups, prompt, max_slots=S)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    arr_d = torch.from_numpy(arrival.astype(np.int64)).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    checked = []
    pf_tokens = 1024 + prompt

    def hook(p):
        if p not in (3, 40, 90):
            return p >= 90
        b = eng.buffers()
        maxp = b.max_pages
        lens = _dev(b.seq_lens, (S,), "<i4", cuda).cpu().numpy()
        pt = _dev(b.page_table, (S, maxp), "<i4", cuda).cpu().numpy()
        q = _dev(b.q, (S, HQ, 128), "<i2", cuda).cpu().numpy().view(np.uint16)
        out = _dev(b.attn_out, (S, HQ, 128), "<f4", cuda).cpu().numpy()
        act = lens > 0
        kv = arena.buf.view(torch.int16).cpu().numpy().view(np.uint16)
        ref = orc.paged_gqa_attention(q, kv, np.where(act[:, None], pt, 0), lens, HQ, HKV,
                                      128 ** -0.5)
        err = np.abs(out - ref) * act[:, None, None]
        assert np.all(err <= 2e-3 + 1e-2 * np.abs(ref)), f"pass {p}: max err {err.max()}"
        # copy-on-write: a decoding slot whose prefix ends mid-page holds, in
        # the page-table entry after the prefix's full pages (its first
        # private page), the prefix's partial page rows
        slots = state.cpu().numpy()[:72 * 256].view(np.uint32).reshape(256, 18)
        pages = kv.reshape(-1, HKV, 2, 16, 128)
        cow = 0
        for s_ in np.nonzero(act)[0]:
            g = (int(slots[s_, 1]) - 1) // 16
            L = int(pf_tokens[g])
            if L % 16 == 0:
                continue
            full, r = L // 16, L % 16
            mine, src = int(pt[s_, full]), int(pf_pages[g][full])
            assert mine != src
            assert np.array_equal(pages[mine, :, :, :r], pages[src, :, :, :r]), \
                f"pass {p} slot {s_}: copy-on-write page differs from the prefix page"
            cow += 1
        checked.append((p, int(act.sum()), cow))
        return p >= 90

    eng.step(hook, requests=req_d, n_requests=n, state=state, arrivals=arr_d,
             arrival_unit=pkg.RT_ARRIVAL_PASS)
    assert [c[0] for c in checked] == [3, 40, 90]
    assert sum(c[2] for c in checked) > 0  # copy-on-write slots were checked
    eng.close()


def test_c5_shape_two_waves(pkg, orc, cuda):
    """256 slots, 32 groups x 16 sharing 512-token prompts, 256 new tokens:
    two full waves.  Done stream, state bytes and pass count equal the oracle;
    grouped and per-sequence prefix attention give identical trajectories;
    every 16th rollout's 256 tokens equal the replay."""
    n_groups, P, GEN = 32, 512, 256
    n = n_groups * 16
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    gid = np.arange(n) // 16
    r["request_id"] = np.arange(1, n + 1, dtype=np.uint64) | \
        ((gid.astype(np.uint64) + np.uint64(1)) << np.uint64(32))
    r["max_tokens"] = GEN
    r["kv_blocks"] = P // 16
    r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 1234
    trajs = {}
    for mode in (pkg.RT_PREFIX_ATTN_GROUPED, pkg.RT_PREFIX_ATTN_PER_SEQUENCE):
        arena = pkg.DeviceArena(n_groups * (P // 16) + 256 * ((GEN + 31) // 16) + 16)
        cfg = dict(num_q_heads=HQ, num_kv_heads=HKV, vocab=VOCAB, max_slots=256,
                   max_context=P + GEN, max_new_tokens=GEN, max_admit=256, drop_when_full=0,
                   decode_mode=1, reward_mode=0, logit_std=2.0, max_prefixes=n_groups,
                   max_prefix_pages=n_groups * (P // 16), max_passes=1 << 22,
                   idle_timeout_ms=5000, prefix_attention=mode)
        eng = pkg.RolloutEngine(cfg, arena)
        pages = arena.acquire(n_groups * (P // 16))
        arena.fill_pages(pages, seed=4, stream_id=0)
        for g in range(n_groups):
            eng.set_prefix(g, pages[g * (P // 16):(g + 1) * (P // 16)], P)
        req_d = torch.from_numpy(r.view(np.uint8).copy()).to(cuda)
        dones = torch.zeros(n * 24, dtype=torch.uint8, device=cuda)
        state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
        traj = torch.full((n, GEN), -1, dtype=torch.int32, device=cuda)
        eng.launch(requests=req_d, n_requests=n, dones=dones, state=state, trajectories=traj,
                   n_rows=n)
        st = eng.wait()
        assert st["error"] == 0 and st["attn_error"] == 0 and st["max_active"] == 256
        od, _, ostate, opasses = orc.scheduler_run(r, max_admit=256, drop_when_full=False)
        got = dones[: st["done"] * 24].cpu().numpy().view(orc.DONE_DTYPE)
        assert got.tobytes() == od.tobytes()
        assert state.cpu().numpy().tobytes() == ostate.tobytes()
        assert st["passes"] == opasses
        trajs[mode] = traj.cpu().numpy()
        eng.close()
    a, b = trajs.values()
    assert np.array_equal(a, b)
    bad, total = replay(pkg, cuda, r, a, r["max_tokens"], range(0, n, 16))
    assert not bad, f"{len(bad)}/{total} tokens differ, first {bad[:3]}"
