"""Pins of the CPU oracle itself: published known-answer vectors, the
reference's own test expectations, and self-consistency properties."""
import numpy as np
import pytest


# Philox4x32-10 known-answer vectors published with Random123 (Salmon et al.)
PHILOX_KAT = [
    ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
    ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
    ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
     [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
]


@pytest.mark.parametrize("ctr,key,want", PHILOX_KAT)
def test_philox_known_answers(orc, ctr, key, want):
    assert orc.philox(ctr, key) == want


def test_reference_cpu_tests_pass_here(orc):
    """The reference's own CPU test binaries (built from its tree into
    oracle/_ref) pass in this environment."""
    import os
    import subprocess
    for t in ("test_hw_ring", "test_smoke"):
        path = os.path.join(orc.REF, t)
        if not os.path.exists(path):
            pytest.skip("oracle/_ref not built")
        r = subprocess.run([path], capture_output=True, text=True, timeout=120)
        assert r.returncode == 0 and "passed" in r.stdout


def test_fixed128_known_answer_inputs(orc):
    """reference test/test_bench.cu:91-107 input pattern; the CPU reference
    (test_bench.cu:109-155) output is finite and its token is the argmax."""
    q, block = fixed128_inputs(orc)
    out, tok = orc.fixed128_attention(q, block, 17)
    assert np.all(np.isfinite(out)) and tok == int(np.argmax(out))
    # seq_len > 32 clamps to the 32-token block
    o32, _ = orc.fixed128_attention(q, block, 32)
    o99, _ = orc.fixed128_attention(q, block, 99)
    assert np.array_equal(o32, o99)


def fixed128_inputs(orc):
    q = np.array([orc.oracle_lib().orc_f32_to_f16_rne(((d % 17) - 8) / 8.0) for d in range(128)],
                 dtype=np.uint16)
    block = np.zeros(2 * 32 * 128, dtype=np.uint16)
    for t in range(32):
        for d in range(128):
            k = (((t + 1) * ((d % 13) + 1)) % 23 - 11) / 32.0
            v = (((t + 3) * ((d % 11) + 5)) % 29 - 14) / 29.0
            block[t * 128 + d] = orc.oracle_lib().orc_f32_to_f16_rne(k)
            block[32 * 128 + t * 128 + d] = orc.oracle_lib().orc_f32_to_f16_rne(v)
    return q, block


def test_f16_roundtrip(orc):
    lib = orc.oracle_lib()
    for x in [0.0, 1.0, -0.125, 0.333251953125, 65504.0, 6.103515625e-05, 5.960464477539063e-08]:
        h = lib.orc_f32_to_f16_rne(x)
        assert lib.orc_f16_to_f32(h) == np.float32(x)
    assert np.float16(lib.orc_f16_to_f32(lib.orc_f32_to_f16_rne(0.1))) == np.float16(0.1)


def test_paged_attention_oracle_matches_dense_numpy(orc):
    rng = np.random.default_rng(0)
    B, Hq, Hkv, P = 3, 8, 2, 4
    lens = np.array([5, 33, 64], dtype=np.int32)
    npages = 20
    pt = rng.permutation(npages)[: B * P].reshape(B, P).astype(np.int32)
    arena = rng.standard_normal(npages * Hkv * 2 * 16 * 128).astype(np.float32)
    q = rng.standard_normal((B, Hq, 128)).astype(np.float32)
    to_bits = lambda x: (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    qb, ab = to_bits(q), to_bits(arena)
    out = orc.paged_gqa_attention(qb, ab, pt, lens, Hq, Hkv, 128 ** -0.5)
    qf = (qb.astype(np.uint32) << 16).view(np.float32)
    af = (ab.astype(np.uint32) << 16).view(np.float32).reshape(npages, Hkv, 2, 16, 128)
    for b in range(B):
        L = lens[b]
        K = np.concatenate([af[pt[b, p], :, 0] for p in range(P)], axis=1)[:, :L]
        V = np.concatenate([af[pt[b, p], :, 1] for p in range(P)], axis=1)[:, :L]
        for h in range(Hq):
            s = K[h // (Hq // Hkv)] @ qf[b, h].astype(np.float64) * 128 ** -0.5
            p = np.exp(s - s.max())
            ref = (p / p.sum()) @ V[h // (Hq // Hkv)]
            np.testing.assert_allclose(out[b, h], ref, rtol=1e-5, atol=1e-6)


def test_scheduler_oracle_reference_semantics(orc):
    """cu/gpu_scheduler.cu:26-83: one admission per pass into the lowest free
    slot, then one token per active slot per pass; a slot finishes in the
    pass where tokens == max_tokens."""
    reqs = np.zeros(3, dtype=orc.REQUEST_DTYPE)
    reqs["request_id"] = [10, 11, (7 << 32) | 12]
    reqs["max_tokens"] = [2, 0, 1]
    dones, passes, state, _ = orc.scheduler_run(reqs)
    # r0 admitted pass 0 -> tokens 1 (p0), 2 (p1), done p2; r1 admitted p1
    # (slot 1), max 0 -> done p1; r2 admitted p2 (slot 1 again), done p3
    assert [(int(d["request_id"]), int(d["rollout_id"]), int(p)) for d, p in zip(dones, passes)] == \
        [(11, 1, 1), (10, 0, 2), (12, 1, 3)]
    assert np.allclose(dones["reward"], [0.0, 2 / 255, 1 / 255])


def test_scheduler_oracle_drop_vs_backpressure(orc):
    reqs = np.zeros(300, dtype=orc.REQUEST_DTYPE)
    reqs["request_id"] = np.arange(300)
    reqs["max_tokens"] = 1000
    d_drop, _, _, _ = orc.scheduler_run(reqs, max_admit=300, drop_when_full=True)
    d_bp, _, _, _ = orc.scheduler_run(reqs, max_admit=300, drop_when_full=False)
    assert len(d_drop) == 256 and len(d_bp) == 300


def test_grpo_oracle(orc):
    r = np.random.default_rng(1).random(64).astype(np.float32)
    a = orc.grpo_advantages(r, 16)
    g = r.reshape(4, 16).astype(np.float64)
    ref = (g - g.mean(1, keepdims=True)) / (g.std(1, keepdims=True) + 1e-6)
    np.testing.assert_allclose(a.reshape(4, 16), ref, rtol=1e-4, atol=1e-5)


def test_sample_oracle_semantics(orc):
    """cu/sample.cu:40-123: top-k keeps ties at the cutoff, top-p in (0,1)
    only gates the walk, r == 0 returns index 0."""
    logits = np.array([0.0, 5.0, 5.0, 1.0, -3.0], dtype=np.float32)
    # k = 1 keeps both 5.0 entries (ties at the cutoff survive)
    assert orc.sample_row(logits, 1.0, 1, 0.9, 0) == 0
    assert orc.sample_row(logits, 1.0, 1, 0.9, 1) == 1
    assert orc.sample_row(logits, 1.0, 1, 0.9, 0xFFFFFF) == 2
    # no top-p gate: division walk
    assert orc.sample_row(logits, 1.0, 0, 1.0, 0x800000) in (1, 2)


def test_sampler_uniform_matches_oracle_philox(pkg, orc):
    """rt_sample_uniform24 (product, host side) == oracle Philox stream."""
    for seed, r, s in [(1234, 0, 0), (1234, 255, 0), (5, 77, 2**40 + 3), (2**63 + 1, 2**32 - 1, 7)]:
        assert pkg.sample_uniform24(seed, r, s) == orc.sample_u24(seed, r, s)


def test_xoshiro_inversion(orc):
    """The reference's first xoshiro256** draw reproduces any injected value."""
    M = 1 << 64
    rotl = lambda x, k: ((x << k) | (x >> (64 - k))) % M
    for v in [0, 1, 0xFFFFFF, 0x123456, 12345678]:
        s1 = orc.xoshiro_s1_for_first_output(v)
        assert (rotl((s1 * 5) % M, 7) * 9) % M == v


def test_scheduler_oracle_arrivals_and_slot_limit(orc):
    """The arrival gate and a slot count below 256 (the device loop's
    rt_rollout_io_t.arrivals and max_slots): a request is admitted no earlier
    than its arrival pass, in order, into the lowest free slot below
    max_slots; admission precedes retirement within a pass."""
    reqs = np.zeros(3, dtype=orc.REQUEST_DTYPE)
    reqs["request_id"] = [1, 2, 3]
    reqs["max_tokens"] = [2, 1, 1]
    dones, dpass, _, passes, admit = orc.scheduler_run(
        reqs, arrival_pass=[0, 3, 3], max_admit=256, drop_when_full=False, with_admit=True,
        max_slots=1)
    # r1 holds the only slot until it retires in pass 2; r2 arrives in pass 3
    # and is admitted at once; r3 waits for the slot r2 frees in pass 4
    assert admit.tolist() == [0, 3, 5]
    assert dpass.tolist() == [2, 4, 6]
    assert dones["rollout_id"].tolist() == [0, 0, 0] and passes == 7


def test_scheduler_oracle_arrival_properties(orc):
    rng = np.random.default_rng(12)
    n = 200
    reqs = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    reqs["request_id"] = np.arange(1, n + 1)
    reqs["max_tokens"] = rng.integers(0, 40, size=n)
    arrival = np.sort(rng.integers(0, 300, size=n)).astype(np.uint32)
    for slots in (256, 16, 3):
        dones, dpass, _, _, admit = orc.scheduler_run(
            reqs, arrival_pass=arrival, max_admit=256, drop_when_full=False, with_admit=True,
            max_slots=slots)
        assert len(dones) == n
        assert np.all(admit >= arrival) and np.all(np.diff(admit.astype(np.int64)) >= 0)
        assert np.all(dones["rollout_id"] < slots)
        # each rollout is done max(1, max_tokens) + ... passes after admission:
        # tokens reach max_tokens after max_tokens decode passes
        by_id = {int(d["request_id"]): int(p) for d, p in zip(dones, dpass)}
        for i in range(n):
            assert by_id[i + 1] == int(admit[i]) + int(reqs["max_tokens"][i])


def test_paced_pump_pushes_at_arrival_times(pkg, orc):
    """rt_host_pump_paced on the host alone (no consumer): every request and
    then the stop sentinel are pushed in order, none before its arrival
    time, so the call takes at least the last arrival."""
    import time
    n = 40
    reqs = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    reqs["request_id"] = np.arange(1, n + 1)
    arrival = (np.arange(n, dtype=np.uint64) * 500_000).astype(np.uint64)  # every 0.5 ms
    rings = pkg.HostRings()
    try:
        t0 = time.perf_counter()
        got, _, _ = rings.pump_paced(reqs, arrival, 0, send_sentinel=True, timeout_ms=5000)
        dt = time.perf_counter() - t0
        assert got == 0
        assert dt >= float(arrival[-1]) / 1e9
        raw = (ctypes_bytes(rings.req, 128 + 1024 * 34))
        tail = int(np.frombuffer(raw[64:68], dtype=np.uint32)[0])
        assert tail == n + 1
        recs = np.frombuffer(raw[128:128 + (n + 1) * 34], dtype=orc.REQUEST_DTYPE)
        assert recs["request_id"][:n].tolist() == list(range(1, n + 1))
        assert int(recs["request_id"][n]) == np.iinfo(np.uint64).max
    finally:
        rings.close()


def ctypes_bytes(ptr, n):
    import ctypes
    return ctypes.string_at(ptr, n)
