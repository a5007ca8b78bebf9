"""Per-step CommandRing decode path on the GPU through the C ABI
(rt_attention_fixed128, rt_launch_decode_worker + rt_host_decode_pump).

Checked against
  - the reference's own fixed128 step (cu/attention_decode.cu, compiled
    unmodified into oracle/_ref/libref_cuda.so): outputs bit-identical,
    token ids, byte / tile / cycle counts equal;
  - the CPU oracle (process_descriptor + the reference test's CPU
    attention): outputs within the reference test's 1e-4 absolute
    (test/test_bench.cu:717), completion records equal, token ids equal
    except where the oracle's own top two outputs lie within 2e-4 (fp32
    rounding decides those; the GPU-vs-GPU check covers them exactly).
"""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 1e-4
BLOCK = 16384
RT_ETIMEOUT, RT_EDEVICE = -3, -5


def make_arena(dev, n_blocks, seed, std=1.0):
    rng = np.random.default_rng(seed)
    host = (rng.standard_normal(n_blocks * BLOCK // 2) * std).astype(np.float16).view(np.uint8)
    return host, torch.from_numpy(host.copy()).to(dev)


def make_descs(orc, n, n_blocks, seed, offsets=None):
    rng = np.random.default_rng(seed)
    d = np.zeros(n, orc.DESCRIPTOR_DTYPE)
    d["seq_id"] = rng.integers(0, 2 ** 63, n, dtype=np.uint64)
    d["kv_block_offset"] = rng.integers(0, n_blocks, n)
    d["num_kv_blocks"] = rng.choice([0, 1, 2, 7, 15, 16, 17, 31, 32, 33, 64, 1000, 65535], n)
    d["attention_flags"] = rng.integers(0, 256, n)
    d["output_token_offset"] = (offsets if offsets is not None else
                                rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32))
    d["reward_cookie"] = rng.integers(0, 2 ** 64 - 1, n, dtype=np.uint64)
    d["batch_size"] = rng.integers(0, 64, n)
    d["batch_index"] = rng.integers(0, 64, n)
    return d


def sample_state(dev, seed):
    st = np.zeros(48, np.uint8)
    st[:32] = np.random.default_rng(seed).integers(0, 256, 32, dtype=np.uint8)
    return torch.from_numpy(st).to(dev), st[:32].view(np.uint64).copy()


def check_tokens_vs_oracle(tok, o_orc, tok_orc):
    """Token ids equal the oracle's unless its top two outputs are within
    2e-4 (then the GPU's pick must be one of those near-maximal entries)."""
    diff = tok != tok_orc
    for i in np.nonzero(diff)[0]:
        row = o_orc[i]
        assert row[tok[i]] >= row.max() - 2e-4, (i, tok[i], tok_orc[i])
    assert diff.sum() <= max(2, len(tok) // 500)


def known_answer_inputs(orc):
    """The input pattern of reference test/test_bench.cu:91-107."""
    f16 = orc.oracle_lib().orc_f32_to_f16_rne
    q = np.array([f16(((d % 17) - 8) / 8.0) for d in range(128)], dtype=np.uint16)
    block = np.zeros(2 * 32 * 128, dtype=np.uint16)
    for t in range(32):
        for d in range(128):
            block[t * 128 + d] = f16((((t + 1) * ((d % 13) + 1)) % 23 - 11) / 32.0)
            block[4096 + t * 128 + d] = f16((((t + 3) * ((d % 11) + 5)) % 29 - 14) / 29.0)
    return q, block


def test_known_answer_pattern(pkg, orc, cuda):
    """Reference test/test_bench.cu:91-107 inputs, seq_len 17, slot 3."""
    q, block = known_answer_inputs(orc)
    arena_t = torch.from_numpy(block.view(np.uint8).copy()).to(cuda)
    arena = pkg.device_arena(arena_t, BLOCK)
    q_buf = torch.from_numpy(np.tile(q, (4, 1)).view(np.int16)).to(cuda).view(torch.float16)
    o_buf = torch.zeros(4, 128, dtype=torch.float32, device=cuda)
    d = np.zeros(1, orc.DESCRIPTOR_DTYPE)
    d["seq_id"], d["num_kv_blocks"], d["output_token_offset"] = 99, 17, 3
    res = pkg.attention_fixed128(d, arena, q_buffer=q_buf, o_buffer=o_buf, io_slots=4)
    got = o_buf[3].cpu().numpy()
    want, plain_tok = orc.fixed128_attention(q, block, 17)
    assert np.max(np.abs(got - want)) < ATOL
    # The pattern's V columns repeat with period 11 in d, so o has exact
    # ties (o[9] == o[20] == ... == o[119]).  The kernel's lane-then-stride
    # scan returns 64 (lane 0, third stride); the reference test's CPU
    # argmax returns the lowest index, 9, so its assertion
    # (test_bench.cu:720) disagrees with its own kernel on this input.
    assert plain_tok == 9
    comps, _, _ = orc.decode_steps(d, block.view(np.uint8), BLOCK, q_buf=np.tile(q, (4, 1)),
                                   io_slots=4)
    assert res["token_id"][0] == comps["token_id"][0] == 64
    assert res["path_kind"][0] == 1
    assert res["bytes_touched"][0] == 17 * 128 * 2 * 2
    assert res["tile_count"][0] == 2
    # the kernel's estimate (cu/attention_decode.cu:200); the reference test's
    # assertion seq_len*128*2 (test_bench.cu:722) disagrees with its own kernel
    assert res["cycle_estimate"][0] == 2 * 128 * 24
    try:
        ref = orc.RefCuda()
    except OSError as e:
        pytest.skip(str(e))
    r_o, r_tok, r_b, r_t, r_c = ref.fixed128(d, arena_t, BLOCK, q_buf=q_buf, io_slots=4)
    assert np.array_equal(r_o[0].view(np.uint32), got.view(np.uint32))
    assert (r_tok[0], r_b[0], r_t[0], r_c[0]) == (res["token_id"][0], res["bytes_touched"][0],
                                                  res["tile_count"][0], res["cycle_estimate"][0])


@pytest.mark.parametrize("q_mode", ["buffer", "synth", "synth_state"])
def test_step_matches_reference_kernel_and_oracle(pkg, orc, cuda, q_mode):
    n, n_blocks, slots = 3000, 97, 4096
    host, arena_t = make_arena(cuda, n_blocks, seed=3)
    arena = pkg.device_arena(arena_t, BLOCK)
    rng = np.random.default_rng(4)
    offsets = (rng.permutation(slots)[:n] + slots * rng.integers(0, 2 ** 19, n)).astype(np.uint32)
    d = make_descs(orc, n, n_blocks, seed=5, offsets=offsets)
    q_bits = None
    q_buf = ss = rng4 = None
    if q_mode == "buffer":
        q_bits = rng.standard_normal((slots, 128)).astype(np.float16).view(np.uint16)
        q_buf = torch.from_numpy(q_bits.view(np.int16)).to(cuda).view(torch.float16)
    elif q_mode == "synth_state":
        ss, rng4 = sample_state(cuda, 6)
    o_buf = torch.full((slots, 128), float("nan"), dtype=torch.float32, device=cuda)
    res = pkg.attention_fixed128(d, arena, sample_st=ss, q_buffer=q_buf, o_buffer=o_buf,
                                 io_slots=slots)
    slot = d["output_token_offset"] & (slots - 1)
    o = o_buf.cpu().numpy()[slot]
    comps, o_orc, bad = orc.decode_steps(d, host, BLOCK, rng4=rng4, q_buf=q_bits,
                                         io_slots=slots)
    assert bad == 0
    assert np.max(np.abs(o - o_orc)) < ATOL
    check_tokens_vs_oracle(res["token_id"], o_orc, comps["token_id"])
    assert np.array_equal(res["cycle_estimate"], comps["cycles_taken"])
    seq = np.minimum(np.maximum(d["num_kv_blocks"].astype(np.int64), 1), 32)
    assert np.array_equal(res["bytes_touched"], seq * 512)
    assert np.array_equal(res["tile_count"], (seq + 15) // 16)
    try:
        ref = orc.RefCuda()
    except OSError as e:
        pytest.skip(str(e))
    r_o, r_tok, r_b, r_t, r_c = ref.fixed128(d, arena_t, BLOCK, sample_st=ss, q_buf=q_buf,
                                             io_slots=slots)
    assert np.array_equal(r_o.view(np.uint32), o.view(np.uint32)), \
        f"max |diff| {np.max(np.abs(r_o - o)):.3e}"
    assert np.array_equal(r_tok, res["token_id"])
    assert np.array_equal(r_b, res["bytes_touched"])
    assert np.array_equal(r_t, res["tile_count"])
    assert np.array_equal(r_c, res["cycle_estimate"])


def test_argmax_ties_follow_the_reference_lane_order(pkg, orc, cuda):
    """Exact ties: V columns 5 and 64 equal and largest (block 0), 2 and 33
    (block 1).  The reference's lane-then-stride scan picks 64 and 33; a
    plain lowest-index argmax would pick 5 and 2."""
    rng = np.random.default_rng(8)
    blocks = (rng.standard_normal((2, 2, 32, 128)) * 0.1).astype(np.float16)
    blocks[0, 1, :, 5] = blocks[0, 1, :, 64] = 2.0
    blocks[1, 1, :, 2] = blocks[1, 1, :, 33] = 2.5
    host = blocks.reshape(-1).view(np.uint8)
    arena_t = torch.from_numpy(host.copy()).to(cuda)
    arena = pkg.device_arena(arena_t, BLOCK)
    d = make_descs(orc, 64, 2, seed=9)
    d["kv_block_offset"] = np.arange(64) % 2
    res = pkg.attention_fixed128(d, arena)
    want = np.where(d["kv_block_offset"] == 0, 64, 33)
    assert np.array_equal(res["token_id"], want)
    comps, _, _ = orc.decode_steps(d, host, BLOCK)
    assert np.array_equal(comps["token_id"], want)
    try:
        ref = orc.RefCuda()
    except OSError:
        return
    assert np.array_equal(ref.fixed128(d, arena_t, BLOCK)[1], want)


def run_worker(pkg, rings, arena, descs, n_sentinels=1, n_expected=None, stop_sentinels=1,
               idle_ms=20000, **kw):
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    pkg.launch_decode_worker(rings, arena, step_count=step, stop_sentinels=stop_sentinels,
                             idle_timeout_ms=idle_ms, **kw)
    n_expected = len(descs) if n_expected is None else n_expected
    n, raw = rings.pump(descs, n_sentinels, n_expected, timeout_ms=60000)
    torch.cuda.synchronize()
    stats = pkg.decode_worker_stats()
    return n, raw, int(step.item()), stats


def test_worker_over_rings_matches_oracle(pkg, orc, cuda):
    """20,000 descriptors (five laps of the 4,096-slot rings) with the
    synthesized query and a SampleState; completions arrive in ring order."""
    n, n_blocks = 20000, 61
    host, arena_t = make_arena(cuda, n_blocks, seed=11)
    arena = pkg.device_arena(arena_t, BLOCK)
    ss, rng4 = sample_state(cuda, 12)
    d = make_descs(orc, n, n_blocks, seed=13)
    rings = pkg.CommandRings()
    try:
        got, raw, steps, st = run_worker(pkg, rings, arena, d, sample_st=ss)
        assert got == n
        comps = raw.view(orc.COMPLETION_DTYPE)[:n]
        want, o_orc, _ = orc.decode_steps(d, host, BLOCK, rng4=rng4)
        for f in ("seq_id", "kv_block_offset", "reward_cookie", "cycles_taken"):
            assert np.array_equal(comps[f], want[f]), f
        check_tokens_vs_oracle(comps["token_id"], o_orc, want["token_id"])
        assert steps == n
        assert st["consumed"] == n + 1 and st["completed"] == n and st["sentinels"] == 1
        assert st["error"] == 0 and st["finished"] == 1 and st["workers"] > 0
        assert rings.header("cmd") == (n + 1, n + 1)
        assert rings.header("comp")[:2] == (n, n)
        # same tokens as the stateless batch launcher (which the GPU-vs-GPU
        # test pins to the reference kernel)
        res = pkg.attention_fixed128(d, arena, sample_st=ss)
        assert np.array_equal(res["token_id"], comps["token_id"])
    finally:
        rings.close()


def test_worker_q_and_o_buffers(pkg, orc, cuda):
    n, n_blocks, slots = 3000, 40, 4096
    host, arena_t = make_arena(cuda, n_blocks, seed=21)
    arena = pkg.device_arena(arena_t, BLOCK)
    rng = np.random.default_rng(22)
    q_bits = rng.standard_normal((slots, 128)).astype(np.float16).view(np.uint16)
    q_buf = torch.from_numpy(q_bits.view(np.int16)).to(cuda).view(torch.float16)
    o_buf = torch.zeros(slots, 128, dtype=torch.float32, device=cuda)
    offsets = rng.permutation(slots)[:n].astype(np.uint32)
    d = make_descs(orc, n, n_blocks, seed=23, offsets=offsets)
    rings = pkg.CommandRings()
    try:
        got, raw, steps, st = run_worker(pkg, rings, arena, d, q_buffer=q_buf, o_buffer=o_buf,
                                         io_slots=slots)
        assert got == n and steps == n and st["error"] == 0
        comps = raw.view(orc.COMPLETION_DTYPE)[:n]
        want, o_orc, _ = orc.decode_steps(d, host, BLOCK, q_buf=q_bits, io_slots=slots)
        o = o_buf.cpu().numpy()[offsets]
        assert np.max(np.abs(o - o_orc)) < ATOL
        check_tokens_vs_oracle(comps["token_id"], o_orc, want["token_id"])
        assert np.array_equal(comps["cycles_taken"], want["cycles_taken"])
    finally:
        rings.close()


def test_worker_stops_at_the_nth_sentinel(pkg, orc, cuda):
    """stop_sentinels = 3: work between the sentinels is done, the records
    behind the third stay in the ring (one reference worker warp exits per
    sentinel)."""
    host, arena_t = make_arena(cuda, 8, seed=31)
    arena = pkg.device_arena(arena_t, BLOCK)
    parts = [make_descs(orc, k, 8, seed=32 + k) for k in (100, 50, 20, 30)]
    stop = np.zeros(1, orc.DESCRIPTOR_DTYPE)
    stop["seq_id"] = np.uint64(2 ** 64 - 1)
    stream = np.concatenate([parts[0], stop, parts[1], stop, parts[2], stop, parts[3]])
    rings = pkg.CommandRings()
    try:
        got, raw, steps, st = run_worker(pkg, rings, arena, stream, n_sentinels=0,
                                         n_expected=170, stop_sentinels=3)
        assert got == 170 and steps == 170
        comps = raw.view(orc.COMPLETION_DTYPE)[:170]
        want = np.concatenate(parts[:3])
        assert np.array_equal(comps["seq_id"], want["seq_id"])
        assert st["sentinels"] == 3 and st["consumed"] == 173 and st["error"] == 0
        assert rings.header("cmd") == (173, 203)
    finally:
        rings.close()


def test_worker_idle_timeout_is_reported(pkg, orc, cuda):
    """No stop sentinel ever arrives: the worker gives up after its idle
    limit with RT_ETIMEOUT, having delivered the work it got."""
    host, arena_t = make_arena(cuda, 4, seed=41)
    arena = pkg.device_arena(arena_t, BLOCK)
    d = make_descs(orc, 10, 4, seed=42)
    rings = pkg.CommandRings()
    try:
        t0 = time.time()
        got, raw, steps, st = run_worker(pkg, rings, arena, d, n_sentinels=0, idle_ms=300)
        assert got == 10 and steps == 10
        assert st["error"] == RT_ETIMEOUT and st["finished"] == 1 and st["completed"] == 10
        assert time.time() - t0 < 30
    finally:
        rings.close()


def test_worker_flags_a_block_outside_the_arena(pkg, orc, cuda):
    host, arena_t = make_arena(cuda, 16, seed=51)
    arena = pkg.device_arena(arena_t, BLOCK)
    d = make_descs(orc, 200, 16, seed=52)
    d["kv_block_offset"][77] = 21
    rings = pkg.CommandRings()
    try:
        got, raw, steps, st = run_worker(pkg, rings, arena, d)
        assert got == 200
        comps = raw.view(orc.COMPLETION_DTYPE)[:200]
        want, o_orc, bad = orc.decode_steps(d, host, BLOCK)
        assert bad == 1
        assert comps["token_id"][77] == 0xFFFFFFFF and comps["cycles_taken"][77] == 0
        assert np.array_equal(comps["cycles_taken"], want["cycles_taken"])
        assert st["error"] == RT_EDEVICE and st["bad_block"] == 21
    finally:
        rings.close()


def test_worker_waits_on_a_full_completion_ring(pkg, orc, cuda):
    """6,000 completions with nobody draining: the worker holds them (ring
    full, counted once per stall), then delivers all in order."""
    n = 6000
    host, arena_t = make_arena(cuda, 8, seed=61)
    arena = pkg.device_arena(arena_t, BLOCK)
    d = make_descs(orc, n, 8, seed=62)
    rings = pkg.CommandRings()
    try:
        step = torch.zeros(1, dtype=torch.int64, device=cuda)
        pkg.launch_decode_worker(rings, arena, step_count=step, idle_timeout_ms=20000)
        pushed, _ = rings.pump(d, 1, 0)
        time.sleep(0.3)
        head, tail, overflow = rings.header("comp")
        assert tail - head == 4096 and overflow >= 1
        got, raw = rings.pump(d[:0], 0, n)
        torch.cuda.synchronize()
        st = pkg.decode_worker_stats()
        assert got == n and int(step.item()) == n
        comps = raw.view(orc.COMPLETION_DTYPE)[:n]
        assert np.array_equal(comps["seq_id"], d["seq_id"])
        assert st["comp_ring_full"] >= 1 and st["error"] == 0
    finally:
        rings.close()


def test_second_launch_while_running_is_refused(pkg, orc, cuda):
    host, arena_t = make_arena(cuda, 2, seed=71)
    arena = pkg.device_arena(arena_t, BLOCK)
    rings = pkg.CommandRings()
    try:
        pkg.launch_decode_worker(rings, arena, idle_timeout_ms=5000)
        with pytest.raises(pkg.RuntimeErrorRT, match="still running"):
            pkg.launch_decode_worker(rings, arena, idle_timeout_ms=5000)
        got, _ = rings.pump(make_descs(orc, 5, 2, seed=72), 1, 5)
        torch.cuda.synchronize()
        assert got == 5 and pkg.decode_worker_stats()["error"] == 0
    finally:
        rings.close()
