"""Drop-in parity of the C API on CPU.

oracle/harness/abi_caller.c is one C caller compiled twice: against the
reference's headers + sources (oracle/_ref) and against include/*.h +
librlrt_b200.so.  Every scripted call sequence must give byte-identical
results; the golden fixtures (tests/golden/golden.json, generated from the
reference build by tests/golden/make_golden.py) pin the same values where
the reference tree is absent.
"""
import hashlib

import numpy as np
import pytest


def rec(a):
    return {k: int(a[k]) for k in a.dtype.names}


def test_c1_stream_matches_reference_golden(mine, golden):
    g = golden["c1"]
    descs = mine.gen_c1(g["n"], seed=g["seed"], max_tokens=g["max_tokens"])
    assert hashlib.sha256(descs.tobytes()).hexdigest() == g["sha256_input"]
    done, tokens, comps, _ = mine.run_c1(descs, depth_cap=g["depth_cap"])
    assert len(done) == g["n_done"]
    assert tokens == g["decoded_tokens"] and comps == g["completions"]
    assert [rec(d) for d in done[:8]] == g["done_head"]
    assert [rec(d) for d in done[-4:]] == g["done_tail"]
    assert hashlib.sha256(done.tobytes()).hexdigest() == g["sha256_done"]


@pytest.mark.parametrize("cap,bell", [(1, 1), (7, 3), (1024, 32), (65536, 64)])
def test_c1_stream_independent_of_backpressure(mine, ref, cap, bell):
    descs = mine.gen_c1(3000, seed=5, max_tokens=300)
    a, ta, ca, _ = mine.run_c1(descs, depth_cap=cap, doorbell_batch=bell)
    b, tb, cb, _ = ref.run_c1(descs, depth_cap=cap, doorbell_batch=bell)
    assert a.tobytes() == b.tobytes() and (ta, ca) == (tb, cb)


def test_c1_stream_equals_oracle_restatement(mine, orc):
    descs = mine.gen_c1(5000, seed=9, max_tokens=1000)
    # mix in non-DECODE opcodes: they must be dropped without a completion
    descs["opcode"][::97] = 2
    descs["opcode"][::131] = 3
    done, tokens, _, _ = mine.run_c1(descs, depth_cap=512)
    odone, otokens = orc.worker_sim_stream(descs)
    assert done.tobytes() == odone.tobytes() and tokens == otokens


def test_submit_known_answers(mine, golden):
    for k in golden["submit"]:
        rc, bell, d = mine.kat_submit(*k["args"])
        assert (rc, bell, rec(d)) == (k["rc"], k["doorbell"], k["desc"])
    first = golden["submit"][0]
    # reference test/test_hw_ring.c:116-125
    assert first["doorbell"] == 1 and first["desc"]["flags"] & 4
    assert mine.kat_submit_errors() == golden["submit_errors"] == [-1, -1, -1, -1]


def test_submit_matches_oracle_fill(mine, orc):
    for args in [(1, 2, 3, 4, 5, 0, 6, 7), (9, 9, 2**32 - 1, 2**63, 17, 4, 0, 1)]:
        rc, _, d = mine.kat_submit(*args)
        o = np.zeros(1, orc.HW_DESC_DTYPE)
        orc.oracle_lib().orc_submit_desc(args[0], args[1], args[2], args[3], args[4], args[5],
                                         args[6], args[7], o.ctypes.data)
        assert rc == 0 and d.tobytes() == o[0].tobytes()


def test_hw_ring_invariants(mine, golden):
    assert mine.lib.hx_kat_hw_ring() == golden["hw_ring_mask"] == 0x3F


def test_worker_known_answers(mine, golden):
    for k in golden["worker"]:
        d = np.zeros(1, mine_dtype(mine))[0]
        for f, v in k["in"].items():
            d[f] = v
        rc, out, tok, comp = mine.kat_worker(d)
        assert (rc, rec(out), tok, comp) == (k["rc"], k["out"], k["tokens"], k["completions"])
    # reference test/test_hw_ring.c:168-217 and RTL tb_rl_runtime_top.sv:80-147
    w = {k["in"]["rollout_id"]: k["out"] for k in golden["worker"]}
    assert w[77]["seq_len"] == 32 and w[77]["flags"] == 1      # NEEDS_REWARD
    assert w[7]["seq_len"] == 10 and w[7]["flags"] == 2        # DONE
    assert w[9]["seq_len"] == 32 and w[9]["flags"] == 1
    assert w[11]["seq_len"] == 12 and w[11]["flags"] == 2
    assert w[5]["seq_len"] == 64 and w[5]["flags"] == 0        # already at max: echoed


def mine_dtype(mine):
    import __graft_entry__ as ge
    return ge.load_oracle().HW_DESC_DTYPE


@pytest.mark.parametrize("name", ["command_ring", "kv_prefix", "arena"])
def test_scripts_match_reference(mine, golden, name):
    if name == "command_ring":
        import __graft_entry__ as ge
        batch = np.zeros(3, dtype=ge.load_oracle().DESCRIPTOR_DTYPE)
        log = mine.script("hx_script_command_ring", batch)
        assert [int(x) for x in log] == golden["command_ring_log"]
        assert [rec(b) for b in batch] == golden["command_ring_batch"]
    elif name == "kv_prefix":
        assert [int(x) for x in mine.script("hx_script_kv_prefix")] == golden["kv_prefix_log"]
    else:
        assert [int(x) for x in mine.script("hx_script_arena_bitmap", 4096)] == golden["arena_log"]


def test_request_and_reward_rings(mine, golden, orc):
    req = np.zeros(1, dtype=orc.REQUEST_DTYPE)
    dn = np.zeros(1, dtype=orc.DONE_DTYPE)
    assert [int(x) for x in mine.script("hx_script_request_ring", req, dn)] == golden["request_ring_log"]
    assert int(req[0]["request_id"]) == golden["request_ring_req"]["request_id"]
    scores = np.zeros(600, dtype=np.float32)
    assert [int(x) for x in mine.script("hx_script_reward", scores)] == golden["reward_log"]
    assert hashlib.sha256(scores.tobytes()).hexdigest() == golden["reward_scores_sha256"]


def test_arena_never_exceeds_capacity(mine):
    log = mine.script("hx_script_arena_bitmap", 10)
    # capacity of 10 blocks: ids 0..9 then -1 (the reference hands out ids
    # past the allocation; this runtime bounds them)
    assert [int(x) for x in log[:11]] == list(range(10)) + [-1]


def test_completion_wire_record(pkg, mine, golden):
    """The 64-byte completion wire record (hw_desc.h): the done descriptor
    byte for byte with the completion status in the high byte of flags; it
    decodes to the compact completion_t of the RTL."""
    import ctypes
    import __graft_entry__ as ge
    dt = ge.load_oracle().HW_DESC_DTYPE
    lib = pkg.lib()
    enc, dec = lib.hw_completion_wire_encode, lib.hw_completion_wire_decode
    enc.argtypes = dec.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    enc.restype = dec.restype = None
    descs = mine.gen_c1(2000, seed=3, max_tokens=300)
    done, _, _, _ = mine.run_c1(descs, depth_cap=256)
    stop = np.zeros(1, dt)
    stop["opcode"], stop["rollout_id"], stop["seq_len"] = 255, 70000, 5
    recs = np.concatenate([done, stop])
    for d in recs:
        d = np.array([d], dt)
        w = np.zeros(1, dt)
        enc(d.ctypes.data, w.ctypes.data)
        f = int(d["flags"][0])
        want = (0xFF if d["opcode"][0] == 255 else 1 if f & 2 else 2 if f & 1 else 0)
        assert int(w["flags"][0]) == (f & 0xFF) | (want << 8)
        a, b = d.copy(), w.copy()
        a["flags"] = b["flags"] = 0
        assert a.tobytes() == b.tobytes()  # every other field at its offset, unchanged
        c = pkg.completion_t()
        dec(w.ctypes.data, ctypes.addressof(c))
        assert (c.rollout_id, c.status, c.final_seq_len, c.reward_id) == (
            int(d["rollout_id"][0]) & 0xFFFF, want, int(d["seq_len"][0]) & 0xFFFF,
            int(d["reward_model_id"][0]) & 0xFFFF)
    # RTL known answers (reference rtl/tb_rl_runtime_top.sv:80-147) through the wire
    w_out = {k["in"]["rollout_id"]: k["out"] for k in golden["worker"]}
    for rid, status, seq in [(77, 2, 32), (7, 1, 10), (11, 1, 12), (5, 0, 64)]:
        d = np.zeros(1, dt)
        for f, v in w_out[rid].items():
            d[f] = v
        w = np.zeros(1, dt)
        enc(d.ctypes.data, w.ctypes.data)
        c = pkg.completion_t()
        dec(w.ctypes.data, ctypes.addressof(c))
        assert (c.rollout_id, c.status, c.final_seq_len) == (rid, status, seq)
