"""Regenerate tests/golden/golden.json from the reference's own C code.

Run in a container where the reference tree is mounted and oracle/_ref has
been built (`make -C oracle`):  python tests/golden/make_golden.py

Every value comes from oracle/_ref/libabi_ref.so, i.e. the caller harness
compiled against the reference's headers and linked with the reference's
unmodified C sources.  The CPU tests compare this repository's library
against these fixtures (and against the live reference build when present).
"""
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402


def rec(a):
    return {k: int(a[k]) for k in a.dtype.names}


def main():
    orc = ge.load_oracle()
    ref = orc.Harness("ref")
    g = {"source": "reference C sources via oracle/_ref/libabi_ref.so"}

    descs = ref.gen_c1(10000, seed=0, max_tokens=2048)
    done, tokens, comps, _ = ref.run_c1(descs, depth_cap=1024)
    g["c1"] = {
        "n": 10000, "seed": 0, "max_tokens": 2048, "depth_cap": 1024,
        "sha256_input": hashlib.sha256(descs.tobytes()).hexdigest(),
        "sha256_done": hashlib.sha256(done.tobytes()).hexdigest(),
        "n_done": int(len(done)), "decoded_tokens": tokens, "completions": comps,
        "done_head": [rec(d) for d in done[:8]],
        "done_tail": [rec(d) for d in done[-4:]],
    }

    kats = []
    for args in [(7, 42, 99, 0x1000, 0x2000, 5, 17, 64), (3, 11, 1, 0x1000, 0x2000, 7, 16, 64),
                 (0, 0, 0xFFFFFFFF, 2**64 - 1, 0x55, 0, 0xFFFFFFFF, 0)]:
        rc, bell, d = ref.kat_submit(*args)
        kats.append({"args": list(args), "rc": rc, "doorbell": bell, "desc": rec(d)})
    g["submit"] = kats
    g["submit_errors"] = ref.kat_submit_errors()
    g["hw_ring_mask"] = int(ref.lib.hx_kat_hw_ring())

    worker = []
    for rid, seq, mx in [(77, 31, 96), (7, 0, 10), (9, 0, 40), (11, 8, 12), (5, 64, 64),
                         (6, 63, 64), (8, 95, 200), (4, 0xFFFFFFF0, 0xFFFFFFFF)]:
        d = np.zeros(1, dtype=orc.HW_DESC_DTYPE)[0]
        d["opcode"], d["rollout_id"], d["seq_len"], d["max_tokens"] = 1, rid, seq, mx
        d["reward_model_id"] = rid % 7
        rc, out, tok, comp = ref.kat_worker(d)
        worker.append({"in": rec(d), "rc": rc, "out": rec(out), "tokens": tok, "completions": comp})
    g["worker"] = worker

    batch = np.zeros(3, dtype=orc.DESCRIPTOR_DTYPE)
    g["command_ring_log"] = [int(x) for x in ref.script("hx_script_command_ring", batch)]
    g["command_ring_batch"] = [rec(b) for b in batch]
    req = np.zeros(1, dtype=orc.REQUEST_DTYPE)
    dn = np.zeros(1, dtype=orc.DONE_DTYPE)
    g["request_ring_log"] = [int(x) for x in ref.script("hx_script_request_ring", req, dn)]
    g["request_ring_req"] = rec(req[0]) | {"top_p": float(req[0]["top_p"])}
    g["kv_prefix_log"] = [int(x) for x in ref.script("hx_script_kv_prefix")]
    scores = np.zeros(600, dtype=np.float32)
    g["reward_log"] = [int(x) for x in ref.script("hx_script_reward", scores)]
    g["reward_scores_sha256"] = hashlib.sha256(scores.tobytes()).hexdigest()
    g["arena_log"] = [int(x) for x in ref.script("hx_script_arena_bitmap", 4096)]

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(out, "w") as f:
        json.dump(g, f, indent=1)
    print("wrote", out)


if __name__ == "__main__":
    main()
