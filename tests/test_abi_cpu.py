"""The C-ABI library loads on CPU and exports every function include/*.h
declares; record layouts seen through ctypes match the headers."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")

# Declared in headers but defined inline there (no exported symbol).
INLINE_ONLY = set()


def declared_functions():
    names = set()
    pat = re.compile(r"^[A-Za-z_][\w \*]*?\b([a-z_][a-z0-9_]*)\s*\(", re.M)
    for fn in sorted(os.listdir(INCLUDE)):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(INCLUDE, fn)).read()
        src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)      # drop comments
        src = re.sub(r"//[^\n]*", " ", src)
        # only prototypes inside extern "C" blocks are exported functions
        for block in re.findall(r'extern "C" \{\s*#endif(.*?)#ifdef __cplusplus\s*\}', src, re.S):
            block = "\n".join(l for l in block.split("\n") if not l.strip().startswith("#"))
            for decl in block.split(";"):
                decl = " ".join(decl.split())
                if decl.startswith(("typedef", "#")) or "{" in decl or "}" in decl:
                    continue
                m = pat.search(decl)
                if m:
                    names.add(m.group(1))
    return sorted(names)


def test_headers_declare_reference_symbols():
    names = set(declared_functions())
    for sym in ["infer_submit_decode", "hw_ring_create", "hw_ring_reset", "hw_ring_destroy",
                "hw_ring_load_acquire", "hw_ring_store_release", "hw_worker_sim_run",
                "ring_create", "ring_destroy", "comp_ring_create", "comp_ring_destroy",
                "decode_batch_reset", "decode_batch_push", "decode_batch_submit",
                "decode_batch_contract", "arena_init", "arena_acquire", "arena_release",
                "arena_destroy", "kv_prefix_table_init", "kv_prefix_register", "kv_prefix_acquire",
                "kv_prefix_release", "kv_prefix_get", "kv_branch_alloc", "kv_branch_free",
                "kv_branch_get", "kv_branch_total_offset", "reward_ring_init", "reward_push",
                "reward_pop", "reward_score_mock", "attention_decode_config_fixed128"]:
        assert sym in names, sym


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    missing = [n for n in declared_functions() if n not in INLINE_ONLY and not hasattr(lib, n)]
    assert not missing, missing


def test_record_sizes(pkg):
    assert ctypes.sizeof(pkg.hw_desc_t) == 64
    assert ctypes.sizeof(pkg.completion_t) == 7
    assert ctypes.sizeof(pkg.Descriptor) == 32
    assert ctypes.sizeof(pkg.Completion) == 32
    assert ctypes.sizeof(pkg.RolloutRequest) == 34
    assert ctypes.sizeof(pkg.RolloutDone) == 24
    assert ctypes.sizeof(pkg.GpuRolloutSlot) == 72
    assert ctypes.sizeof(pkg.GpuRolloutState) == 72 * 256 + 32


def test_fixed128_config(pkg):
    class Cfg(ctypes.Structure):
        _fields_ = [(n, ctypes.c_uint32) for n in
                    ("head_dim", "tokens_per_block", "tile_tokens", "prefetch_stages", "shared_bytes")]
    f = pkg.lib().attention_decode_config_fixed128
    f.restype = Cfg
    c = f()
    assert (c.head_dim, c.tokens_per_block, c.tile_tokens, c.prefetch_stages, c.shared_bytes) == \
        (128, 32, 16, 3, 3 * 16384)


def test_attention_params_validation_on_cpu(pkg):
    p = pkg.rt_attn_params_t(64, 32, 8, 128, 256, 4096, 100000, 128 ** -0.5, 0, 0)
    assert pkg.lib().rt_attn_workspace_bytes(ctypes.byref(p)) > 0
    bad = pkg.rt_attn_params_t(64, 32, 8, 64, 256, 4096, 100000, 1.0, 0)
    assert pkg.lib().rt_attn_workspace_bytes(ctypes.byref(bad)) == 0
    assert b"head_dim" in pkg.lib().rt_last_error()
    bad = pkg.rt_attn_params_t(64, 24, 8, 128, 256, 4096, 100000, 1.0, 0)  # group 3
    assert pkg.lib().rt_attn_workspace_bytes(ctypes.byref(bad)) == 0
    bad = pkg.rt_attn_params_t(64, 32, 8, 128, 16, 4096, 100000, 1.0, 0)   # 16 pages < 4096 tok
    assert pkg.lib().rt_attn_workspace_bytes(ctypes.byref(bad)) == 0
    cp, mc, ctas = pkg.PagedDecodeAttention.plan(type("X", (), {"params": p})())
    # 48-page items would leave fewer than two per warp slot (148 SMs x 3 CTAs
    # x 4 warps), so the plan halves them to 24
    assert cp == 24 and mc == 11 and ctas == min(11 * 8 * 64 // 4, 148 * 3)
