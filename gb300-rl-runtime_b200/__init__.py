"""Python mirror of the rollout runtime's C ABI (include/*.h, include/rlrt.h).

The product is ``librlrt_b200.so`` in this directory: host C plus sm_100a CUDA
behind ``extern "C"`` entry points.  This module only binds those entry points
with ctypes and wraps device buffers given as torch tensors (torch supplies
device memory and streams; it is not part of the compute path).  Importing it
fails loudly if the shared library has not been built - there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librlrt_b200.so")

RT_OK, RT_EINVAL, RT_ECUDA, RT_ETIMEOUT, RT_ENOMEM, RT_EDEVICE = 0, -1, -2, -3, -4, -5
RT_ARRIVAL_PASS, RT_ARRIVAL_NS = 0, 1

# ----------------------------------------------------------------- records
class hw_desc_t(ctypes.Structure):
    _pack_ = 1
    _fields_ = [
        ("opcode", ctypes.c_uint16), ("flags", ctypes.c_uint16),
        ("rollout_id", ctypes.c_uint32), ("kv_arena_id", ctypes.c_uint32),
        ("prefix_id", ctypes.c_uint32), ("kv_offset", ctypes.c_uint64),
        ("delta_offset", ctypes.c_uint64), ("seq_len", ctypes.c_uint32),
        ("max_tokens", ctypes.c_uint32), ("reward_model_id", ctypes.c_uint32),
        ("reserved0", ctypes.c_uint32), ("user_data", ctypes.c_uint64),
        ("checksum_or_cookie", ctypes.c_uint64),
    ]


class completion_t(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("rollout_id", ctypes.c_uint16), ("status", ctypes.c_uint8),
                ("final_seq_len", ctypes.c_uint16), ("reward_id", ctypes.c_uint16)]


class Descriptor(ctypes.Structure):
    _pack_ = 1
    _fields_ = [
        ("seq_id", ctypes.c_uint64), ("kv_block_offset", ctypes.c_uint32),
        ("num_kv_blocks", ctypes.c_uint16), ("attention_flags", ctypes.c_uint8),
        ("pad", ctypes.c_uint8), ("output_token_offset", ctypes.c_uint32),
        ("reward_cookie", ctypes.c_uint64), ("batch_size", ctypes.c_uint16),
        ("batch_index", ctypes.c_uint16),
    ]


class Completion(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("seq_id", ctypes.c_uint64), ("token_id", ctypes.c_uint32),
                ("kv_block_offset", ctypes.c_uint32), ("reward_cookie", ctypes.c_uint64),
                ("cycles_taken", ctypes.c_uint64)]


class RolloutRequest(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("request_id", ctypes.c_uint64), ("max_tokens", ctypes.c_uint32),
                ("kv_blocks", ctypes.c_uint32), ("temperature", ctypes.c_float),
                ("top_k", ctypes.c_uint16), ("top_p", ctypes.c_float),
                ("rng_seed", ctypes.c_uint64)]


class RolloutDone(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("request_id", ctypes.c_uint64), ("rollout_id", ctypes.c_uint32),
                ("tokens_generated", ctypes.c_uint32), ("reward", ctypes.c_float),
                ("status", ctypes.c_uint32)]


class GpuRolloutSlot(ctypes.Structure):
    _fields_ = [("active", ctypes.c_uint32), ("request_id", ctypes.c_uint32),
                ("tokens_generated", ctypes.c_uint32), ("max_tokens", ctypes.c_uint32),
                ("kv_blocks", ctypes.c_uint32), ("rng_state", ctypes.c_uint64 * 4),
                ("temperature", ctypes.c_float), ("top_k", ctypes.c_uint16),
                ("top_p", ctypes.c_float)]


class GpuRolloutState(ctypes.Structure):
    _fields_ = [("slots", GpuRolloutSlot * 256), ("bitmap", ctypes.c_uint64 * 4)]


class rt_attn_params_t(ctypes.Structure):
    _fields_ = [("num_seqs", ctypes.c_uint32), ("num_q_heads", ctypes.c_uint32),
                ("num_kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("max_pages_per_seq", ctypes.c_uint32), ("max_seq_len", ctypes.c_uint32),
                ("arena_pages", ctypes.c_uint64), ("scale", ctypes.c_float),
                ("chunk_pages", ctypes.c_uint32), ("kv_evict_first", ctypes.c_uint32)]


class rt_attn_group_t(ctypes.Structure):
    _fields_ = [("n_members", ctypes.c_uint32), ("shared_pages", ctypes.c_uint32),
                ("members", ctypes.c_uint32 * 16)]


class rt_attn_group_params_t(ctypes.Structure):
    _fields_ = [("max_groups", ctypes.c_uint32), ("max_shared_pages", ctypes.c_uint32),
                ("chunk_pages", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class rt_sample_row_t(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32),
                ("top_p", ctypes.c_float), ("rollout_id", ctypes.c_uint32),
                ("step", ctypes.c_uint64), ("seed", ctypes.c_uint64)]


class rt_sample_params_t(ctypes.Structure):
    _fields_ = [("num_rows", ctypes.c_uint32), ("vocab", ctypes.c_uint32),
                ("row_stride", ctypes.c_uint64), ("fused_cum", ctypes.c_uint32),
                ("row_enable", ctypes.c_void_p)]


class KVArena(ctypes.Structure):
    _fields_ = [("base", ctypes.c_void_p), ("capacity", ctypes.c_size_t),
                ("block_size", ctypes.c_size_t), ("bitmap", ctypes.c_uint64 * 16384)]


class rt_rollout_config_t(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "num_q_heads", "num_kv_heads", "vocab", "max_slots", "max_context", "max_new_tokens",
        "max_admit", "drop_when_full", "decode_mode", "reward_mode")] + [
        ("reward_seed", ctypes.c_uint64), ("logit_std", ctypes.c_float),
        ("max_prefixes", ctypes.c_uint32), ("max_prefix_pages", ctypes.c_uint32),
        ("max_passes", ctypes.c_uint64), ("idle_timeout_ms", ctypes.c_uint32),
        ("chunk_pages", ctypes.c_uint32), ("prefix_attention", ctypes.c_uint32)]


class rt_rollout_io_t(ctypes.Structure):
    _fields_ = [("ring", ctypes.c_void_p), ("requests", ctypes.c_void_p),
                ("n_requests", ctypes.c_uint32), ("done_ring", ctypes.c_void_p),
                ("dones", ctypes.c_void_p), ("state", ctypes.c_void_p),
                ("step_count", ctypes.c_void_p), ("trajectories", ctypes.c_void_p),
                ("rewards", ctypes.c_void_p), ("n_rows", ctypes.c_uint32),
                ("arrival_unit", ctypes.c_uint32), ("arrivals", ctypes.c_void_p)]


class rt_rollout_stats_t(ctypes.Structure):
    _fields_ = [("passes", ctypes.c_uint64), ("tokens", ctypes.c_uint64),
                ("consumed", ctypes.c_uint32), ("admitted", ctypes.c_uint32),
                ("dropped", ctypes.c_uint32), ("done", ctypes.c_uint32),
                ("max_active", ctypes.c_uint32), ("stopped_by_sentinel", ctypes.c_uint32),
                ("error", ctypes.c_int32), ("attn_error", ctypes.c_int32),
                ("model_error", ctypes.c_int32), ("pad", ctypes.c_uint32)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_ if n != "pad"}


class rt_rollout_buffers_t(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "attn_out", "page_table", "seq_lens",
                                               "groups", "n_groups", "skip_pages")] + [
        ("max_pages", ctypes.c_uint32), ("max_groups", ctypes.c_uint32)] + [
        (n, ctypes.c_void_p) for n in ("logits", "tokens", "enable", "sample_rows", "hidden_in",
                                       "qkv", "hidden_out", "embed_tokens")]


class rt_model_weights_t(ctypes.Structure):
    _fields_ = [("embed", ctypes.c_void_p), ("w_qkv", ctypes.c_void_p), ("w_lm", ctypes.c_void_p),
                ("d_model", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class rt_gemm_params_t(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("M", "N", "K", "lda", "ldb", "ldc", "split_k",
                                               "flags")]


class rt_decode_worker_stats_t(ctypes.Structure):
    _fields_ = [("consumed", ctypes.c_uint64), ("completed", ctypes.c_uint64)] + [
        (n, ctypes.c_uint32) for n in ("published", "sentinels", "comp_ring_full")] + [
        ("error", ctypes.c_int32)] + [
        (n, ctypes.c_uint32) for n in ("bad_block", "workers", "finished", "pad")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_ if n != "pad"}


PASS_HOOK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64)


class rt_rollout_profile_t(ctypes.Structure):
    _fields_ = [("passes", ctypes.c_uint64), ("attn_launches", ctypes.c_uint64),
                ("sample_rows", ctypes.c_uint64)] + [
        (n, ctypes.c_double) for n in ("ms_schedule", "ms_prepare", "ms_attention", "ms_logits",
                                       "ms_sample", "attn_bytes_logical", "attn_bytes_unique")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


# ------------------------------------------------------------------ loader
_lib = None

_P = ctypes.c_void_p
_SIGS = {
    "rt_last_error": (ctypes.c_char_p, []),
    "rt_version": (ctypes.c_char_p, []),
    "rt_attn_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(rt_attn_params_t)]),
    "rt_attn_workspace_init": (ctypes.c_int, [_P, ctypes.c_size_t, _P]),
    "rt_attn_plan": (ctypes.c_int, [ctypes.POINTER(rt_attn_params_t),
                                    ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.POINTER(ctypes.c_uint64)]),
    "rt_paged_decode_attention": (ctypes.c_int, [ctypes.POINTER(rt_attn_params_t), _P, _P, _P,
                                                 _P, _P, _P, ctypes.c_size_t, _P]),
    "rt_attn_grouped_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(rt_attn_params_t),
                                                          ctypes.POINTER(rt_attn_group_params_t)]),
    "rt_paged_decode_attention_grouped": (ctypes.c_int, [ctypes.POINTER(rt_attn_params_t),
                                                         ctypes.POINTER(rt_attn_group_params_t)]
                                          + [_P] * 9 + [ctypes.c_size_t, _P]),
    "rt_attn_workspace_error": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_int32)]),
    "rt_sample_rows": (ctypes.c_int, [ctypes.POINTER(rt_sample_params_t), _P, _P, _P, _P]),
    "rt_sample_uniform24": (ctypes.c_uint32, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64]),
    "rt_chunk_max_stride": (ctypes.c_uint32, [ctypes.c_uint32]),
    "rt_logits_chunk_max": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64,
                                           _P, ctypes.c_uint32, _P]),
    "rt_sample_rows_cmax": (ctypes.c_int, [ctypes.POINTER(rt_sample_params_t), _P, _P,
                                           ctypes.c_uint32, _P, _P, _P]),
    "rt_rollout_create": (ctypes.c_int, [ctypes.POINTER(rt_rollout_config_t),
                                         ctypes.POINTER(KVArena), ctypes.POINTER(_P)]),
    "rt_rollout_destroy": (ctypes.c_int, [_P]),
    "rt_rollout_set_prefix": (ctypes.c_int, [_P, ctypes.c_uint32, _P, ctypes.c_uint32,
                                             ctypes.c_uint32]),
    "rt_rollout_launch": (ctypes.c_int, [_P, ctypes.POINTER(rt_rollout_io_t), _P]),
    "rt_rollout_profile": (ctypes.c_int, [_P, ctypes.POINTER(rt_rollout_io_t), _P,
                                          ctypes.POINTER(rt_rollout_profile_t)]),
    "rt_rollout_profile_hook": (ctypes.c_int, [_P, ctypes.POINTER(rt_rollout_io_t), _P,
                                               ctypes.POINTER(rt_rollout_profile_t), _P, _P]),
    "rt_rollout_buffers": (ctypes.c_int, [_P, ctypes.POINTER(rt_rollout_buffers_t)]),
    "rt_reward_score": (ctypes.c_int, [_P, ctypes.c_uint32, _P, _P]),
    "rt_kv_branch_resolve": (ctypes.c_int, [_P, _P, _P, ctypes.c_uint32, _P]),
    "rt_paged_decode_attention_noalloc": (ctypes.c_int, [ctypes.POINTER(rt_attn_params_t)]
                                          + [_P] * 6),
    "rt_paged_decode_attention_noalloc_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32),
                                                               _P]),
    "rt_grpo_advantages": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_float,
                                          _P, _P]),
    "rt_nccl_unique_id": (ctypes.c_int, [_P]),
    "rt_nccl_init": (ctypes.c_int, [ctypes.POINTER(_P), ctypes.c_int, _P, ctypes.c_int]),
    "rt_nccl_destroy": (ctypes.c_int, [_P]),
    "rt_reward_allgather": (ctypes.c_int, [_P, _P, _P, ctypes.c_uint64, _P]),
    "rt_nccl_wait": (ctypes.c_int, [_P, _P, ctypes.c_uint32]),
    "rt_rollout_wait": (ctypes.c_int, [_P, _P, ctypes.POINTER(rt_rollout_stats_t)]),
    "rt_logits_synth": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
                                       ctypes.c_uint64, ctypes.c_float, _P]),
    "rt_launch_rollout_worker": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_uint32, _P]),
    "rt_rollout_worker_stats": (ctypes.c_int, [_P, ctypes.POINTER(rt_rollout_stats_t)]),
    "rt_host_pump": (ctypes.c_int64, [_P, _P, ctypes.c_uint32, _P, _P, ctypes.c_uint32,
                                      ctypes.c_int, ctypes.c_uint32]),
    "rt_host_pump_paced": (ctypes.c_int64, [_P, _P, _P, ctypes.c_uint32, _P, _P, _P,
                                            ctypes.c_uint32, ctypes.c_int, ctypes.c_uint32]),
    "rt_launch_decode_worker": (ctypes.c_int, [_P, ctypes.POINTER(KVArena), _P, _P, _P, _P,
                                               ctypes.c_uint32, _P, ctypes.c_uint32,
                                               ctypes.c_uint32, _P]),
    "rt_decode_worker_stats": (ctypes.c_int, [_P, ctypes.POINTER(rt_decode_worker_stats_t)]),
    "rt_attention_fixed128": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.POINTER(KVArena), _P,
                                             _P, _P, ctypes.c_uint32, _P, _P]),
    "rt_host_decode_pump": (ctypes.c_int64, [_P, _P, ctypes.c_uint32, ctypes.c_uint32, _P, _P,
                                             ctypes.c_uint32, ctypes.c_uint32]),
    "rt_rollout_set_model": (ctypes.c_int, [_P, ctypes.POINTER(rt_model_weights_t)]),
    "rt_trace_bytes": (ctypes.c_size_t, [ctypes.c_uint32]),
    "rt_trace_init": (ctypes.c_int, [_P, ctypes.c_uint32, _P]),
    "rt_rollout_set_trace": (ctypes.c_int, [_P, _P]),
    "rt_trace_read": (ctypes.c_int, [_P, _P, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint64), _P]),
    "rt_rollout_prefill": (ctypes.c_int, [_P, ctypes.c_uint32, _P, ctypes.c_uint32, _P]),
    "rt_gemm_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(rt_gemm_params_t)]),
    "rt_gemm_bf16": (ctypes.c_int, [ctypes.POINTER(rt_gemm_params_t), _P, _P, _P, _P,
                                    ctypes.c_size_t, _P, _P]),
    "rt_gemm_bf16_chunk_max": (ctypes.c_int, [ctypes.POINTER(rt_gemm_params_t), _P, _P, _P, _P,
                                              ctypes.c_size_t, _P, _P, ctypes.c_uint32, _P]),
    "ring_create": (_P, []), "ring_destroy": (None, [_P]),
    "comp_ring_create": (_P, []), "comp_ring_destroy": (None, [_P]),
    "req_ring_create": (_P, []), "req_ring_destroy": (None, [_P]),
    "done_ring_create": (_P, []), "done_ring_destroy": (None, [_P]),
    "arena_init": (None, [ctypes.POINTER(KVArena), ctypes.c_size_t, ctypes.c_size_t]),
    "arena_acquire": (ctypes.c_int64, [ctypes.POINTER(KVArena)]),
    "arena_release": (None, [ctypes.POINTER(KVArena), ctypes.c_int64]),
    "arena_destroy": (None, [ctypes.POINTER(KVArena)]),
    "rt_fill_normal_bf16": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32,
                                           ctypes.c_float, ctypes.c_float, _P]),
    "rt_fill_normal_f32": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32,
                                          ctypes.c_float, ctypes.c_float, _P]),
}


def lib() -> ctypes.CDLL:
    """Load librlrt_b200.so (raises OSError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run `make -C {HERE}` (or __graft_entry__.build())")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


class RuntimeErrorRT(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != RT_OK:
        msg = lib().rt_last_error().decode(errors="replace")
        raise RuntimeErrorRT(f"{what} failed ({rc}): {msg}")


def _stream_ptr(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


# --------------------------------------------------------------- attention
class PagedDecodeAttention:
    """Paged GQA decode attention (rlrt.h rt_paged_decode_attention).

    Owns the split-K workspace (device scratch, zeroed once here).
    q: bf16 [B, Hq, 128]; arena: bf16 pages (kv_layout.h); page_table,
    seq_lens: int32; returns fp32 [B, Hq, 128].
    """

    def __init__(self, num_seqs, num_q_heads, num_kv_heads, max_pages_per_seq, max_seq_len,
                 arena_pages, scale=None, chunk_pages=0, evict_first=False, device="cuda"):
        import torch
        self.params = rt_attn_params_t(
            num_seqs, num_q_heads, num_kv_heads, 128, max_pages_per_seq, max_seq_len,
            arena_pages, scale if scale is not None else 128 ** -0.5, chunk_pages,
            1 if evict_first else 0)
        n = lib().rt_attn_workspace_bytes(ctypes.byref(self.params))
        if n == 0:
            raise RuntimeErrorRT("bad attention params: " + lib().rt_last_error().decode())
        self.workspace = torch.zeros(n, dtype=torch.uint8, device=device)
        self.device = device

    def plan(self):
        cp, mc, ctas = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint64()
        check(lib().rt_attn_plan(ctypes.byref(self.params), ctypes.byref(cp), ctypes.byref(mc),
                                 ctypes.byref(ctas)), "rt_attn_plan")
        return cp.value, mc.value, ctas.value

    def __call__(self, q, arena, page_table, seq_lens, out=None, stream=None):
        import torch
        if out is None:
            out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        check(lib().rt_paged_decode_attention(
            ctypes.byref(self.params), _ptr(q), _ptr(arena), _ptr(page_table), _ptr(seq_lens),
            _ptr(out), _ptr(self.workspace), self.workspace.numel(), _stream_ptr(stream)),
            "rt_paged_decode_attention")
        return out

    def error_code(self, stream=None) -> int:
        code = ctypes.c_int32()
        check(lib().rt_attn_workspace_error(_ptr(self.workspace), _stream_ptr(stream),
                                            ctypes.byref(code)), "rt_attn_workspace_error")
        return code.value


GROUP_RECORD_WORDS = 18  # rt_attn_group_t as uint32 words


def group_table(groups, max_groups=None):
    """Pack [(shared_pages, [members...]), ...] into an int32 array of
    rt_attn_group_t records (n_members, shared_pages, members[16])."""
    import numpy as np
    n = max_groups or max(1, len(groups))
    t = np.zeros((n, GROUP_RECORD_WORDS), dtype=np.uint32)
    for i, (shared, members) in enumerate(groups):
        t[i, 0] = len(members)
        t[i, 1] = shared
        t[i, 2:2 + len(members)] = members
    return t


class GroupedDecodeAttention(PagedDecodeAttention):
    """Shared-prefix decode attention (rlrt.h rt_paged_decode_attention_grouped).

    groups: device uint32 [max_groups, 18] (group_table), n_groups: device
    uint32 [1], skip_pages: device uint32 [B]."""

    def __init__(self, num_seqs, num_q_heads, num_kv_heads, max_pages_per_seq, max_seq_len,
                 arena_pages, max_groups, max_shared_pages, group_chunk_pages=0, scale=None,
                 chunk_pages=0, evict_first=False, device="cuda"):
        import torch
        self.params = rt_attn_params_t(
            num_seqs, num_q_heads, num_kv_heads, 128, max_pages_per_seq, max_seq_len,
            arena_pages, scale if scale is not None else 128 ** -0.5, chunk_pages,
            1 if evict_first else 0)
        self.gparams = rt_attn_group_params_t(max_groups, max_shared_pages, group_chunk_pages, 0)
        n = lib().rt_attn_grouped_workspace_bytes(ctypes.byref(self.params),
                                                  ctypes.byref(self.gparams))
        if n == 0:
            raise RuntimeErrorRT("bad attention params: " + lib().rt_last_error().decode())
        self.workspace = torch.zeros(n, dtype=torch.uint8, device=device)
        self.device = device

    def __call__(self, q, arena, page_table, seq_lens, groups, n_groups, skip_pages, out=None,
                 stream=None):
        import torch
        if out is None:
            out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        check(lib().rt_paged_decode_attention_grouped(
            ctypes.byref(self.params), ctypes.byref(self.gparams), _ptr(q), _ptr(arena),
            _ptr(page_table), _ptr(seq_lens), _ptr(groups), _ptr(n_groups), _ptr(skip_pages),
            _ptr(out), _ptr(self.workspace), self.workspace.numel(), _stream_ptr(stream)),
            "rt_paged_decode_attention_grouped")
        return out


def fill_normal_bf16(t, seed, stream_id=0, mean=0.0, std=1.0, stream=None):
    check(lib().rt_fill_normal_bf16(_ptr(t), t.numel(), seed, stream_id, mean, std,
                                    _stream_ptr(stream)), "rt_fill_normal_bf16")
    return t


def fill_normal_f32(t, seed, stream_id=0, mean=0.0, std=1.0, stream=None):
    check(lib().rt_fill_normal_f32(_ptr(t), t.numel(), seed, stream_id, mean, std,
                                   _stream_ptr(stream)), "rt_fill_normal_f32")
    return t


# ----------------------------------------------------------------- sampler
SAMPLE_ROW_BYTES = 32


def sample_row_table(temperature, top_k, top_p, rollout_id, step, seed):
    """Pack per-row sampling parameters (rt_sample_row_t) into a numpy record
    array; scalars broadcast."""
    import numpy as np
    dt = np.dtype([("temperature", "<f4"), ("top_k", "<u4"), ("top_p", "<f4"),
                   ("rollout_id", "<u4"), ("step", "<u8"), ("seed", "<u8")])
    assert dt.itemsize == SAMPLE_ROW_BYTES
    n = max(np.size(x) for x in (temperature, top_k, top_p, rollout_id, step, seed))
    t = np.zeros(n, dtype=dt)
    t["temperature"], t["top_k"], t["top_p"] = temperature, top_k, top_p
    t["rollout_id"], t["step"], t["seed"] = rollout_id, step, seed
    return t


def sample_rows(logits, rows, vocab, fused_cum=True, out=None, row_enable=None, stream=None):
    """rt_sample_rows: logits fp32 [R, stride] (device), rows = device uint8
    tensor holding R rt_sample_row_t records; returns int32 tokens [R]."""
    import torch
    R = logits.shape[0]
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=logits.device)
    p = rt_sample_params_t(R, vocab, logits.stride(0), 1 if fused_cum else 0,
                           None if row_enable is None else row_enable.data_ptr())
    check(lib().rt_sample_rows(ctypes.byref(p), _ptr(logits), _ptr(rows), _ptr(out),
                               _stream_ptr(stream)), "rt_sample_rows")
    return out


def chunk_max_stride(vocab) -> int:
    """Floats per row of a chunk-maximum array (rt_chunk_max_stride)."""
    return int(lib().rt_chunk_max_stride(vocab))


def logits_chunk_max(logits, vocab, out=None, stream=None):
    """rt_logits_chunk_max: each 16-column chunk's maximum (NaN if the chunk
    holds a NaN) of fp32 logits [R, stride] (device); returns fp32
    [R, chunk_max_stride(vocab)]."""
    import torch
    R = logits.shape[0]
    cs = chunk_max_stride(vocab)
    if out is None:
        out = torch.empty(R, cs, dtype=torch.float32, device=logits.device)
    check(lib().rt_logits_chunk_max(_ptr(logits), R, vocab, logits.stride(0), _ptr(out),
                                    out.stride(0), _stream_ptr(stream)), "rt_logits_chunk_max")
    return out


def sample_rows_cmax(logits, chunk_max, rows, vocab, fused_cum=True, out=None, row_enable=None,
                     stream=None):
    """rt_sample_rows_cmax: rt_sample_rows given the logits' chunk maxima
    (fp32 [R, chunk_max_stride(vocab)], device); returns int32 tokens [R]."""
    import torch
    R = logits.shape[0]
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=logits.device)
    p = rt_sample_params_t(R, vocab, logits.stride(0), 1 if fused_cum else 0,
                           None if row_enable is None else row_enable.data_ptr())
    check(lib().rt_sample_rows_cmax(ctypes.byref(p), _ptr(logits), _ptr(chunk_max),
                                    chunk_max.stride(0), _ptr(rows), _ptr(out),
                                    _stream_ptr(stream)), "rt_sample_rows_cmax")
    return out


def sample_uniform24(seed, rollout_id, step) -> int:
    return int(lib().rt_sample_uniform24(seed, rollout_id, step))


# ------------------------------------------------------------ rollout loop
RT_ROLLOUT_DECODE_NONE, RT_ROLLOUT_DECODE_FULL, RT_ROLLOUT_DECODE_MODEL = 0, 1, 2
RT_REWARD_MOCK, RT_REWARD_PHILOX = 0, 1
RT_PREFIX_ATTN_GROUPED = 0
RT_PREFIX_ATTN_PER_SEQUENCE = 1
PAGE_TOKENS = 16


def page_bytes(num_kv_heads: int) -> int:
    return num_kv_heads * 2 * 16 * 128 * 2


class DeviceArena:
    """A KVArena (arena.h) whose blocks live in a torch-allocated HBM buffer.
    arena_acquire / arena_release from the C library manage the bitmap."""

    def __init__(self, n_pages, num_kv_heads=8, device="cuda"):
        import torch
        self.block = page_bytes(num_kv_heads)
        self.n_pages = n_pages
        self.buf = torch.zeros(n_pages * self.block, dtype=torch.uint8, device=device)
        self.c = KVArena()
        self.c.base = self.buf.data_ptr()
        self.c.capacity = n_pages * self.block
        self.c.block_size = self.block

    def acquire(self, n):
        out = []
        for _ in range(n):
            b = lib().arena_acquire(ctypes.byref(self.c))
            if b < 0:
                raise RuntimeErrorRT("arena exhausted")
            out.append(b)
        return out

    def bf16(self):
        import torch
        return self.buf.view(torch.bfloat16)

    def fill_pages(self, pages, seed, stream_id=0):
        """Fill whole pages with N(0,1) bf16 (synthetic prefill; contiguous runs)."""
        import numpy as np
        pages = np.sort(np.asarray(pages, dtype=np.int64))
        if len(pages) == 0:
            return
        starts = np.concatenate([[0], np.nonzero(np.diff(pages) != 1)[0] + 1])
        ends = np.concatenate([starts[1:], [len(pages)]])
        v = self.bf16()
        per = self.block // 2
        for a, b in zip(starts, ends):
            lo = int(pages[a]) * per
            hi = (int(pages[b - 1]) + 1) * per
            fill_normal_bf16(v[lo:hi], seed=seed, stream_id=stream_id + int(pages[a]))


class RolloutEngine:
    """rt_rollout_* (GPU-resident rollout loop).  cfg: dict of
    rt_rollout_config_t fields (missing ones default to 0)."""

    def __init__(self, cfg: dict, arena: DeviceArena | None = None):
        self.cfg = rt_rollout_config_t(**cfg)
        self.arena = arena
        h = ctypes.c_void_p()
        check(lib().rt_rollout_create(ctypes.byref(self.cfg),
                                      ctypes.byref(arena.c) if arena else None,
                                      ctypes.byref(h)), "rt_rollout_create")
        self.h = h

    def set_prefix(self, prefix_id, pages, token_len):
        import numpy as np
        arr = np.ascontiguousarray(pages, dtype=np.int32)
        check(lib().rt_rollout_set_prefix(self.h, prefix_id, arr.ctypes.data_as(ctypes.c_void_p),
                                          len(arr), token_len), "rt_rollout_set_prefix")

    @staticmethod
    def _io(ring, requests, n_requests, done_ring, dones, state, step_count, trajectories,
            rewards, n_rows, arrivals=None, arrival_unit=RT_ARRIVAL_PASS):
        ptr = lambda t: None if t is None else (t if isinstance(t, int) else t.data_ptr())
        return rt_rollout_io_t(ptr(ring), ptr(requests), n_requests, ptr(done_ring), ptr(dones),
                               ptr(state), ptr(step_count), ptr(trajectories), ptr(rewards),
                               n_rows, arrival_unit, ptr(arrivals))

    def launch(self, *, requests=None, n_requests=0, ring=None, done_ring=None, dones=None,
               state=None, step_count=None, trajectories=None, rewards=None, n_rows=0,
               arrivals=None, arrival_unit=RT_ARRIVAL_PASS, stream=None):
        """rt_rollout_launch.  arrivals: optional uint64 device tensor, one
        arrival per request of an array source, in passes (RT_ARRIVAL_PASS)
        or ns since the first pass (RT_ARRIVAL_NS)."""
        io = self._io(ring, requests, n_requests, done_ring, dones, state, step_count,
                      trajectories, rewards, n_rows, arrivals, arrival_unit)
        check(lib().rt_rollout_launch(self.h, ctypes.byref(io), _stream_ptr(stream)),
              "rt_rollout_launch")

    def profile(self, *, requests=None, n_requests=0, dones=None, state=None, trajectories=None,
                rewards=None, n_rows=0, arrivals=None, arrival_unit=RT_ARRIVAL_PASS,
                stream=None):
        """rt_rollout_profile: host-stepped replay with per-kernel CUDA events."""
        io = self._io(None, requests, n_requests, None, dones, state, None, trajectories,
                      rewards, n_rows, arrivals, arrival_unit)
        out = rt_rollout_profile_t()
        check(lib().rt_rollout_profile(self.h, ctypes.byref(io), _stream_ptr(stream),
                                       ctypes.byref(out)), "rt_rollout_profile")
        return out.as_dict()

    def step(self, hook, *, requests=None, n_requests=0, dones=None, state=None,
             trajectories=None, rewards=None, n_rows=0, arrivals=None,
             arrival_unit=RT_ARRIVAL_PASS, stream=None):
        """rt_rollout_profile_hook: host-stepped replay calling hook(pass) after
        every pass; a truthy return stops it."""
        io = self._io(None, requests, n_requests, None, dones, state, None, trajectories,
                      rewards, n_rows, arrivals, arrival_unit)
        out = rt_rollout_profile_t()
        err = []

        def tramp(_user, p):
            try:
                return 1 if hook(int(p)) else 0
            except BaseException as exc:  # surface after the C call returns
                err.append(exc)
                return 1

        cb = PASS_HOOK(tramp)
        rc = lib().rt_rollout_profile_hook(self.h, ctypes.byref(io), _stream_ptr(stream),
                                           ctypes.byref(out), ctypes.cast(cb, ctypes.c_void_p),
                                           None)
        if err:
            raise err[0]
        check(rc, "rt_rollout_profile_hook")
        return out.as_dict()

    def set_model(self, embed, w_qkv, w_lm):
        """rt_rollout_set_model: bf16 device tensors embed [vocab][d],
        w_qkv [(hq + 2 hkv) * 128][d], w_lm [vocab][d] (kept referenced)."""
        self._weights = (embed, w_qkv, w_lm)
        w = rt_model_weights_t(embed.data_ptr(), w_qkv.data_ptr(), w_lm.data_ptr(),
                               embed.shape[1], 0)
        check(lib().rt_rollout_set_model(self.h, ctypes.byref(w)), "rt_rollout_set_model")

    def prefill(self, prefix_id, tokens, stream=None):
        """rt_rollout_prefill: K / V of the prefix's prompt tokens (device
        uint32 / int32 tensor) from the model weights."""
        check(lib().rt_rollout_prefill(self.h, prefix_id, ctypes.c_void_p(tokens.data_ptr()),
                                       tokens.numel(), _stream_ptr(stream)), "rt_rollout_prefill")

    def set_trace(self, trace):
        """rt_rollout_set_trace: a DeviceTrace, or None to detach."""
        self._trace = trace
        check(lib().rt_rollout_set_trace(self.h, None if trace is None else
                                         ctypes.c_void_p(trace.buf.data_ptr())),
              "rt_rollout_set_trace")

    def buffers(self):
        b = rt_rollout_buffers_t()
        check(lib().rt_rollout_buffers(self.h, ctypes.byref(b)), "rt_rollout_buffers")
        return b

    def wait(self, stream=None, check_errors=True):
        st = rt_rollout_stats_t()
        rc = lib().rt_rollout_wait(self.h, _stream_ptr(stream), ctypes.byref(st))
        if check_errors:
            check(rc, "rt_rollout_wait")
        return st.as_dict()

    def close(self):
        if self.h:
            lib().rt_rollout_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


TRACE_ROLLOUT_ALLOC, TRACE_ROLLOUT_FREE, TRACE_DESC_CONSUMED = 0, 1, 4
TRACE_DECODE_BATCH, TRACE_REWARD_POSTED, TRACE_TRAJECTORY_DONE = 7, 8, 10


class DeviceTrace:
    """A device trace ring (rt_trace_*) of `capacity` records (power of two)."""

    def __init__(self, capacity, device="cuda"):
        import torch
        n = lib().rt_trace_bytes(capacity)
        if n == 0:
            raise RuntimeErrorRT(lib().rt_last_error().decode())
        self.capacity = capacity
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)
        check(lib().rt_trace_init(ctypes.c_void_p(self.buf.data_ptr()), capacity,
                                  _stream_ptr(None)), "rt_trace_init")

    def read(self, max_records=None):
        """(records as a numpy structured array in append order, appended)."""
        import numpy as np
        dt = np.dtype([("tsc", "<u8"), ("type", "<u4"), ("rollout_id", "<u4"), ("seq", "<u4")])
        n = self.capacity if max_records is None else max_records
        out = np.zeros(n, dtype=dt)
        total = ctypes.c_uint64()
        check(lib().rt_trace_read(ctypes.c_void_p(self.buf.data_ptr()),
                                  out.ctypes.data_as(ctypes.c_void_p), n, ctypes.byref(total),
                                  _stream_ptr(None)), "rt_trace_read")
        return out[:min(n, total.value, self.capacity)], total.value


def replay_trajectories(requests, traj, rows, vocab, logit_std=2.0, chunk=2048, device="cuda"):
    """Re-derive the tokens a synthetic-logits loop (RT_ROLLOUT_DECODE_FULL)
    must have produced for the trajectory rows `rows` (consume indices into
    the request array) and compare them with `traj` (a host int array
    [n_rows][max_new]): the loop's logits for (request rng_seed, request low
    32 bits, token index) are regenerated with rt_logits_synth and sampled by
    rt_sample_rows with the request's parameters.  Returns (tokens checked,
    list of (row, token index, expected, got) mismatches)."""
    import numpy as np
    import torch
    meta = [(int(i), t) for i in rows for t in range(int(requests["max_tokens"][i]))]
    bad = []
    for c0 in range(0, len(meta), chunk):
        part = meta[c0:c0 + chunk]
        logits = torch.empty(len(part), vocab, dtype=torch.float32, device=device)
        rq = [int(requests["request_id"][i]) & 0xFFFFFFFF for i, _ in part]
        seed = [int(requests["rng_seed"][i]) for i, _ in part]
        for k, (_, t) in enumerate(part):
            logits_synth(logits[k], vocab, seed[k], rq[k], t, logit_std)
        tab = sample_row_table(np.array([float(requests["temperature"][i]) for i, _ in part]),
                               np.array([int(requests["top_k"][i]) for i, _ in part]),
                               np.array([float(requests["top_p"][i]) for i, _ in part]),
                               np.array(rq, dtype=np.uint32), np.array([t for _, t in part]),
                               np.array(seed, dtype=np.uint64))
        tok = sample_rows(logits, torch.from_numpy(tab.view(np.uint8)).to(device), vocab)
        tok = tok.cpu().numpy()
        for k, (i, t) in enumerate(part):
            if int(tok[k]) != int(traj[i, t]):
                bad.append((i, t, int(tok[k]), int(traj[i, t])))
    return len(meta), bad


def logits_synth(out, vocab, seed, request_lo, token_index, logit_std, stream=None):
    check(lib().rt_logits_synth(_ptr(out), vocab, seed, request_lo, token_index, logit_std,
                                _stream_ptr(stream)), "rt_logits_synth")
    return out


class HostRings:
    """A RequestRing and a DoneRing in pinned, device-mapped host memory."""

    def __init__(self):
        self.req = lib().req_ring_create()
        self.done = lib().done_ring_create()
        if not self.req or not self.done:
            raise RuntimeErrorRT("ring allocation failed")

    def pump(self, requests, n_expected, send_sentinel=True, timeout_ms=60000):
        """rt_host_pump: requests holds 34-byte RolloutRequest records (a
        structured array, or raw bytes); returns (n drained, RolloutDone bytes)."""
        import numpy as np
        reqs = np.ascontiguousarray(requests)
        if reqs.nbytes % 34:
            raise ValueError("requests must be whole 34-byte RolloutRequest records")
        n_req = reqs.nbytes // 34
        out = np.zeros(max(n_expected, 1) * 24, dtype=np.uint8)
        n = lib().rt_host_pump(self.req, reqs.ctypes.data_as(ctypes.c_void_p), n_req,
                               self.done, out.ctypes.data_as(ctypes.c_void_p), n_expected,
                               1 if send_sentinel else 0, timeout_ms)
        return n, out

    def pump_paced(self, requests, arrival_ns, n_expected, send_sentinel=True,
                   timeout_ms=60000):
        """rt_host_pump_paced: push request i no earlier than arrival_ns[i]
        after the call starts; returns (n drained, RolloutDone bytes, drain
        time of each record in ns on the same clock)."""
        import numpy as np
        reqs = np.ascontiguousarray(requests)
        if reqs.nbytes % 34:
            raise ValueError("requests must be whole 34-byte RolloutRequest records")
        n_req = reqs.nbytes // 34
        arr = np.ascontiguousarray(arrival_ns, dtype=np.uint64)
        if arr.size != n_req:
            raise ValueError("one arrival per request")
        out = np.zeros(max(n_expected, 1) * 24, dtype=np.uint8)
        t = np.zeros(max(n_expected, 1), dtype=np.uint64)
        n = lib().rt_host_pump_paced(self.req, reqs.ctypes.data_as(ctypes.c_void_p),
                                     arr.ctypes.data_as(ctypes.c_void_p), n_req, self.done,
                                     out.ctypes.data_as(ctypes.c_void_p),
                                     t.ctypes.data_as(ctypes.c_void_p), n_expected,
                                     1 if send_sentinel else 0, timeout_ms)
        return n, out, t

    def close(self):
        if self.req:
            lib().req_ring_destroy(self.req)
            lib().done_ring_destroy(self.done)
            self.req = self.done = None


class CommandRings:
    """A CommandRing and a CompletionRing in pinned, device-mapped host
    memory (the per-step decode path's rings)."""

    def __init__(self):
        self.cmd = lib().ring_create()
        self.comp = lib().comp_ring_create()
        if not self.cmd or not self.comp:
            raise RuntimeErrorRT("ring allocation failed")

    def header(self, which):
        """(head, tail) of 'cmd' or 'comp' (plus the comp overflow counter)."""
        base = self.cmd if which == "cmd" else self.comp
        head = ctypes.c_uint32.from_address(base).value
        tail = ctypes.c_uint32.from_address(base + 64).value
        if which == "cmd":
            return head, tail
        return head, tail, ctypes.c_uint32.from_address(base + 128).value

    def pump(self, descs, n_sentinels, n_expected, timeout_ms=60000):
        """rt_host_decode_pump: descs holds 32-byte Descriptor records;
        returns (n drained, Completion bytes)."""
        import numpy as np
        d = np.ascontiguousarray(descs)
        if d.nbytes % 32:
            raise ValueError("descs must be whole 32-byte Descriptor records")
        out = np.zeros(max(n_expected, 1) * 32, dtype=np.uint8)
        n = lib().rt_host_decode_pump(self.cmd, d.ctypes.data_as(ctypes.c_void_p), d.nbytes // 32,
                                      n_sentinels, self.comp,
                                      out.ctypes.data_as(ctypes.c_void_p), n_expected, timeout_ms)
        return n, out

    def close(self):
        if self.cmd:
            lib().ring_destroy(self.cmd)
            lib().comp_ring_destroy(self.comp)
            self.cmd = self.comp = None


def device_arena(arena_u8, block_size):
    """A KVArena describing an existing device buffer (torch uint8) of
    whole blocks; the bitmap stays empty (no allocation through it)."""
    a = KVArena()
    a.base = arena_u8.data_ptr()
    a.capacity = arena_u8.numel()
    a.block_size = block_size
    return a


def launch_decode_worker(rings, arena, sample_st=None, q_buffer=None, o_buffer=None,
                         io_slots=0, step_count=None, stop_sentinels=1, idle_timeout_ms=0,
                         stream=None):
    check(lib().rt_launch_decode_worker(rings.cmd, ctypes.byref(arena), rings.comp,
                                        _ptr(sample_st), _ptr(q_buffer), _ptr(o_buffer),
                                        io_slots, _ptr(step_count), stop_sentinels,
                                        idle_timeout_ms, _stream_ptr(stream)),
          "rt_launch_decode_worker")


def decode_worker_stats(stream=None):
    st = rt_decode_worker_stats_t()
    check(lib().rt_decode_worker_stats(_stream_ptr(stream), ctypes.byref(st)),
          "rt_decode_worker_stats")
    return st.as_dict()


def attention_fixed128(descs, arena, sample_st=None, q_buffer=None, o_buffer=None, io_slots=0,
                       stream=None):
    """rt_attention_fixed128 over a numpy array of 32-byte Descriptor
    records; returns the DecodeStepResult records as numpy
    (path_kind, token_id, bytes_touched, tile_count, cycle_estimate)."""
    import numpy as np
    import torch
    d = np.ascontiguousarray(descs)
    n = d.nbytes // 32
    dev = torch.device("cuda", torch.cuda.current_device())
    dd = torch.from_numpy(d.view(np.uint8).copy()).to(dev)
    res = torch.zeros(max(n, 1) * 24, dtype=torch.uint8, device=dev)
    check(lib().rt_attention_fixed128(_ptr(dd) if n else None, n, ctypes.byref(arena),
                                      _ptr(sample_st), _ptr(q_buffer), _ptr(o_buffer), io_slots,
                                      _ptr(res), _stream_ptr(stream)), "rt_attention_fixed128")
    torch.cuda.synchronize()
    dt = np.dtype([("path_kind", "<u4"), ("token_id", "<u4"), ("bytes_touched", "<u4"),
                   ("tile_count", "<u4"), ("cycle_estimate", "<u8")])
    return res.cpu().numpy().view(dt)[:n]


# ----------------------------------------------------------- rewards / NCCL
def grpo_advantages(rewards, group, eps=1e-6, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty_like(rewards)
    check(lib().rt_grpo_advantages(_ptr(rewards), rewards.numel(), group, eps, _ptr(out),
                                   _stream_ptr(stream)), "rt_grpo_advantages")
    return out


class NcclRewards:
    """rt_nccl_* communicator for the reward allgather.  `exchange_id(id_bytes)`
    distributes rank 0's 128-byte unique id (e.g. through torch.distributed)."""

    def __init__(self, rank, world, exchange_id):
        buf = ctypes.create_string_buffer(128)
        if rank == 0:
            check(lib().rt_nccl_unique_id(buf), "rt_nccl_unique_id")
        uid = exchange_id(bytes(buf.raw))
        buf = ctypes.create_string_buffer(uid, 128)
        comm = ctypes.c_void_p()
        check(lib().rt_nccl_init(ctypes.byref(comm), world, buf, rank), "rt_nccl_init")
        self.comm = comm
        self.world = world

    def allgather(self, send, recv, stream=None):
        check(lib().rt_reward_allgather(self.comm, _ptr(send), _ptr(recv), send.numel(),
                                        _stream_ptr(stream)), "rt_reward_allgather")
        return recv

    def wait(self, stream=None, timeout_ms=60000):
        check(lib().rt_nccl_wait(self.comm, _stream_ptr(stream), timeout_ms), "rt_nccl_wait")

    def close(self):
        if self.comm:
            lib().rt_nccl_destroy(self.comm)
            self.comm = None


# ------------------------------------------------------- GRPO host helpers
REQUEST_RECORD = [("request_id", "<u8"), ("max_tokens", "<u4"), ("kv_blocks", "<u4"),
                  ("temperature", "<f4"), ("top_k", "<u2"), ("top_p", "<f4"), ("rng_seed", "<u8")]


def shard_groups(total_groups, world, rank):
    """Contiguous split of GRPO groups over ranks: (first group, count).
    A group never straddles two GPUs, so its shared prefix lives on one."""
    base, rem = divmod(total_groups, world)
    g0 = rank * base + min(rank, rem)
    return g0, base + (1 if rank < rem else 0)


def grpo_requests(g0, ng, group_size, max_tokens, prompt_pages, temperature=0.8, top_k=50,
                  top_p=0.9, seed=1234):
    """RolloutRequest records for local groups g0 .. g0+ng-1: request ids
    1 + global rollout index (low 32 bits), shared prefix = local group
    (request_id bits 32..63 = local group + 1)."""
    import numpy as np
    n = ng * group_size
    r = np.zeros(n, dtype=np.dtype(REQUEST_RECORD))
    local_group = np.arange(n) // group_size
    r["request_id"] = (np.arange(n, dtype=np.uint64) + np.uint64(g0 * group_size + 1)) | \
        ((local_group.astype(np.uint64) + np.uint64(1)) << np.uint64(32))
    r["max_tokens"] = max_tokens
    r["kv_blocks"] = prompt_pages
    r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = temperature, top_k, top_p, seed
    return r
