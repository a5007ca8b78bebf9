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
                ("chunk_pages", ctypes.c_uint32)]


class rt_sample_row_t(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32),
                ("top_p", ctypes.c_float), ("rollout_id", ctypes.c_uint32),
                ("step", ctypes.c_uint64)]


class rt_sample_params_t(ctypes.Structure):
    _fields_ = [("num_rows", ctypes.c_uint32), ("vocab", ctypes.c_uint32),
                ("row_stride", ctypes.c_uint64), ("seed", ctypes.c_uint64),
                ("fused_cum", ctypes.c_uint32)]


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
    "rt_attn_workspace_error": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_int32)]),
    "rt_sample_rows": (ctypes.c_int, [ctypes.POINTER(rt_sample_params_t), _P, _P, _P, _P]),
    "rt_sample_uniform24": (ctypes.c_uint32, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64]),
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
    return ctypes.c_void_p(t.data_ptr())


# --------------------------------------------------------------- attention
class PagedDecodeAttention:
    """Paged GQA decode attention (rlrt.h rt_paged_decode_attention).

    Owns the split-K workspace (device scratch, zeroed once here).
    q: bf16 [B, Hq, 128]; arena: bf16 pages (kv_layout.h); page_table,
    seq_lens: int32; returns fp32 [B, Hq, 128].
    """

    def __init__(self, num_seqs, num_q_heads, num_kv_heads, max_pages_per_seq, max_seq_len,
                 arena_pages, scale=None, chunk_pages=0, device="cuda"):
        import torch
        self.params = rt_attn_params_t(
            num_seqs, num_q_heads, num_kv_heads, 128, max_pages_per_seq, max_seq_len,
            arena_pages, scale if scale is not None else 128 ** -0.5, chunk_pages)
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


def fill_normal_bf16(t, seed, stream_id=0, mean=0.0, std=1.0, stream=None):
    check(lib().rt_fill_normal_bf16(_ptr(t), t.numel(), seed, stream_id, mean, std,
                                    _stream_ptr(stream)), "rt_fill_normal_bf16")
    return t


def fill_normal_f32(t, seed, stream_id=0, mean=0.0, std=1.0, stream=None):
    check(lib().rt_fill_normal_f32(_ptr(t), t.numel(), seed, stream_id, mean, std,
                                   _stream_ptr(stream)), "rt_fill_normal_f32")
    return t


# ----------------------------------------------------------------- sampler
SAMPLE_ROW_BYTES = 24


def sample_row_table(temperature, top_k, top_p, rollout_id, step):
    """Pack per-row sampling parameters (rt_sample_row_t) into a numpy record
    array; scalars broadcast."""
    import numpy as np
    dt = np.dtype([("temperature", "<f4"), ("top_k", "<u4"), ("top_p", "<f4"),
                   ("rollout_id", "<u4"), ("step", "<u8")])
    assert dt.itemsize == SAMPLE_ROW_BYTES
    n = max(np.size(x) for x in (temperature, top_k, top_p, rollout_id, step))
    t = np.zeros(n, dtype=dt)
    t["temperature"], t["top_k"], t["top_p"] = temperature, top_k, top_p
    t["rollout_id"], t["step"] = rollout_id, step
    return t


def sample_rows(logits, rows, vocab, seed, fused_cum=True, out=None, stream=None):
    """rt_sample_rows: logits fp32 [R, stride] (device), rows = device uint8
    tensor holding R rt_sample_row_t records; returns int32 tokens [R]."""
    import torch
    R = logits.shape[0]
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=logits.device)
    p = rt_sample_params_t(R, vocab, logits.stride(0), seed, 1 if fused_cum else 0)
    check(lib().rt_sample_rows(ctypes.byref(p), _ptr(logits), _ptr(rows), _ptr(out),
                               _stream_ptr(stream)), "rt_sample_rows")
    return out


def sample_uniform24(seed, rollout_id, step) -> int:
    return int(lib().rt_sample_uniform24(seed, rollout_id, step))
