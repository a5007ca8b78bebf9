"""ctypes bindings of the CPU oracle and the caller harness.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product never imports it.

Libraries (built by oracle/Makefile):
  _build/liboracle.so    CPU restatement of the reference hot path (oracle.c)
  _build/libabi_mine.so  harness/abi_caller.c against this repo's C ABI
  _ref/libabi_ref.so     the same harness against the reference's own sources
  _ref/libgbref.so       the reference's C sources, compiled unmodified
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF = os.path.join(HERE, "_ref")

# numpy views of the packed records (layouts pinned in include/*.h)
HW_DESC_DTYPE = np.dtype([
    ("opcode", "<u2"), ("flags", "<u2"), ("rollout_id", "<u4"), ("kv_arena_id", "<u4"),
    ("prefix_id", "<u4"), ("kv_offset", "<u8"), ("delta_offset", "<u8"), ("seq_len", "<u4"),
    ("max_tokens", "<u4"), ("reward_model_id", "<u4"), ("reserved0", "<u4"),
    ("user_data", "<u8"), ("checksum_or_cookie", "<u8")])
assert HW_DESC_DTYPE.itemsize == 64

REQUEST_DTYPE = np.dtype([
    ("request_id", "<u8"), ("max_tokens", "<u4"), ("kv_blocks", "<u4"), ("temperature", "<f4"),
    ("top_k", "<u2"), ("top_p", "<f4"), ("rng_seed", "<u8")])
assert REQUEST_DTYPE.itemsize == 34

DONE_DTYPE = np.dtype([
    ("request_id", "<u8"), ("rollout_id", "<u4"), ("tokens_generated", "<u4"),
    ("reward", "<f4"), ("status", "<u4")])
assert DONE_DTYPE.itemsize == 24

DESCRIPTOR_DTYPE = np.dtype([
    ("seq_id", "<u8"), ("kv_block_offset", "<u4"), ("num_kv_blocks", "<u2"),
    ("attention_flags", "u1"), ("pad", "u1"), ("output_token_offset", "<u4"),
    ("reward_cookie", "<u8"), ("batch_size", "<u2"), ("batch_index", "<u2")])
assert DESCRIPTOR_DTYPE.itemsize == 32

COMPLETION_DTYPE = np.dtype([
    ("seq_id", "<u8"), ("token_id", "<u4"), ("kv_block_offset", "<u4"),
    ("reward_cookie", "<u8"), ("cycles_taken", "<u8")])
assert COMPLETION_DTYPE.itemsize == 32

GPU_STATE_BYTES = 72 * 256 + 32

_P = ctypes.c_void_p
_u32, _u64, _i32, _f32, _int = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32, ctypes.c_float, ctypes.c_int


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


_oracle = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        path = os.path.join(BUILD, "liboracle.so")
        if not os.path.exists(path):
            raise OSError(f"{path} missing: run `make -C {HERE}`")
        l = ctypes.CDLL(path)
        sig = {
            "orc_philox4x32_10": (None, [_P, _P, _P]),
            "orc_paged_gqa_attention": (None, [_P, _P, _P, _P, _u32, _u32, _u32, _u32, _u32,
                                               _f32, _P, _int]),
            "orc_fixed128_attention": (None, [_P, _P, _u32, _P, _P]),
            "orc_f32_to_f16_rne": (ctypes.c_uint16, [_f32]),
            "orc_f16_to_f32": (_f32, [ctypes.c_uint16]),
            "orc_worker_sim_stream": (_u32, [_P, _u32, _P, _P]),
            "orc_submit_desc": (None, [_u32, _u32, _u32, _u64, _u64, _u32, _u32, _u32, _P]),
            "orc_sample_row": (_u32, [_P, _u32, _f32, _u32, _f32, _u32, _int, _P]),
            "orc_sample_u24": (_u32, [_u64, _u32, _u64]),
            "orc_scheduler_run": (_u32, [_P, _u32, _P, _u32, _int, _u32, _P, _P, _P, _P, _P, _u32]),
            "orc_grpo_advantages": (None, [_P, _u32, _u32, _f32, _P]),
            "orc_reward_u01": (_f32, [_u64, _u32]),
            "orc_decode_synth_q": (_f32, [_u64, _u64, _P, _u32]),
            "orc_decode_steps": (_u32, [_P, _u32, _P, _u64, _u64, _P, _P, _u32, _P, _P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _oracle = l
    return _oracle


# ----------------------------------------------------------------- oracle
def philox(ctr, key) -> list[int]:
    c = np.array(ctr, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    o = np.zeros(4, dtype=np.uint32)
    oracle_lib().orc_philox4x32_10(_ptr(c), _ptr(k), _ptr(o))
    return [int(x) for x in o]


def paged_gqa_attention(q_bits, arena_bits, page_table, seq_lens, Hq, Hkv, scale, n_threads=0):
    """q_bits uint16 [B,Hq,128]; arena_bits uint16 flat; returns fp32 [B,Hq,128]."""
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    arena_bits = np.ascontiguousarray(arena_bits, dtype=np.uint16)
    page_table = np.ascontiguousarray(page_table, dtype=np.int32)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    B = q_bits.shape[0]
    out = np.zeros((B, Hq, 128), dtype=np.float32)
    oracle_lib().orc_paged_gqa_attention(
        _ptr(q_bits), _ptr(arena_bits), _ptr(page_table), _ptr(seq_lens), B, Hq, Hkv, 128,
        page_table.shape[1], scale, _ptr(out), n_threads or os.cpu_count() or 1)
    return out


def fixed128_attention(q_f16_bits, block_f16_bits, seq_len):
    out = np.zeros(128, dtype=np.float32)
    tok = np.zeros(1, dtype=np.uint32)
    oracle_lib().orc_fixed128_attention(
        _ptr(np.ascontiguousarray(q_f16_bits, dtype=np.uint16)),
        _ptr(np.ascontiguousarray(block_f16_bits, dtype=np.uint16)), seq_len, _ptr(out), _ptr(tok))
    return out, int(tok[0])


def decode_steps(descs, arena_u8, block_size, rng4=None, q_buf=None, io_slots=0):
    """The reference decode step (process_descriptor + fixed128 attention)
    over DESCRIPTOR_DTYPE records; arena_u8 is the arena's bytes.  Returns
    (COMPLETION_DTYPE records, fp32 output rows [n][128], number of
    out-of-range blocks)."""
    descs = np.ascontiguousarray(descs, dtype=DESCRIPTOR_DTYPE)
    arena_u8 = np.ascontiguousarray(arena_u8, dtype=np.uint8)
    n = len(descs)
    comps = np.zeros(n, dtype=COMPLETION_DTYPE)
    o = np.zeros((n, 128), dtype=np.float32)
    rng = None if rng4 is None else np.ascontiguousarray(rng4, dtype=np.uint64)
    q = None if q_buf is None else np.ascontiguousarray(q_buf, dtype=np.uint16)
    bad = oracle_lib().orc_decode_steps(
        _ptr(descs), n, _ptr(arena_u8), block_size, arena_u8.nbytes // block_size,
        None if rng is None else _ptr(rng), None if q is None else _ptr(q), io_slots,
        _ptr(o), _ptr(comps))
    return comps, o, int(bad)


def worker_sim_stream(descs: np.ndarray):
    descs = np.ascontiguousarray(descs, dtype=HW_DESC_DTYPE)
    out = np.zeros(len(descs), dtype=HW_DESC_DTYPE)
    tokens = np.zeros(1, dtype=np.uint64)
    n = oracle_lib().orc_worker_sim_stream(_ptr(descs), len(descs), _ptr(out), _ptr(tokens))
    return out[:n], int(tokens[0])


def sample_row(logits, temperature, top_k, top_p, u24, fma_cum=True) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    scratch = np.empty_like(logits)
    return int(oracle_lib().orc_sample_row(_ptr(logits), logits.size, temperature, top_k, top_p,
                                           u24, int(fma_cum), _ptr(scratch)))


def sample_u24(seed, rollout_id, step) -> int:
    return int(oracle_lib().orc_sample_u24(seed, rollout_id, step))


def scheduler_run(reqs: np.ndarray, arrival_pass=None, max_admit=1, drop_when_full=True,
                  max_passes=1 << 20, with_admit=False, max_slots=256):
    """The reference pass loop (cu/gpu_scheduler.cu:33-82) with max_admit /
    drop switches, an optional per-request arrival pass and a slot count
    below the reference's 256 (lowest free slot below max_slots).  Returns (dones,
    done pass of each, final GpuRolloutState bytes, passes run) and, with
    with_admit, the pass in which each request was admitted (UINT32_MAX if
    never)."""
    reqs = np.ascontiguousarray(reqs, dtype=REQUEST_DTYPE)
    n = len(reqs)
    dones = np.zeros(max(n, 1), dtype=DONE_DTYPE)
    done_pass = np.zeros(max(n, 1), dtype=np.uint32)
    admit = np.zeros(max(n, 1), dtype=np.uint32)
    state = np.zeros(GPU_STATE_BYTES, dtype=np.uint8)
    passes = np.zeros(1, dtype=np.uint32)
    arr = None if arrival_pass is None else np.ascontiguousarray(arrival_pass, dtype=np.uint32)
    nd = oracle_lib().orc_scheduler_run(
        _ptr(reqs), n, None if arr is None else _ptr(arr), max_admit, int(drop_when_full),
        max_passes, _ptr(dones), _ptr(done_pass), _ptr(state), _ptr(passes), _ptr(admit),
        max_slots)
    out = (dones[:nd], done_pass[:nd], state, int(passes[0]))
    return out + (admit[:n],) if with_admit else out


def reward_u01(seed, request_lo) -> float:
    return float(np.float32(oracle_lib().orc_reward_u01(seed, request_lo)))


def grpo_advantages(rewards, group, eps=1e-6):
    r = np.ascontiguousarray(rewards, dtype=np.float32)
    adv = np.zeros_like(r)
    oracle_lib().orc_grpo_advantages(_ptr(r), r.size, group, eps, _ptr(adv))
    return adv


# ---------------------------------------------------------------- harness
class Harness:
    """One build of harness/abi_caller.c (against 'mine' or 'ref' headers)."""

    def __init__(self, which: str):
        path = os.path.join(BUILD if which == "mine" else REF,
                            "libabi_mine.so" if which == "mine" else "libabi_ref.so")
        if not os.path.exists(path):
            raise OSError(f"{path} missing: run `make -C {HERE}`")
        self.which = which
        l = ctypes.CDLL(path)
        sig = {
            "hx_gen_c1": (None, [_u64, _u32, _u32, _P]),
            "hx_run_c1": (_int, [_P, _u32, _u32, _u32, _P, _P, _P, _P, _P]),
            "hx_kat_submit": (_int, [_u32, _u32, _u32, _u64, _u64, _u32, _u32, _u32, _P, _P]),
            "hx_kat_submit_errors": (None, [_P]),
            "hx_kat_hw_ring": (_u32, []),
            "hx_kat_worker": (_int, [_P, _P, _P, _P]),
            "hx_script_command_ring": (_u32, [_P, _P]),
            "hx_script_request_ring": (_u32, [_P, _P, _P]),
            "hx_script_kv_prefix": (_u32, [_P]),
            "hx_script_reward": (_u32, [_P, _P]),
            "hx_script_arena_bitmap": (_u32, [_P, _u32]),
            "hx_run_decode_batch": (_int, [_P, _u32, _u32, _P, _P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = l

    def run_decode_batch(self, descs, window=32):
        """decode_batch_submit windows of `window` into a CommandRing with a
        consumer thread; returns (the consumed records in ring order, seconds)."""
        descs = np.ascontiguousarray(descs, dtype=DESCRIPTOR_DTYPE)
        out = np.zeros(len(descs), dtype=DESCRIPTOR_DTYPE)
        secs = np.zeros(1, dtype=np.float64)
        rc = self.lib.hx_run_decode_batch(_ptr(descs), len(descs), window, _ptr(out), _ptr(secs))
        if rc != 0:
            raise RuntimeError(f"hx_run_decode_batch failed ({rc})")
        return out, float(secs[0])

    def gen_c1(self, n=10000, seed=0, max_tokens=2048):
        out = np.zeros(n, dtype=HW_DESC_DTYPE)
        self.lib.hx_gen_c1(seed, n, max_tokens, _ptr(out))
        return out

    def run_c1(self, descs, depth_cap=1024, doorbell_batch=1):
        descs = np.ascontiguousarray(descs, dtype=HW_DESC_DTYPE)
        out = np.zeros(len(descs), dtype=HW_DESC_DTYPE)
        n_out = np.zeros(1, np.uint32)
        tok = np.zeros(1, np.uint64)
        comp = np.zeros(1, np.uint64)
        secs = np.zeros(1, np.float64)
        rc = self.lib.hx_run_c1(_ptr(descs), len(descs), depth_cap, doorbell_batch, _ptr(out),
                                _ptr(n_out), _ptr(tok), _ptr(comp), _ptr(secs))
        assert rc == 0
        return out[:int(n_out[0])], int(tok[0]), int(comp[0]), float(secs[0])

    def kat_submit(self, *args):
        bell = np.zeros(1, np.uint32)
        d = np.zeros(1, HW_DESC_DTYPE)
        rc = self.lib.hx_kat_submit(*args, _ptr(bell), _ptr(d))
        return rc, int(bell[0]), d[0]

    def kat_submit_errors(self):
        rc = np.zeros(4, np.int32)
        self.lib.hx_kat_submit_errors(_ptr(rc))
        return rc.tolist()

    def kat_worker(self, desc):
        inp = np.array([desc], dtype=HW_DESC_DTYPE)
        out = np.zeros(1, HW_DESC_DTYPE)
        tok = np.zeros(1, np.uint64)
        comp = np.zeros(1, np.uint64)
        rc = self.lib.hx_kat_worker(_ptr(inp), _ptr(out), _ptr(tok), _ptr(comp))
        return rc, out[0], int(tok[0]), int(comp[0])

    def script(self, name, *extra):
        log = np.zeros(256, np.int64)
        fn = getattr(self.lib, name)
        n = fn(_ptr(log), *[_ptr(e) if isinstance(e, np.ndarray) else e for e in extra])
        return log[:n]


# ------------------------------------------------------- reference on GPU
_M64 = 1 << 64
_INV5 = pow(5, -1, _M64)
_INV9 = pow(9, -1, _M64)


def xoshiro_s1_for_first_output(value: int) -> int:
    """State word s1 that makes the reference's first xoshiro256** draw
    (rotl(s1 * 5, 7) * 9, reference cu/sample.cu:13-14) equal `value`."""
    x = (value * _INV9) % _M64
    x = ((x >> 7) | (x << 57)) % _M64          # rotr 7
    return (x * _INV5) % _M64


class RefCuda:
    """The reference's own cu/sample.cu compiled for sm_100a into
    oracle/_ref/libref_cuda.so, driven by harness/ref_sample.cu."""

    def __init__(self):
        path = os.path.join(REF, "libref_cuda.so")
        if not os.path.exists(path):
            raise OSError(f"{path} missing: build oracle/_ref where the reference tree exists")
        l = ctypes.CDLL(path)
        l.hx_ref_sample_rows.restype = _int
        l.hx_ref_sample_rows.argtypes = [_P, _u32, _u64, _P, _P, _P, _P, _P, _u32]
        l.hx_ref_fixed128.restype = _int
        l.hx_ref_fixed128.argtypes = [_P, _u32, _P, _u64, _P, _P, _u32, _P, _P, _P, _P, _P]
        l.hx_ref_rollout_worker.restype = _int
        l.hx_ref_rollout_worker.argtypes = [_P, _P, _P, _P]
        l.hx_ref_reward_score.restype = _int
        l.hx_ref_reward_score.argtypes = [_P, _int, _P]
        l.hx_ref_kv_branch_resolve.restype = _int
        l.hx_ref_kv_branch_resolve.argtypes = [_P, _P, _P, _int]
        l.hx_ref_sizeof.restype = _u64
        l.hx_ref_sizeof.argtypes = [_int]
        self.lib = l

    def sizeof(self, what):
        """sizeof of the reference's RequestRing (0), DoneRing (1),
        GpuRolloutState (2), KVPrefixTable (3), RewardDesc (4)."""
        return int(self.lib.hx_ref_sizeof(what))

    def rollout_worker(self, req_ring, done_ring, state, step_count):
        """The reference rollout_worker<<<1, 32>>> (cu/gpu_scheduler.cu:26-83,
        unmodified) on torch uint8 device buffers holding a RequestRing
        filled before the launch (ending with the stop sentinel), an empty
        DoneRing, a GpuRolloutState and a uint64 step counter.  The harness
        refuses ring contents on which the kernel could wait forever."""
        rc = self.lib.hx_ref_rollout_worker(req_ring.data_ptr(), done_ring.data_ptr(),
                                            state.data_ptr(), step_count.data_ptr())
        assert rc == 0, f"reference rollout_worker not run / failed: {rc}"

    def reward_score(self, descs, scores):
        """reference reward_score_kernel (cu/reward.cu:4-15) over torch device
        buffers: descs uint8 [n * 24] (RewardDesc), scores fp32 [n]."""
        n = descs.numel() // 24
        rc = self.lib.hx_ref_reward_score(descs.data_ptr(), n,
                                          None if scores is None else scores.data_ptr())
        assert rc == 0, f"reference reward_score_kernel failed: {rc}"

    def kv_branch_resolve(self, table, ids, out):
        """reference kv_branch_resolve (cu/kv_prefix.cu:17-23) over torch
        device buffers: table uint8 (a KVPrefixTable), ids int32, out int64."""
        rc = self.lib.hx_ref_kv_branch_resolve(table.data_ptr(), ids.data_ptr(), out.data_ptr(),
                                               ids.numel())
        assert rc == 0, f"reference kv_branch_resolve failed: {rc}"

    def fixed128(self, descs, arena, block_size, sample_st=None, q_buf=None, io_slots=0):
        """The reference's attention_decode_step_fixed128 (cu/attention_decode.cu,
        unmodified) over DESCRIPTOR_DTYPE records.  arena: torch uint8 on the
        GPU; sample_st: torch 48-byte SampleState on the GPU or None; q_buf:
        torch fp16 [rows][128] on the GPU or None.  Returns numpy (o [n][128],
        token, bytes, tiles, cycles)."""
        import torch
        descs = np.ascontiguousarray(descs, dtype=DESCRIPTOR_DTYPE)
        n = len(descs)
        n_blocks = arena.numel() // block_size
        # the harness reads whole 16 KiB blocks and q rows: check bounds here
        assert block_size >= 16384 and n_blocks > 0
        assert np.all(descs["kv_block_offset"] < n_blocks), "block outside the arena"
        if q_buf is not None:
            rows = q_buf.shape[0]
            slots = descs["output_token_offset"] & (io_slots - 1) if io_slots else np.zeros(n)
            assert q_buf.shape[1] == 128 and np.all(slots < rows)
        dev = arena.device
        d = torch.from_numpy(descs.view(np.uint8).copy()).to(dev)
        o = torch.zeros(n, 128, dtype=torch.float32, device=dev)
        tok = torch.zeros(n, dtype=torch.int32, device=dev)
        byt = torch.zeros(n, dtype=torch.int32, device=dev)
        til = torch.zeros(n, dtype=torch.int32, device=dev)
        cyc = torch.zeros(n, dtype=torch.int64, device=dev)
        rc = self.lib.hx_ref_fixed128(
            d.data_ptr(), n, arena.data_ptr(), block_size,
            None if sample_st is None else sample_st.data_ptr(),
            None if q_buf is None else q_buf.data_ptr(), io_slots, o.data_ptr(), tok.data_ptr(),
            byt.data_ptr(), til.data_ptr(), cyc.data_ptr())
        assert rc == 0, f"reference fixed128 step failed: {rc}"
        u32 = lambda t: t.cpu().numpy().view(np.uint32)
        return o.cpu().numpy(), u32(tok), u32(byt), u32(til), cyc.cpu().numpy().view(np.uint64)

    def sample_rows(self, logits, vocab, temperature, top_k, top_p, u24):
        """logits: torch fp32 [R, stride] on the GPU (copied; the reference
        filters in place).  Per-row arrays are numpy.  Returns numpy uint32."""
        import torch
        R = logits.shape[0]
        dev = logits.device
        work = logits.clone()
        bc = lambda x, dt: torch.from_numpy(np.ascontiguousarray(np.broadcast_to(x, R), dtype=dt)).to(dev)
        t = bc(temperature, np.float32)
        k = bc(top_k, np.int16)  # uint16 bits
        p = bc(top_p, np.float32)
        s1 = np.array([xoshiro_s1_for_first_output(int(u)) for u in np.broadcast_to(u24, R)],
                      dtype=np.uint64)
        s1t = torch.from_numpy(s1.view(np.int64)).to(dev)
        out = torch.zeros(R, dtype=torch.int32, device=dev)
        rc = self.lib.hx_ref_sample_rows(work.data_ptr(), vocab, work.stride(0), t.data_ptr(),
                                         k.data_ptr(), p.data_ptr(), s1t.data_ptr(),
                                         out.data_ptr(), R)
        assert rc == 0, f"reference sampler failed: {rc}"
        return out.cpu().numpy().view(np.uint32)
