"""Allocation-free paged attention (rt_paged_decode_attention_noalloc).

Callers that must not allocate device memory where they run decode
attention (a no-allocation hot path, a host that owns all device memory, a
loop where cudaMalloc would synchronise) use this entry point: its split-K
scratch is a fixed array inside the library.  These checks call it through
the C ABI and compare it with the workspace entry point on the same inputs,
twice in a row, since the array keeps the previous call's contents, and
check that the calls after the first leave device memory untouched (the
driver's free bytes and torch's allocator).  The file is named to be
collected last and depends on no other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _bind(pkg):
    fn = pkg.lib().rt_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(pkg.rt_attn_params_t)] + [ctypes.c_void_p] * 6
    return fn


def _case(pkg, dev, seed, n_seqs=24, max_len=3000):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_len + 1, size=n_seqs).astype(np.int32)
    lens[0] = 0
    n_pages = (lens + 15) // 16
    P = int(n_pages.max())
    arena_pages = int(n_pages.sum() * 1.2) + 1
    pt = np.zeros((n_seqs, P), dtype=np.int32)
    perm = rng.permutation(arena_pages).astype(np.int32)
    k = 0
    for b, n in enumerate(n_pages):
        pt[b, :n] = perm[k:k + n]
        k += n
    arena = torch.empty(arena_pages * 8 * 2 * 16 * 128, dtype=torch.bfloat16, device=dev)
    q = torch.empty(n_seqs, 32, 128, dtype=torch.bfloat16, device=dev)
    pkg.fill_normal_bf16(arena, seed=seed, stream_id=1)
    pkg.fill_normal_bf16(q, seed=seed, stream_id=2)
    return q, arena, torch.from_numpy(pt).to(dev), torch.from_numpy(lens).to(dev), lens, P, \
        arena_pages


def _call(pkg, fn, params, q, arena, pt, lens_d, out, stream):
    rc = fn(ctypes.byref(params), q.data_ptr(), arena.data_ptr(), pt.data_ptr(),
            lens_d.data_ptr(), out.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, pkg.lib().rt_last_error()


def _error(pkg, stream):
    code = ctypes.c_int32(-99)
    rc = pkg.lib().rt_paged_decode_attention_noalloc_error(ctypes.byref(code),
                                                           ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, pkg.lib().rt_last_error()
    return code.value


def test_noalloc_matches_workspace_entry_point_twice(pkg, cuda):
    fn = _bind(pkg)
    q, arena, pt, lens_d, lens, P, ap = _case(pkg, cuda, seed=31)
    attn = pkg.PagedDecodeAttention(len(lens), 32, 8, P, int(lens.max()), ap)
    want = attn(q, arena, pt, lens_d).clone()
    torch.cuda.synchronize()
    assert attn.error_code() == 0
    stream = torch.cuda.current_stream()
    outs = [torch.full_like(want, float("nan")) for _ in range(2)]
    # the first call on the device resolves the array's address; the calls
    # after it must leave device memory untouched (no allocation anywhere)
    _call(pkg, fn, attn.params, q, arena, pt, lens_d, outs[0], stream)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch_bytes0 = torch.cuda.memory_allocated()
    for i in range(2):
        out = outs[i]
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        free_a, _ = torch.cuda.mem_get_info()
        _call(pkg, fn, attn.params, q, arena, pt, lens_d, out, stream)
        torch.cuda.synchronize()
        free_b, _ = torch.cuda.mem_get_info()
        assert free_b == free_a == free0, "device memory changed across a no-alloc call"
        assert torch.cuda.memory_allocated() == torch_bytes0
        assert _error(pkg, stream) == 0
        got, ref = out.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.abs(got - ref) <= ATOL + RTOL * np.abs(ref))


def test_noalloc_error_word_is_readable(pkg, cuda):
    """A page id outside the arena is caught by the kernel's bounds check
    (the load is clamped into the arena) and reported through
    rt_paged_decode_attention_noalloc_error until the next call clears it."""
    fn = _bind(pkg)
    q, arena, pt, lens_d, lens, P, ap = _case(pkg, cuda, seed=37, n_seqs=8, max_len=400)
    attn = pkg.PagedDecodeAttention(len(lens), 32, 8, P, int(lens.max()), ap)
    stream = torch.cuda.current_stream()
    out = torch.zeros(len(lens), 32, 128, dtype=torch.float32, device=cuda)
    bad = pt.clone()
    b = int(np.argmax(lens))
    bad[b, 0] = ap + 5  # outside the arena
    _call(pkg, fn, attn.params, q, arena, bad, lens_d, out, stream)
    assert _error(pkg, stream) == 2
    assert _error(pkg, stream) == 0  # read and cleared
    _call(pkg, fn, attn.params, q, arena, bad, lens_d, out, stream)
    _call(pkg, fn, attn.params, q, arena, pt, lens_d, out, stream)  # clears the earlier code
    assert _error(pkg, stream) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(pkg):
    fn = _bind(pkg)
    # 4096 sequences x 8 heads x 64 chunks of partials is far beyond 32 MiB
    p = pkg.rt_attn_params_t(4096, 32, 8, 128, 1024, 16384, 1 << 20, 128 ** -0.5, 16, 0)
    rc = fn(ctypes.byref(p), 16, 16, 16, 16, 16, None)
    assert rc == pkg.RT_ENOMEM
    assert b"scratch" in pkg.lib().rt_last_error()
