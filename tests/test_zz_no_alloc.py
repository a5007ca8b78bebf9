"""Allocation-free paged attention (rt_paged_decode_attention_noalloc).

Callers that must not allocate device memory where they run decode
attention (a no-allocation hot path, a host that owns all device memory, a
loop where cudaMalloc would synchronise) use this entry point: its split-K
scratch is a fixed array inside the library.  These checks call it through
the C ABI and compare it with the workspace entry point on the same inputs,
twice in a row, since the array keeps the previous call's contents.  The file
is named to be collected last and depends on no other test."""
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


def test_noalloc_matches_workspace_entry_point_twice(pkg, cuda):
    fn = _bind(pkg)
    q, arena, pt, lens_d, lens, P, ap = _case(pkg, cuda, seed=31)
    attn = pkg.PagedDecodeAttention(len(lens), 32, 8, P, int(lens.max()), ap)
    want = attn(q, arena, pt, lens_d).clone()
    torch.cuda.synchronize()
    assert attn.error_code() == 0
    stream = torch.cuda.current_stream()
    for _ in range(2):
        out = torch.full_like(want, float("nan"))
        rc = fn(ctypes.byref(attn.params), q.data_ptr(), arena.data_ptr(), pt.data_ptr(),
                lens_d.data_ptr(), out.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, pkg.lib().rt_last_error()
        torch.cuda.synchronize()
        got, ref = out.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.abs(got - ref) <= ATOL + RTOL * np.abs(ref))


def test_noalloc_rejects_shapes_beyond_its_scratch(pkg):
    fn = _bind(pkg)
    # 4096 sequences x 8 heads x 64 chunks of partials is far beyond 32 MiB
    p = pkg.rt_attn_params_t(4096, 32, 8, 128, 1024, 16384, 1 << 20, 128 ** -0.5, 16, 0)
    rc = fn(ctypes.byref(p), 16, 16, 16, 16, 16, None)
    assert rc == pkg.RT_ENOMEM
    assert b"scratch" in pkg.lib().rt_last_error()
