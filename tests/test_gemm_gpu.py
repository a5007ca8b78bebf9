"""bf16 GEMM on the tensor cores (rt_gemm_bf16, tcgen05) against a float64
product of the same bf16 inputs computed by torch.

Tolerance: fp32 accumulation of exact bf16 products, so the error of each
output is bounded by a small multiple of 2^-24 * K * sum_k |a_k b_k|; the
test allows |C - C64| <= 2^-16 * sum_k |a_k b_k| + 1e-6 (far inside that
bound for K <= 4096, far outside any layout or indexing error)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def gemm(pkg, A, B, C=None, split_k=0, accumulate=False, ldc=None):
    M, K = A.shape
    N = B.shape[0]
    if C is None:
        C = torch.full((M, ldc or N), float("nan"), dtype=torch.float32, device=A.device)
    p = pkg.rt_gemm_params_t(M, N, K, A.stride(0), B.stride(0), C.stride(0), split_k,
                             1 if accumulate else 0)
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    wsb = pkg.lib().rt_gemm_workspace_bytes(ctypes.byref(p))
    ws = torch.full((max(wsb, 4) // 4,), float("nan"), device=A.device) if wsb else None
    pkg.check(pkg.lib().rt_gemm_bf16(ctypes.byref(p), pkg._ptr(A), pkg._ptr(B), pkg._ptr(C),
                                     pkg._ptr(ws), wsb, pkg._ptr(err), pkg._stream_ptr(None)),
              "rt_gemm_bf16")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return C


def check(C, A, B, base=None):
    A64, B64 = A.double(), B.double()
    ref = A64 @ B64.T
    if base is not None:
        ref = ref + base.double()
    bound = (A64.abs() @ B64.abs().T) * 2.0 ** -16 + 1e-6
    err = (C.double() - ref).abs()
    bad = err > bound
    assert not bool(bad.any()), f"{int(bad.sum())} of {bad.numel()} outside; max err {err.max():.3e}"


def rand(shape, seed, dev, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 224, 64), (1, 1, 64), (130, 300, 128), (256, 448, 640),
                                   (200, 1000, 256), (384, 32, 4096)])
def test_gemm_shapes(pkg, cuda, M, N, K):
    A, B = rand((M, K), 1, cuda), rand((N, K), 2, cuda)
    check(gemm(pkg, A, B), A, B)


def test_gemm_lm_head_shape(pkg, cuda):
    """The decode step's LM head: 256 slots x 4096 -> 32,000 logits."""
    A, B = rand((256, 4096), 3, cuda), rand((32000, 4096), 4, cuda, scale=0.02)
    check(gemm(pkg, A, B), A, B)


@pytest.mark.parametrize("split", [2, 4, 7, 64])
def test_gemm_split_k(pkg, cuda, split):
    """The QKV projection shape (N = 6,144) with K divided among CTAs."""
    A, B = rand((256, 4096), 5, cuda), rand((6144, 4096), 6, cuda, scale=0.02)
    check(gemm(pkg, A, B, split_k=split), A, B)


def test_gemm_accumulate_and_strides(pkg, cuda):
    """C += A B^T into a wider C; A and B are row slices of larger buffers."""
    Abig, Bbig = rand((160, 1024), 7, cuda), rand((520, 640), 8, cuda)
    A, B = Abig[:, 64:64 + 512], Bbig[:, :512]
    base = torch.randn(160, 600, device=cuda)
    C = base.clone()
    gemm(pkg, A, B, C=C, accumulate=True)
    check(C[:, :520], A, B, base=base[:, :520])
    assert torch.equal(C[:, 520:], base[:, 520:])   # columns past N untouched
    C2 = base.clone()
    gemm(pkg, A, B, C=C2, accumulate=True, split_k=3)
    check(C2[:, :520], A, B, base=base[:, :520])


def test_gemm_rejects_bad_shapes(pkg, cuda):
    A, B = rand((8, 100), 9, cuda), rand((8, 100), 10, cuda)
    with pytest.raises(pkg.RuntimeErrorRT, match="multiple of 64"):
        gemm(pkg, A, B)
    A, B = rand((8, 128), 9, cuda), rand((8, 128), 10, cuda)
    p = pkg.rt_gemm_params_t(8, 8, 128, 128, 128, 8, 2, 0)
    C = torch.empty(8, 8, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = pkg.lib().rt_gemm_bf16(ctypes.byref(p), pkg._ptr(A), pkg._ptr(B), pkg._ptr(C), None, 0,
                                pkg._ptr(err), pkg._stream_ptr(None))
    assert rc == pkg.RT_ENOMEM


def test_gemm_split_k_is_deterministic(pkg, cuda):
    """K-splits add in split order: repeated calls give identical bits."""
    A, B = rand((256, 4096), 11, cuda), rand((2048, 4096), 12, cuda, scale=0.05)
    first = gemm(pkg, A, B, split_k=14)
    for _ in range(3):
        assert torch.equal(gemm(pkg, A, B, split_k=14), first)
    check(first, A, B)


def gemm_cmax(pkg, A, B, split_k=0, accumulate=False, ldc=None, base=None):
    """rt_gemm_bf16_chunk_max; returns (C, chunk maxima)."""
    M, K = A.shape
    N = B.shape[0]
    C = torch.full((M, ldc or N), float("nan"), dtype=torch.float32, device=A.device)
    if base is not None:
        C[:, :N] = base
    cs = pkg.chunk_max_stride(N)
    cm = torch.full((M, cs), -7.0, dtype=torch.float32, device=A.device)
    p = pkg.rt_gemm_params_t(M, N, K, A.stride(0), B.stride(0), C.stride(0), split_k,
                             1 if accumulate else 0)
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    wsb = pkg.lib().rt_gemm_workspace_bytes(ctypes.byref(p))
    ws = torch.full((max(wsb, 4) // 4,), float("nan"), device=A.device) if wsb else None
    pkg.check(pkg.lib().rt_gemm_bf16_chunk_max(ctypes.byref(p), pkg._ptr(A), pkg._ptr(B),
                                               pkg._ptr(C), pkg._ptr(ws), wsb, pkg._ptr(err),
                                               pkg._ptr(cm), cs, pkg._stream_ptr(None)),
              "rt_gemm_bf16_chunk_max")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return C, cm


def chunk_max_of(C, N):
    x = C[:, :N].double().cpu().numpy()
    M = x.shape[0]
    nch = (N + 15) // 16
    pad = np.full((M, nch * 16), -np.inf)
    pad[:, :N] = x
    c = pad.reshape(M, nch, 16)
    m = c.max(axis=2)
    m[np.isnan(c).any(axis=2)] = np.nan
    return m


@pytest.mark.parametrize("M,N,K,split,acc,ldc", [
    (256, 32000 // 8, 256, 0, False, None),   # epilogue path, TMA stores
    (130, 300, 128, 0, False, 301),           # epilogue path, plain stores, N % 16 != 0
    (64, 1000, 512, 4, False, None),          # K-splits: maxima from C afterwards
    (64, 448, 128, 0, True, None),            # accumulate: maxima from C afterwards
])
def test_gemm_chunk_max(pkg, cuda, M, N, K, split, acc, ldc):
    """The LM head's maxima for the sampler equal the maxima of the C it
    wrote, whichever path produced them."""
    A, B = rand((M, K), 1, cuda), rand((N, K), 2, cuda)
    base = rand((M, N), 3, cuda).float() if acc else None
    C, cm = gemm_cmax(pkg, A, B, split_k=split, accumulate=acc, ldc=ldc, base=base)
    check(C[:, :N], A, B, base)
    want = chunk_max_of(C, N)
    got = cm[:, : want.shape[1]].double().cpu().numpy()
    assert np.array_equal(got, want)


def test_gemm_chunk_max_propagates_nan(pkg, cuda):
    M, N, K = 32, 224, 64
    A, B = rand((M, K), 4, cuda), rand((N, K), 5, cuda)
    A[3, 7] = float("nan")                    # row 3 of C is all NaN
    B[40, 0] = float("inf")                   # column 40 is +-inf or NaN
    C, cm = gemm_cmax(pkg, A, B)
    want = chunk_max_of(C, N)
    got = cm[:, : want.shape[1]].double().cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])
    assert np.isnan(got[3]).all()
