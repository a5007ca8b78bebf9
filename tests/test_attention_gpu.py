"""Paged GQA decode attention on the GPU, through the C ABI, against the CPU
oracle (fp64 accumulation).  Tolerance: 2e-3 absolute + 1e-2 relative
(bf16 KV, fp32 accumulate), as the parity contract states."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def make_case(pkg, dev, lens, Hq, Hkv, seed, slack=1.3, max_pages=None):
    lens = np.asarray(lens, dtype=np.int32)
    rng = np.random.default_rng(seed)
    n_pages = [(int(L) + 15) // 16 for L in lens]
    P = max_pages or max(1, max(n_pages))
    total = sum(n_pages)
    arena_pages = max(1, int(total * slack) + 1)
    perm = rng.permutation(arena_pages).astype(np.int32)
    pt = np.full((len(lens), P), -7, dtype=np.int32)   # unused entries stay invalid
    k = 0
    for b, n in enumerate(n_pages):
        pt[b, :n] = perm[k:k + n]
        k += n
    arena = torch.empty(arena_pages * Hkv * 2 * 16 * 128, dtype=torch.bfloat16, device=dev)
    q = torch.empty(len(lens), Hq, 128, dtype=torch.bfloat16, device=dev)
    pkg.fill_normal_bf16(arena, seed=seed, stream_id=1)
    pkg.fill_normal_bf16(q, seed=seed, stream_id=2)
    return q, arena, pt, lens, arena_pages, P


def run(pkg, dev, q, arena, pt, lens, Hq, Hkv, arena_pages, P, chunk_pages=0, max_seq_len=None):
    attn = pkg.PagedDecodeAttention(len(lens), Hq, Hkv, P, int(max_seq_len or max(lens.max(), 1)),
                                    arena_pages, chunk_pages=chunk_pages)
    out = attn(q, arena, torch.from_numpy(pt).to(dev), torch.from_numpy(lens).to(dev))
    torch.cuda.synchronize()
    return out.cpu().numpy(), attn


def check(orc, q, arena, pt, lens, Hq, Hkv, got):
    ref = orc.paged_gqa_attention(bits(q), bits(arena), pt, lens, Hq, Hkv, 128 ** -0.5)
    err = np.abs(got - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} mismatches, max abs err {err.max():.3e}"
    return err.max()


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_group_sizes(pkg, orc, cuda, G):
    Hkv = 4 if G < 8 else 2
    Hq = Hkv * G
    lens = [1, 15, 16, 17, 100, 257]
    case = make_case(pkg, cuda, lens, Hq, Hkv, seed=G)
    got, attn = run(pkg, cuda, *case[:4], Hq, Hkv, case[4], case[5], chunk_pages=4)
    assert attn.error_code() == 0
    check(orc, *case[:4], Hq, Hkv, got)


@pytest.mark.parametrize("chunk_pages", [1, 2, 3, 8, 32, 64])
def test_chunk_sizes_agree(pkg, orc, cuda, chunk_pages):
    lens = [16 * 128, 16 * 37 + 5, 33, 2049]
    case = make_case(pkg, cuda, lens, 32, 8, seed=11)
    got, attn = run(pkg, cuda, *case[:4], 32, 8, case[4], case[5], chunk_pages=chunk_pages)
    assert attn.error_code() == 0
    check(orc, *case[:4], 32, 8, got)


def test_empty_and_ragged(pkg, orc, cuda):
    lens = [0, 1, 0, 31, 4096, 0, 129]
    case = make_case(pkg, cuda, lens, 32, 8, seed=5)
    got, attn = run(pkg, cuda, *case[:4], 32, 8, case[4], case[5])
    assert attn.error_code() == 0
    assert np.all(got[[0, 2, 5]] == 0.0)
    check(orc, *case[:4], 32, 8, got)


def test_deterministic_and_workspace_reusable(pkg, orc, cuda):
    lens = np.random.default_rng(3).integers(128, 4097, size=16)
    case = make_case(pkg, cuda, lens, 32, 8, seed=3)
    q, arena, pt, lens_, ap, P = case
    attn = pkg.PagedDecodeAttention(len(lens_), 32, 8, P, int(lens_.max()), ap, chunk_pages=4)
    ptd, ld = torch.from_numpy(pt).to(cuda), torch.from_numpy(lens_).to(cuda)
    a = attn(q, arena, ptd, ld).clone()
    b = attn(q, arena, ptd, ld).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert attn.error_code() == 0
    check(orc, q, arena, pt, lens_, 32, 8, a.cpu().numpy())


def test_bad_inputs_reported_not_faulting(pkg, cuda):
    lens = [40, 20]
    q, arena, pt, lens_, ap, P = make_case(pkg, cuda, lens, 32, 8, seed=9)
    # page index outside the arena -> error code 2, no out-of-bounds access
    pt_bad = pt.copy()
    pt_bad[0, 1] = ap + 1000
    _, attn = run(pkg, cuda, q, arena, pt_bad, lens_, 32, 8, ap, P)
    assert attn.error_code() == 2
    # sequence longer than the declared max -> error code 1, sequence skipped
    lens_bad = np.array([40, 33], dtype=np.int32)
    _, attn = run(pkg, cuda, q, arena, pt, lens_bad, 32, 8, ap, P, max_seq_len=32)
    assert attn.error_code() == 1


def test_c2_full_config(pkg, orc, cuda):
    """B=64, L ~ U[128,4096] (seed 2), 32q/8kv, d=128,
    bf16 pages scattered in the arena, Q/K/V ~ N(0,1)."""
    lens = np.random.default_rng(2).integers(128, 4097, size=64).astype(np.int32)
    case = make_case(pkg, cuda, lens, 32, 8, seed=2, slack=1.25)
    got, attn = run(pkg, cuda, *case[:4], 32, 8, case[4], case[5])
    assert attn.error_code() == 0
    err = check(orc, *case[:4], 32, 8, got)
    assert err < 1e-3


@pytest.mark.parametrize("B", [512, 600])
def test_many_sequences_both_item_numberings(pkg, orc, cuda, B):
    """Up to 512 sequences the kernel builds a per-CTA item table (no empty
    items); beyond it, items are numbered statically (chunk, sequence, head)
    with empty items past each sequence's end.  Both must match the oracle,
    with zero-length sequences and multi-chunk ones mixed in."""
    rng = np.random.default_rng(B)
    lens = rng.integers(0, 200, size=B).astype(np.int32)
    lens[::7] = 0
    lens[3::50] = 700          # several chunks at chunk_pages 8
    case = make_case(pkg, cuda, lens, 8, 2, seed=B)
    got, attn = run(pkg, cuda, *case[:4], 8, 2, case[4], case[5], chunk_pages=8)
    assert attn.error_code() == 0
    assert np.all(got[lens == 0] == 0.0)
    check(orc, *case[:4], 8, 2, got)
