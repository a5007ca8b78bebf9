"""Shared-prefix (cascade) decode attention on the GPU through the C ABI
(rt_paged_decode_attention_grouped), against the CPU oracle (fp64) and
against the ungrouped entry point on the same inputs.  Tolerance as for the
plain kernel: 2e-3 absolute + 1e-2 relative (bf16 KV, fp32 accumulate)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def make_grouped_case(pkg, dev, groups, loose, Hq, Hkv, seed):
    """groups: [(shared_pages, [suffix_len per member])]; loose: lengths of
    sequences in no group.  Members share their group's first pages."""
    rng = np.random.default_rng(seed)
    lens, table_rows, recs, skip = [], [], [], []
    next_page = [0]

    def take(n):
        out = list(range(next_page[0], next_page[0] + n))
        next_page[0] += n
        return out

    for shared, suffixes in groups:
        common = take(shared)
        members = []
        for suf in suffixes:
            L = shared * 16 + suf
            own = take((L + 15) // 16 - shared)
            members.append(len(lens))
            lens.append(L)
            table_rows.append(common + own)
            skip.append(shared)
        recs.append((shared, members))
    for L in loose:
        table_rows.append(take((L + 15) // 16))
        lens.append(L)
        skip.append(0)
    # scatter: permute physical pages
    n_pages = next_page[0]
    arena_pages = int(n_pages * 1.2) + 2
    perm = rng.permutation(arena_pages).astype(np.int32)
    P = max(1, max(len(r) for r in table_rows))
    pt = np.full((len(lens), P), -7, dtype=np.int32)
    for b, row in enumerate(table_rows):
        pt[b, :len(row)] = perm[row]
    order = rng.permutation(len(lens))            # members not contiguous in the batch
    inv = np.argsort(order)
    pt = pt[order]
    lens = np.asarray(lens, dtype=np.int32)[order]
    skip = np.asarray(skip, dtype=np.uint32)[order]
    recs = [(s, [int(inv[m]) for m in mem]) for s, mem in recs]
    arena = torch.empty(arena_pages * Hkv * 2 * 16 * 128, dtype=torch.bfloat16, device=dev)
    q = torch.empty(len(lens), Hq, 128, dtype=torch.bfloat16, device=dev)
    pkg.fill_normal_bf16(arena, seed=seed, stream_id=1)
    pkg.fill_normal_bf16(q, seed=seed, stream_id=2)
    return q, arena, pt, lens, skip, recs, arena_pages, P


def run_grouped(pkg, dev, case, Hq, Hkv, gchunk=0, max_groups=None, chunk_pages=0, repeat=1):
    q, arena, pt, lens, skip, recs, ap, P = case
    max_shared = max([s for s, _ in recs] + [0])
    mg = max_groups or max(1, len(recs))
    attn = pkg.GroupedDecodeAttention(len(lens), Hq, Hkv, P, int(max(lens.max(), 1)), ap, mg,
                                      max_shared, group_chunk_pages=gchunk,
                                      chunk_pages=chunk_pages)
    tab = torch.from_numpy(pkg.group_table(recs, mg).view(np.int32)).to(dev)
    ng = torch.tensor([len(recs)], dtype=torch.int32, device=dev)
    sk = torch.from_numpy(skip.view(np.int32)).to(dev)
    ptd, ld = torch.from_numpy(pt).to(dev), torch.from_numpy(lens).to(dev)
    outs = []
    for _ in range(repeat):
        outs.append(attn(q, arena, ptd, ld, tab, ng, sk).clone())
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs], attn


def check_oracle(orc, case, Hq, Hkv, got):
    q, arena, pt, lens = case[0], case[1], case[2], case[3]
    ref = orc.paged_gqa_attention(bits(q), bits(arena), pt, lens, Hq, Hkv, 128 ** -0.5)
    err = np.abs(got - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} mismatches, max abs err {err.max():.3e}"
    return ref


GROUPS = [(32, [0, 1, 15, 16, 17, 100, 256, 5, 9, 33, 64, 65, 128, 200, 255, 3]),  # 16 members
          (3, [40, 2, 0]),
          (1, [7]),
          (20, [300, 301, 302, 303, 304])]
LOOSE = [0, 1, 300, 2049]


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_grouped_matches_oracle_and_plain(pkg, orc, cuda, G):
    Hkv = 8 if G <= 4 else 4
    Hq = Hkv * G
    case = make_grouped_case(pkg, cuda, GROUPS, LOOSE, Hq, Hkv, seed=40 + G)
    (got,), attn = run_grouped(pkg, cuda, case, Hq, Hkv)
    assert attn.error_code() == 0
    check_oracle(orc, case, Hq, Hkv, got)
    q, arena, pt, lens, _, _, ap, P = case
    plain = pkg.PagedDecodeAttention(len(lens), Hq, Hkv, P, int(lens.max()), ap)
    want = plain(q, arena, torch.from_numpy(pt).to(cuda),
                 torch.from_numpy(lens).to(cuda)).cpu().numpy()
    assert np.all(np.abs(got - want) <= ATOL + RTOL * np.abs(want))
    assert np.all(got[lens == 0] == 0.0)


@pytest.mark.parametrize("gchunk,chunk_pages", [(1, 0), (3, 2), (8, 0), (64, 1), (5, 64)])
def test_group_chunk_sizes(pkg, orc, cuda, gchunk, chunk_pages):
    case = make_grouped_case(pkg, cuda, GROUPS, LOOSE, 32, 8, seed=7)
    (got,), attn = run_grouped(pkg, cuda, case, 32, 8, gchunk=gchunk, chunk_pages=chunk_pages)
    assert attn.error_code() == 0
    check_oracle(orc, case, 32, 8, got)


def test_grouped_repeat_deterministic_and_spare_capacity(pkg, orc, cuda):
    """Three calls on one workspace (dispensers and counters must reset);
    the group array holds more records than are live."""
    case = make_grouped_case(pkg, cuda, GROUPS, LOOSE, 32, 8, seed=8)
    outs, attn = run_grouped(pkg, cuda, case, 32, 8, max_groups=64, repeat=3)
    assert attn.error_code() == 0
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    check_oracle(orc, case, 32, 8, outs[0])


def test_grpo_shape(pkg, orc, cuda):
    """The rollout loop's shape: 16 groups x 16 members, 32 shared pages of
    prompt, generated suffixes of 0..255 tokens, 32q/8kv."""
    rng = np.random.default_rng(12)
    groups = [(32, list(rng.integers(0, 256, size=16))) for _ in range(16)]
    case = make_grouped_case(pkg, cuda, groups, [], 32, 8, seed=12)
    (got,), attn = run_grouped(pkg, cuda, case, 32, 8)
    assert attn.error_code() == 0
    check_oracle(orc, case, 32, 8, got)


def test_group_contract_violation_is_flagged(pkg, orc, cuda):
    """A member whose skip_pages disagrees with its group record is skipped
    and error 4 is reported; nothing faults.  Reading the error clears the
    part-counted arrival counters: the next good call on the same workspace
    matches the oracle."""
    case = make_grouped_case(pkg, cuda, [(4, [10, 20, 30])], [50], 32, 8, seed=9)
    q, arena, pt, lens, skip, recs, ap, P = case
    bad_skip = skip.copy()
    bad_skip[recs[0][1][1]] = 3
    bad = (q, arena, pt, lens, bad_skip, recs, ap, P)
    _, attn = run_grouped(pkg, cuda, bad, 32, 8)
    assert attn.error_code() == 4
    tab = torch.from_numpy(pkg.group_table(recs, 1).view(np.int32)).to(cuda)
    ng = torch.tensor([len(recs)], dtype=torch.int32, device=cuda)
    out = attn(q, arena, torch.from_numpy(pt).to(cuda), torch.from_numpy(lens).to(cuda), tab, ng,
               torch.from_numpy(skip.view(np.int32)).to(cuda)).cpu().numpy()
    assert attn.error_code() == 0
    check_oracle(orc, case, 32, 8, out)
