"""Sampler given producer chunk maxima (rt_sample_rows_cmax) and the chunk
maximum kernel (rt_logits_chunk_max).  The tokens must equal, bit for bit,
those of the reference's own sample_token (reference cu/sample.cu, compiled
unmodified for sm_100a into oracle/_ref) and of rt_sample_rows, which reads
the whole row, on the same logits and uniforms."""
import zlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SEED = 1234


def u24s(pkg, rollouts, steps, seed=SEED):
    r, s = np.broadcast_arrays(np.asarray(rollouts), np.asarray(steps))
    return np.array([pkg.sample_uniform24(seed, int(a), int(b)) for a, b in zip(r, s)],
                    dtype=np.uint32)


def normal_logits(pkg, cuda, R, V, seed, std=2.0, stride=None):
    t = torch.empty(R, stride or V, dtype=torch.float32, device=cuda)
    pkg.fill_normal_f32(t, seed=seed, stream_id=3, std=std)
    return t


@pytest.fixture(scope="module")
def refcuda(orc):
    try:
        return orc.RefCuda()
    except OSError as e:
        pytest.skip(str(e))


def chunk_max_numpy(x, V):
    """Each 16-column chunk's maximum of x[:, :V], NaN if the chunk has one."""
    R = x.shape[0]
    nch = (V + 15) // 16
    pad = np.full((R, nch * 16), -np.inf, dtype=np.float32)
    pad[:, :V] = x[:, :V]
    c = pad.reshape(R, nch, 16)
    m = c.max(axis=2)
    m[np.isnan(c).any(axis=2)] = np.nan
    return m


def both(pkg, logits, V, T, k, p, rid, step, fused=True):
    rows = pkg.sample_row_table(T, k, p, rid, step, SEED)
    rows_d = torch.from_numpy(rows.view(np.uint8)).to(logits.device)
    cm = pkg.logits_chunk_max(logits, V)
    a = pkg.sample_rows_cmax(logits, cm, rows_d, V, fused_cum=fused).cpu().numpy().view(np.uint32)
    b = pkg.sample_rows(logits, rows_d, V, fused_cum=fused).cpu().numpy().view(np.uint32)
    return a, b, cm


@pytest.mark.parametrize("V,stride", [(32000, None), (7, None), (4099, 4101), (100000, None),
                                      (16, None), (33, 40)])
def test_chunk_max_kernel_matches_numpy(pkg, cuda, V, stride):
    R = 6
    x = normal_logits(pkg, cuda, R, V, seed=V & 0xFFFF, stride=stride)
    if V > 20:
        x[1, 17] = float("nan")
        x[2, V - 1] = float("inf")
        x[3, :] = -float("inf")
        x[4, 3] = float("nan")
        x[4, 4] = float("inf")
    cm = pkg.logits_chunk_max(x, V).cpu().numpy()
    assert cm.shape[1] == pkg.chunk_max_stride(V) and cm.shape[1] % 4 == 0
    want = chunk_max_numpy(x.cpu().numpy(), V)
    got = cm[:, : want.shape[1]]
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])


def test_c3_cmax_bit_exact_against_reference_kernel(pkg, cuda, refcuda):
    """BASELINE config 3 through the chunk-maximum path."""
    R, V = 256, 32000
    logits = normal_logits(pkg, cuda, R, V, seed=3)
    rid = np.arange(R, dtype=np.uint32)
    ref = refcuda.sample_rows(logits, V, 0.8, 50, 0.9, u24s(pkg, rid, 0))
    a, b, _ = both(pkg, logits, V, 0.8, 50, 0.9, rid, 0)
    assert np.array_equal(a, ref), f"{(a != ref).sum()}/{R} rows differ"
    assert np.array_equal(a, b)


@pytest.mark.parametrize("case", ["topk_off", "topk_over_256", "no_topp", "no_temperature",
                                  "k1", "small_vocab", "odd_vocab_unaligned", "vocab_100000",
                                  "ties_at_cutoff", "all_equal", "neg_inf", "nan_row",
                                  "pos_inf_row", "overflow_on_scaling", "huge_negative",
                                  "top_in_one_chunk", "top_in_one_warp"])
def test_cmax_edge_cases_bit_exact(pkg, cuda, refcuda, case):
    R, V, T, k, p = 64, 4096, 0.8, 50, 0.9
    stride = None
    if case == "small_vocab":
        V = 7
    elif case == "odd_vocab_unaligned":
        V, stride = 4099, 4101        # rows not 16-byte aligned, partial last chunk
    elif case == "vocab_100000":
        V, R = 100000, 8             # more chunk groups than threads
    logits = normal_logits(pkg, cuda, R, V, seed=zlib.crc32(case.encode()) & 0xFFFF, stride=stride)
    if case == "topk_off":
        k = 0
    elif case == "topk_over_256":
        k = 1000
    elif case == "no_topp":
        p = 1.0
    elif case == "no_temperature":
        T = 0.0
    elif case == "k1":
        k = 1
    elif case == "ties_at_cutoff":
        logits = torch.round(logits)
    elif case == "all_equal":
        logits.fill_(0.25)
    elif case == "neg_inf":
        logits[:, ::3] = -float("inf")
    elif case == "nan_row":
        logits[::2, 5] = float("nan")
    elif case == "pos_inf_row":
        logits[1::2, 17] = float("inf")
    elif case == "overflow_on_scaling":
        logits[1::3, 40] = 3.0e38      # finite, +inf once scaled by 1 / T = 1.25
    elif case == "huge_negative":
        logits.fill_(-3.0e38)
        logits[:, 3] = -3.3e38
    elif case == "top_in_one_chunk":
        logits[:, 32:48] = 20.0 + torch.arange(16, device=cuda, dtype=torch.float32) * 0.01
    elif case == "top_in_one_warp":
        # 128 chunks of one warp (columns 0..2047) hold every large value
        logits[:, :2048:3] = 20.0 + torch.arange(683, device=cuda, dtype=torch.float32) * 1e-3
    rid = np.arange(R, dtype=np.uint32) + 77
    step = np.arange(R, dtype=np.uint64) * 3 + 5
    ref = refcuda.sample_rows(logits, V, T, k, p, u24s(pkg, rid, step))
    a, b, _ = both(pkg, logits, V, T, k, p, rid, step)
    assert np.array_equal(b, ref), f"full path: {(b != ref).sum()} rows differ"
    assert np.array_equal(a, ref), f"chunk-max path: {(a != ref).sum()} rows differ"


def test_cmax_row_enable_and_unfused(pkg, cuda, refcuda):
    R, V = 32, 2000
    logits = normal_logits(pkg, cuda, R, V, seed=21)
    rid = np.arange(R, dtype=np.uint32)
    a, b, cm = both(pkg, logits, V, 1.2, 20, 0.7, rid, 4, fused=False)
    assert np.array_equal(a, b)
    rows = pkg.sample_row_table(1.2, 20, 0.7, rid, 4, SEED)
    rows_d = torch.from_numpy(rows.view(np.uint8)).to(cuda)
    en = torch.tensor([i % 3 != 0 for i in range(R)], dtype=torch.int32, device=cuda)
    out = torch.full((R,), -5, dtype=torch.int32, device=cuda)
    pkg.sample_rows_cmax(logits, cm, rows_d, V, fused_cum=False, out=out, row_enable=en)
    got = out.cpu().numpy().view(np.uint32)
    m = en.cpu().numpy().astype(bool)
    assert np.array_equal(got[m], a[m]) and np.all(got[~m].view(np.int32) == -5)


def test_cmax_arguments_checked(pkg, cuda):
    R, V = 4, 100
    logits = normal_logits(pkg, cuda, R, V, seed=2)
    rows = pkg.sample_row_table(1.0, 5, 0.9, np.arange(R, dtype=np.uint32), 0, SEED)
    rows_d = torch.from_numpy(rows.view(np.uint8)).to(cuda)
    cm = pkg.logits_chunk_max(logits, V)
    short = cm[:, :4].contiguous()    # stride below rt_chunk_max_stride(100) = 8
    with pytest.raises(RuntimeError):
        pkg.sample_rows_cmax(logits, short, rows_d, V)
