"""Model decode in the GPU-resident loop (RT_ROLLOUT_DECODE_MODEL).

Host-stepped (rt_rollout_profile_hook), every stage of a pass is checked on
that pass's own buffers:
  - embedding rows: bit-exact rows of the embedding table, and each slot's
    embedded token is the token it sampled the pass before (0 for a new one);
  - QKV projection: within 2^-16 * sum |a b| of a float64 product;
  - q and the new K / V page rows: the bf16 rounding of the projection;
  - attention: the CPU oracle (2e-3 absolute + 1e-2 relative);
  - LM-head input: the bf16 rounding of the attention output;
  - logits: within 2^-16 * sum |a b| of a float64 product;
  - tokens: the sampler rerun on the pass's logits and sampling rows
    (bit-exact; the sampler is pinned to the reference elsewhere).
Then the same requests through the CUDA-graph loop give the same
trajectories."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

S, HQ, HKV, V, D = 64, 32, 8, 2048, 4096
STATE_BYTES = 72 * 256 + 32


class _DevView:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def dev(ptr, shape, typestr):
    return torch.as_tensor(_DevView(ptr, shape, typestr), device="cuda").clone()


def bf16_bits(t):
    return t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)


def within_bound(got, a, b):
    a64, b64 = a.double(), b.double()
    ref = a64 @ b64.T
    bound = (a64.abs() @ b64.abs().T) * 2.0 ** -16 + 1e-6
    return bool(((got.double() - ref).abs() <= bound).all())


def make_requests(orc, n, seed):
    rng = np.random.default_rng(seed)
    r = np.zeros(n, dtype=orc.REQUEST_DTYPE)
    pfx = rng.integers(0, 3, n)  # 0 = no prefix, 1..2 = prefix id + 1
    r["request_id"] = np.arange(1, n + 1, dtype=np.uint64) | (pfx.astype(np.uint64) << np.uint64(32))
    r["max_tokens"] = rng.integers(3, 13, n)
    r["kv_blocks"] = 4
    r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 77
    return r


def build(pkg, cuda, max_context=512):
    cfg = dict(num_q_heads=HQ, num_kv_heads=HKV, vocab=V, max_slots=S, max_context=max_context,
               max_new_tokens=16, max_admit=256, drop_when_full=0,
               decode_mode=pkg.RT_ROLLOUT_DECODE_MODEL, reward_mode=0, logit_std=2.0,
               max_prefixes=4, max_prefix_pages=512, max_passes=1 << 20, idle_timeout_ms=2000)
    arena = pkg.DeviceArena(1024)
    eng = pkg.RolloutEngine(cfg, arena)
    for pid, L in enumerate([40, 64]):
        pages = arena.acquire((L + 15) // 16)
        arena.fill_pages(pages, seed=5, stream_id=100 * pid)
        eng.set_prefix(pid, pages, L)
    g = torch.Generator(device=cuda).manual_seed(11)
    emb = torch.randn(V, D, generator=g, device=cuda).to(torch.bfloat16)
    wqkv = (torch.randn((HQ + 2 * HKV) * 128, D, generator=g, device=cuda) / 64).to(torch.bfloat16)
    wlm = (torch.randn(V, D, generator=g, device=cuda) * 0.05).to(torch.bfloat16)
    return eng, arena, emb, wqkv, wlm


def test_launch_needs_weights(pkg, orc, cuda):
    eng, arena, emb, wqkv, wlm = build(pkg, cuda)
    reqs = make_requests(orc, 4, 1)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    with pytest.raises(pkg.RuntimeErrorRT, match="set_model"):
        eng.launch(requests=req_d, n_requests=4, state=state)
    with pytest.raises(pkg.RuntimeErrorRT, match="d_model"):
        eng.set_model(emb[:, :2048].contiguous(), wqkv[:, :2048].contiguous(),
                      wlm[:, :2048].contiguous())
    eng.close()


def test_model_decode_pass_by_pass(pkg, orc, cuda):
    eng, arena, emb, wqkv, wlm = build(pkg, cuda)
    eng.set_model(emb, wqkv, wlm)
    n = 40
    reqs = make_requests(orc, n, 2)
    req_d = torch.from_numpy(reqs.view(np.uint8).copy()).to(cuda)
    state = torch.zeros(STATE_BYTES, dtype=torch.uint8, device=cuda)
    traj = torch.zeros(n, 16, dtype=torch.int32, device=cuda)
    prev = {}
    deep = []

    def hook(p):
        b = eng.buffers()
        en = dev(b.enable, (S,), "<u4").cpu().numpy() == 1
        lens = dev(b.seq_lens, (S,), "<i4").cpu().numpy()
        tok = dev(b.tokens, (S,), "<u4").cpu().numpy()
        et = dev(b.embed_tokens, (S,), "<u4").cpu().numpy()
        assert en.any()
        for s in np.nonzero(en)[0]:
            # a continuing slot embeds what it sampled last pass; a new one token 0
            assert et[s] == 0 or (s in prev and et[s] == prev[s]), (p, s, et[s], prev.get(s))
        prev.clear()
        prev.update({int(s): int(tok[s]) for s in np.nonzero(en)[0]})
        if p not in (0, 1, 4, 9):
            return False
        act = torch.from_numpy(np.nonzero(en)[0]).cuda()
        hin = dev(b.hidden_in, (S, D), "<i2").view(torch.bfloat16)
        assert torch.equal(hin[act], emb[torch.from_numpy(et).cuda().long()[act]])
        qkv = dev(b.qkv, (S, (HQ + 2 * HKV) * 128), "<f4")
        assert within_bound(qkv[act], hin[act], wqkv)
        q = dev(b.q, (S, HQ * 128), "<i2").view(torch.bfloat16)
        assert torch.equal(q[act], qkv[act, :HQ * 128].to(torch.bfloat16))
        pt = dev(b.page_table, (S, b.max_pages), "<i4").cpu().numpy()
        kv = arena.buf.view(torch.int16).cpu().numpy().view(np.uint16)
        kvp = kv.reshape(-1, HKV, 2, 16, 128)
        qkv_bits = bf16_bits(qkv)
        for s in np.nonzero(en)[0]:
            pos = lens[s] - 1
            page, row = pt[s, pos // 16], pos % 16
            for h in range(HKV):
                for plane in range(2):
                    off = HQ * 128 + plane * HKV * 128 + h * 128
                    assert np.array_equal(kvp[page, h, plane, row], qkv_bits[s, off:off + 128])
        out = dev(b.attn_out, (S, HQ, 128), "<f4").cpu().numpy()
        ref = orc.paged_gqa_attention(q.view(torch.int16).cpu().numpy().view(np.uint16)
                                      .reshape(S, HQ, 128), kv, np.where(en[:, None], pt, 0),
                                      np.where(en, lens, 0), HQ, HKV, 128 ** -0.5)
        err = np.abs(out - ref)[en]
        assert (err <= 2e-3 + 1e-2 * np.abs(ref[en])).all(), err.max()
        hout = dev(b.hidden_out, (S, D), "<i2").view(torch.bfloat16)
        assert torch.equal(hout[act], torch.from_numpy(out).cuda()[act].reshape(-1, D)
                           .to(torch.bfloat16))
        logits = dev(b.logits, (S, V), "<f4")
        assert within_bound(logits[act], hout[act], wlm)
        rows = dev(b.sample_rows, (S * pkg.SAMPLE_ROW_BYTES,), "|u1")
        again = pkg.sample_rows(logits, rows, V)
        assert np.array_equal(again.cpu().numpy()[en], tok[en].astype(np.int32))
        deep.append(p)
        return False

    eng.step(hook, requests=req_d, n_requests=n, state=state, trajectories=traj, n_rows=n)
    assert deep == [0, 1, 4, 9]
    st = eng.wait()
    assert st["error"] == 0 and st["attn_error"] == 0 and st["model_error"] == 0

    # the CUDA-graph loop: same kernels, same data, same trajectories
    traj2 = torch.zeros_like(traj)
    state2 = torch.zeros_like(state)
    eng.launch(requests=req_d, n_requests=n, state=state2, trajectories=traj2, n_rows=n)
    st2 = eng.wait()
    assert st2["error"] == 0 and st2["model_error"] == 0 and st2["done"] == n
    assert torch.equal(traj, traj2)
    lens = reqs["max_tokens"]
    t = traj2.cpu().numpy()
    assert all((t[i, :lens[i]] >= 0).all() and (t[i, :lens[i]] < V).all() for i in range(n))
    eng.close()


def test_prefill_writes_prompt_kv(pkg, orc, cuda):
    """rt_rollout_prefill: every position of a 4,100-token prompt (two
    4,096-token projection chunks) gets bf16(embed[token] . w_kv^T) in its
    prefix page; an out-of-range token id is flagged."""
    eng, arena, emb, wqkv, wlm = build(pkg, cuda, max_context=4352)
    eng.set_model(emb, wqkv, wlm)
    L = 4100
    pages = arena.acquire((L + 15) // 16)
    eng.set_prefix(2, pages, L)
    g = torch.Generator(device=cuda).manual_seed(5)
    toks = torch.randint(0, V, (L,), generator=g, device=cuda, dtype=torch.int32)
    eng.prefill(2, toks)
    torch.cuda.synchronize()
    x = emb[toks.long()]
    wkv = wqkv[HQ * 128:]
    ref = x.double() @ wkv.double().T                     # [L][k heads | v heads]
    bound = (x.double().abs() @ wkv.double().abs().T) * 2.0 ** -16 + ref.abs() * 2.0 ** -8
    kvp = arena.buf.view(torch.bfloat16).view(-1, HKV, 2, 16, 128)
    pg = torch.as_tensor(np.asarray(pages)[np.arange(L) // 16], device=cuda).long()
    row = torch.arange(L, device=cuda) % 16
    got = kvp[pg, :, :, row, :]                            # [L][HKV][2][128]
    want = ref.view(L, 2, HKV, 128).permute(0, 2, 1, 3)
    bnd = bound.view(L, 2, HKV, 128).permute(0, 2, 1, 3)
    assert bool(((got.double() - want).abs() <= bnd).all())
    st = eng.wait()
    assert st["model_error"] == 0
    bad = toks.clone()
    bad[7] = V + 3
    eng.prefill(2, bad)
    st = eng.wait(check_errors=False)
    assert st["model_error"] == pkg.RT_EDEVICE
    with pytest.raises(pkg.RuntimeErrorRT, match="registered"):
        eng.prefill(2, toks[:100])
    eng.close()
