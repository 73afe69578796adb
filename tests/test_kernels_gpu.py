"""sm_100a kernels vs plain PyTorch fp32 references of the same ops.
Shapes include odd tails, 1-token contexts and page-boundary contexts."""

import math

import numpy as np
import pytest
import torch

from swiftllm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from swiftllm_b200.ops import cuda_ext
    return cuda_ext()


def _status_ok(C):
    st = C.read_status(True)
    assert st[0] == 0, f"device status word set: {st}"


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("T,H", [(1, 256), (7, 4096), (33, 8192), (128, 5120), (5, 2560)])
def test_rms_norm(C, T, H):
    x, w = bf(T, H), bf(H)
    out = torch.empty_like(x)
    C.rms_norm(out, x, w, 1e-5)
    r, _ = ref.rms_norm(x.float(), w.float(), 1e-5)
    torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=2e-2)
    res = bf(T, H)
    res0 = res.clone()
    out2 = torch.empty_like(x)
    C.fused_add_rms_norm(out2, x, res, w, 1e-5)
    r2, nr = ref.rms_norm(x, w, 1e-5, res0)
    torch.testing.assert_close(res.float(), nr.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(out2.float(), r2.float(), rtol=2e-2, atol=3e-2)
    _status_ok(C)


def test_layer_norm(C):
    x, w, b = bf(9, 2560), bf(2560), bf(2560)
    out = torch.empty_like(x)
    C.layer_norm(out, x, w, b, 1e-5)
    r, _ = ref.layer_norm(x.float(), w.float(), b.float(), 1e-5)
    torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=3e-2)


def test_silu_gelu_embedding(C):
    x = bf(37, 2 * 688)
    out = torch.empty(37, 688, dtype=torch.bfloat16, device="cuda")
    C.silu_and_mul(out, x)
    torch.testing.assert_close(out.float(), ref.silu_and_mul(x.float()), rtol=2e-2, atol=2e-2)
    g = torch.empty_like(x)
    C.gelu_tanh(g, x)
    torch.testing.assert_close(g.float(), ref.gelu_tanh(x.float()), rtol=2e-2, atol=2e-2)
    w = bf(1000, 256)
    ids = torch.tensor([0, 5, 999, 1000, 3], dtype=torch.int32, device="cuda")
    e = torch.empty(5, 256, dtype=torch.bfloat16, device="cuda")
    C.embedding(e, ids, w, 0)
    assert torch.equal(e[:3], w[[0, 5, 999]]) and e[3].abs().sum() == 0
    e2 = torch.empty_like(e)
    C.embedding(e2, ids, w[500:].contiguous(), 500)
    assert torch.equal(e2[2], w[999]) and e2[0].abs().sum() == 0


@pytest.mark.parametrize("Hq,Hkv,D,rot,bias", [(4, 2, 64, 64, False), (32, 8, 128, 128, True),
                                                (8, 8, 80, 32, True)])
def test_qkv_rope_cache(C, Hq, Hkv, D, rot, bias):
    from swiftllm_b200.models.rope import cos_sin_table
    T, L, bs, nb = 37, 3, 16, 8
    qkv = bf(T, (Hq + 2 * Hkv) * D)
    b = bf((Hq + 2 * Hkv) * D) if bias else None
    pos = torch.randint(0, 500, (T,), dtype=torch.int32, device="cuda")
    slots = torch.randperm(nb * bs, device="cuda")[:T].to(torch.int32)
    slots[3] = -1
    cs = cos_sin_table(rot, 10000.0, 512, device="cuda")
    kv = torch.zeros(nb, L, 2, Hkv, bs, D, dtype=torch.bfloat16, device="cuda")
    kv_ref = kv.clone()
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device="cuda")
    C.qkv_rope_cache(q, qkv, pos, cs, kv, 1, slots, Hq, Hkv, D, rot, b)
    x = qkv.float() + (b.float() if b is not None else 0)
    qr = ref.apply_rope(x[:, :Hq * D].view(T, Hq, D), pos, cs, rot)
    kr = ref.apply_rope(x[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D), pos, cs, rot)
    vr = x[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    ref.write_kv(kv_ref[:, 1, 0], kv_ref[:, 1, 1], kr, vr, slots)
    torch.testing.assert_close(q.float(), qr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kv.float(), kv_ref.float(), rtol=2e-2, atol=2e-2)
    _status_ok(C)


def _paged_setup(lens, q_lens, Hq, Hkv, D, bs=16, L=2):
    S = len(lens)
    nbs = [(l + bs - 1) // bs for l in lens]
    total = sum(nbs) + 3
    kv = bf(total, L, 2, Hkv, bs, D)
    perm = torch.randperm(total, device="cuda").to(torch.int32)
    mb = max(max(nbs), 1)
    bt = torch.zeros((S, mb + 2), dtype=torch.int32, device="cuda")
    o = 0
    for i, n in enumerate(nbs):
        bt[i, :n] = perm[o:o + n]
        o += n
    q_start = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32, device="cuda")
    q = bf(int(sum(q_lens)), Hq, D)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return kv, bt, q_start, q, sl


def _ref_attn(q, kv, bt, q_start, sl, scale, window=None):
    return ref.paged_attention(q.float().cpu(), kv[:, 1, 0].float().cpu(), kv[:, 1, 1].float().cpu(),
                               bt.cpu(), q_start.cpu(), sl.cpu(), scale, sliding_window=window)


@pytest.mark.parametrize("Hq,Hkv,D,bs", [(32, 32, 128, 16), (32, 8, 128, 16), (8, 1, 128, 16),
                                         (4, 2, 64, 16), (32, 32, 80, 16), (8, 8, 128, 32)])
@pytest.mark.parametrize("splits", [1, 3])
def test_paged_decode(C, Hq, Hkv, D, bs, splits):
    lens = [1, 15, 16, 17, 200, 1000, 0, 33]
    kv, bt, q_start, q, sl = _paged_setup(lens, [1] * len(lens), Hq, Hkv, D, bs)
    rows = len(lens)
    ws = torch.empty(rows * Hq * splits * (D + 2), dtype=torch.float32, device="cuda")
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    C.paged_decode(out, q, kv, 1, bt, sl, rows, splits, scale, 0, ws)
    r = _ref_attn(q, kv, bt, q_start, sl, scale)
    for i, l in enumerate(lens):
        if l == 0:
            assert out[i].float().abs().max() == 0
            continue
        torch.testing.assert_close(out[i].float().cpu(), r[i], rtol=2e-2, atol=2e-2)
    _status_ok(C)


def test_paged_decode_window(C):
    lens = [100, 300, 17]
    kv, bt, q_start, q, sl = _paged_setup(lens, [1] * 3, 8, 2, 128)
    ws = torch.empty(3 * 8 * 2 * 130, dtype=torch.float32, device="cuda")
    out = torch.empty_like(q)
    C.paged_decode(out, q, kv, 1, bt, sl, 3, 2, 0.088, 64, ws)
    r = _ref_attn(q, kv, bt, q_start, sl, 0.088, 64)
    torch.testing.assert_close(out.float().cpu(), r, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("impl", [0, -1])
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 32, 128), (32, 8, 128), (64, 8, 128), (8, 2, 128),
                                      (4, 2, 64), (8, 8, 80)])
def test_paged_prefill(C, Hq, Hkv, D, impl):
    # (seq_len, q_len): full prompts, chunked prefill with cached prefix, odd
    # tails, and prompts spanning several 128-key tiles. impl -1 runs the
    # tcgen05 kernel for head_dim 128, 0 the mma.sync kernel.
    pairs = [(64, 64), (130, 130), (300, 45), (17, 17), (1, 1), (200, 129), (700, 700), (600, 300)]
    lens = [p[0] for p in pairs]
    ql = [p[1] for p in pairs]
    kv, bt, q_start, q, sl = _paged_setup(lens, ql, Hq, Hkv, D)
    scale = 1 / math.sqrt(D)
    out = torch.zeros_like(q)
    C.paged_prefill(out, q, kv, 1, bt, q_start, sl, 0, len(lens), max(ql), scale, 0, impl)
    torch.testing.assert_close(out.float().cpu(), _ref_attn(q, kv, bt, q_start, sl, scale),
                               rtol=2e-2, atol=2e-2)
    out2 = torch.zeros_like(q)
    C.paged_prefill(out2, q, kv, 1, bt, q_start, sl, 0, len(lens), max(ql), scale, 50, impl)
    torch.testing.assert_close(out2.float().cpu(), _ref_attn(q, kv, bt, q_start, sl, scale, 50),
                               rtol=2e-2, atol=2e-2)
    _status_ok(C)


def test_paged_prefill_tc_large_logits(C):
    # logits that grow by far more than 2^8 across key tiles: the tcgen05
    # kernel must rescale its running output and still match
    lens, ql = [500, 257], [500, 100]
    kv, bt, q_start, q, sl = _paged_setup(lens, ql, 16, 4, 128)
    q = (q.float() * 6.0).to(torch.bfloat16)
    scale = 1 / math.sqrt(128)
    out = torch.zeros_like(q)
    C.paged_prefill(out, q, kv, 1, bt, q_start, sl, 0, 2, max(ql), scale, 0, 1)
    torch.testing.assert_close(out.float().cpu(), _ref_attn(q, kv, bt, q_start, sl, scale),
                               rtol=3e-2, atol=3e-2)
    _status_ok(C)


@pytest.mark.parametrize("T,N,K", [(1, 4096, 4096), (7, 12288, 4096), (16, 128, 64),
                                   (33, 4096, 11008), (256, 4096, 4096), (256, 22016, 4096),
                                   (1000, 4096, 4096), (4096, 1024, 512), (77, 32000, 4096),
                                   (300, 640, 200)])
def test_gemm(C, T, N, K):
    x = bf(T, K, scale=0.5)
    w = bf(N, K, scale=0.05)
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    C.gemm(out, x, w, None)
    r = x.float() @ w.float().t()
    torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=2e-2 * math.sqrt(K / 64) * 0.5)
    _status_ok(C)


@pytest.mark.parametrize("mt,minper", [(1, 8), (2, 8), (1, 1), (2, 3)])
@pytest.mark.parametrize("T,N,K", [(5, 640, 200), (100, 4096, 4096), (256, 12288, 4096),
                                   (64, 384, 11008), (200, 32000, 1024), (600, 1000, 640),
                                   (1000, 2048, 1024)])
def test_gemm_streamk(C, mt, minper, T, N, K):
    # stream-K decode path: forced unit height and tiny per-CTA ranges so
    # tiles are split across many CTAs (partials + last-arriver fix-up)
    C.gemm_streamk_config(2, mt, minper)
    try:
        _check_streamk(C, mt, T, N, K)
    finally:
        C.gemm_streamk_config(1, 1, 32)


def _check_streamk(C, mt, T, N, K):
    plan = C.gemm_plan(N, T, K)
    assert plan[2] == mt
    x, w, b = bf(T, K, scale=0.5), bf(N, K, scale=0.05), bf(N)
    big = torch.zeros(T, N + 64, dtype=torch.bfloat16, device="cuda")
    out = big[:, 32:32 + N]
    for _ in range(2):  # second launch reuses the self-resetting tile counters
        C.gemm(out, x, w, b)
        r = x.float() @ w.float().t() + b.float()
        torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=2e-2 * math.sqrt(K / 64) * 0.5)
    assert big[:, :32].abs().sum() == 0 and big[:, 32 + N:].abs().sum() == 0
    _status_ok(C)


def test_gemm_bias_and_strided_out(C):
    x, w, b = bf(40, 512), bf(384, 512, scale=0.05), bf(384)
    big = torch.zeros(40, 1024, dtype=torch.bfloat16, device="cuda")
    out = big[:, 128:512]
    C.gemm(out, x, w, b)
    r = x.float() @ w.float().t() + b.float()
    torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=5e-2)
    assert big[:, :128].abs().sum() == 0 and big[:, 512:].abs().sum() == 0


def test_sample_greedy_and_seeded(C):
    from swiftllm_b200 import _core
    from swiftllm_b200.parallel.dummy_init import mix_key
    n, V = 64, 32000
    logits = torch.randn(n, V, device="cuda") * 3
    idx = np.arange(n)
    temp = np.where(idx % 4 == 0, 0.0, 0.8).astype(np.float32)
    top_p = np.where(idx % 3 == 0, 0.9, 1.0).astype(np.float32)
    top_k = np.where(idx % 5 == 0, 50, -1).astype(np.int32)
    min_p = np.where(idx % 7 == 0, 0.05, 0.0).astype(np.float32)
    key = mix_key(1234, 0x5EED)
    c0 = np.arange(n, dtype=np.uint32)
    f = torch.from_numpy(np.stack([temp, top_p, min_p])).cuda()
    i = torch.from_numpy(np.stack([idx.astype(np.int32), top_k, c0.view(np.int32),
                                   np.zeros(n, np.int32)])).cuda()
    keys = torch.full((n,), int(np.uint64(key).view(np.int64)), dtype=torch.int64, device="cuda")
    toks = torch.empty(n, dtype=torch.int32, device="cuda")
    lps = torch.empty(n, dtype=torch.float32, device="cuda")
    C.sample(toks, lps, logits, f, i, keys, True)
    toks, lps = toks.cpu().numpy(), lps.cpu().numpy()
    lg = logits.cpu().numpy()
    mism = 0
    for r in range(n):
        u = _core.philox_uniform(key, int(c0[r]), 0)
        p = _core.SampleParams(temperature=float(temp[r]), top_p=float(top_p[r]),
                               top_k=int(top_k[r]), min_p=float(min_p[r]))
        t, lp = _core.sample_row(lg[r], p, u)
        if t != toks[r]:
            mism += 1
        else:
            assert abs(lp - lps[r]) < 1e-3
        if temp[r] == 0:
            assert toks[r] == int(np.argmax(lg[r]))
    assert mism <= 2, f"{mism} of {n} draws differ from the CPU oracle"


def test_copy_blocks_and_init(C):
    kv = bf(10, 2, 2, 2, 16, 64)
    ref_kv = kv.clone()
    pairs = torch.tensor([[1, 5], [3, 7]], dtype=torch.int32, device="cuda")
    C.copy_blocks(kv, pairs)
    ref_kv[5] = ref_kv[1]
    ref_kv[7] = ref_kv[3]
    assert torch.equal(kv, ref_kv)
    from swiftllm_b200.parallel.dummy_init import fill_normal_sharded
    g = torch.empty(64, 96, dtype=torch.float32, device="cuda")
    c = torch.empty(64, 96, dtype=torch.float32)
    fill_normal_sharded(g, None, 0, 7, 0.02)
    fill_normal_sharded(c, None, 0, 7, 0.02)
    torch.testing.assert_close(g.cpu(), c, rtol=1e-4, atol=1e-6)
    assert abs(float(g.std()) - 0.02) < 0.003


def test_peer_wait_times_out_cleanly(C):
    # a flag nobody sets: the bounded wait must give up, record the status
    # and leave the context usable
    C.read_status(True)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.flag_wait_probe(flag, 1, 0.05)
    torch.cuda.synchronize()
    st = C.read_status(True)
    assert st[0] == 2 and st[1] == 299
    x = bf(4, 256)
    out = torch.empty_like(x)
    C.rms_norm(out, x, bf(256), 1e-5)
    torch.cuda.synchronize()


def test_moe_route_permute_grouped_gemm_combine(C):
    from swiftllm_b200.ops import reference as R
    T, E, k, H, I = 37, 8, 2, 256, 192
    logits = torch.randn(T, E, device="cuda")
    w = torch.empty(T, k, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    C.moe_route(logits, k, True, w, ids)
    rw, rid = R.moe_topk_softmax(logits.cpu(), k)
    assert torch.equal(ids.cpu(), rid) and torch.allclose(w.cpu(), rw, atol=1e-5)
    for e0, El in ((0, 8), (4, 4)):
        off = torch.empty(El + 1, dtype=torch.int32, device="cuda")
        perm = torch.empty(T * k, dtype=torch.int32, device="cuda")
        inv = torch.empty(T * k, dtype=torch.int32, device="cuda")
        C.moe_permute(ids, e0, El, off, perm, inv)
        x = bf(T, H)
        w13 = bf(El, 2 * I, H, scale=0.05)
        w2 = bf(El, H, I, scale=0.05)
        xg = torch.empty(T * k, H, dtype=torch.bfloat16, device="cuda")
        C.moe_gather(xg, x, perm)
        assert torch.equal(xg, x.index_select(0, perm))
        h = torch.empty(T * k, 2 * I, dtype=torch.bfloat16, device="cuda")
        C.gemm_grouped(h, xg, w13, off, T * k // E)
        a = torch.empty(T * k, I, dtype=torch.bfloat16, device="cuda")
        C.silu_and_mul(a, h)
        y = torch.empty(T * k, H, dtype=torch.bfloat16, device="cuda")
        C.gemm_grouped(y, a, w2, off, T * k // E)
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        C.moe_combine(out, y, w, inv)
        ref = torch.zeros(T, H)
        for le in range(El):
            rows, slot = (ids.cpu() == e0 + le).nonzero(as_tuple=True)
            if rows.numel() == 0:
                continue
            hh = R.silu_and_mul(x.float().cpu()[rows] @ w13[le].float().cpu().t())
            ref.index_add_(0, rows, (hh @ w2[le].float().cpu().t()) * w.cpu()[rows, slot].unsqueeze(1))
        torch.testing.assert_close(out.float().cpu(), ref, rtol=3e-2, atol=3e-2)
    _status_ok(C)


@pytest.mark.parametrize("T,k,E,e0,El", [(1, 2, 8, 0, 8), (3000, 2, 8, 2, 3), (517, 8, 64, 5, 40)])
def test_moe_permute_order(C, T, k, E, e0, El):
    # expert-contiguous rows, (token, slot) order inside an expert, against
    # a plain-Python stable ordering; chunks of 1024 pairs cross warps
    g = torch.Generator().manual_seed(T)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    off = torch.empty(El + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(T * k, dtype=torch.int32, device="cuda")
    inv = torch.empty(T * k, dtype=torch.int32, device="cuda")
    C.moe_permute(ids.cuda(), e0, El, off, perm, inv)
    flat = ids.view(-1).tolist()
    want_perm, want_inv, want_off = [], [-1] * (T * k), [0]
    for e in range(e0, e0 + El):
        for i, v in enumerate(flat):
            if v == e:
                want_inv[i] = len(want_perm)
                want_perm.append(i // k)
        want_off.append(len(want_perm))
    n = len(want_perm)
    assert off.cpu().tolist() == want_off
    assert perm.cpu()[:n].tolist() == want_perm and perm.cpu()[n:].eq(0).all()
    assert inv.cpu().tolist() == want_inv
    _status_ok(C)


@pytest.mark.parametrize("T,N,K", [(1, 4096, 4096), (37, 640, 256), (256, 12288, 4096),
                                   (700, 4096, 11008)])
def test_gemm_e4m3(C, T, N, K):
    from swiftllm_b200 import ops
    x = bf(T, K, scale=0.5)
    w = bf(N, K, scale=0.05)
    xq, xs = ops.quantize_e4m3(x)
    wq, wsc = ops.quantize_e4m3(w)
    # quantiser matches torch's E4M3 conversion of the same scaled values
    xs_ref = (x.float().abs().amax(-1) / 448).clamp_min(1e-12)
    torch.testing.assert_close(xs, xs_ref, rtol=1e-6, atol=0)
    q_ref = (x.float() / xs_ref[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    # x * (1/s) vs x / s can round differently right at a rounding boundary
    assert (xq != q_ref).float().mean().item() < 1e-2
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    C.gemm_e4m3(out, xq, xs, wq, wsc, None)
    xd = xq.view(torch.float8_e4m3fn).float() * xs[:, None]
    wd = wq.view(torch.float8_e4m3fn).float() * wsc[:, None]
    r = xd @ wd.t()
    torch.testing.assert_close(out.float(), r, rtol=2e-2, atol=2e-2 * math.sqrt(K / 64) * 0.5)
    _status_ok(C)


def test_fp8_model_gpu():
    from swiftllm_b200 import LLM, SamplingParams
    sp = SamplingParams(temperature=0, max_tokens=16, ignore_eos=True)
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12] * 4, list(range(100, 164))]
    llm = LLM("tiny-llama", load_format="dummy", dtype="bfloat16", gpu_memory_utilization=0.3,
              max_model_len=256, quantization="fp8")
    out = llm.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    assert all(len(o.outputs[0].token_ids) == 16 for o in out)
    llm.shutdown()


def test_linear_odd_k():
    # K not a multiple of 8 (16-byte TMA rows): ops.linear zero-pads
    from swiftllm_b200 import ops
    x, w = bf(19, 172, scale=0.5), bf(96, 172, scale=0.05)
    y = ops.linear(x, w)
    torch.testing.assert_close(y.float(), x.float() @ w.float().t(), rtol=2e-2, atol=2e-2)


def test_apply_penalties_kernel(C):
    # the batched penalty kernel against the same table applied in PyTorch
    import sys, os
    sys.path.insert(0, os.path.dirname(__file__))
    from test_penalties_cpu import _case, apply_csr
    from swiftllm_b200.sampling.batch import BatchSampler
    logits, hist, rep, pres, freq = _case(seed=3)
    n = logits.shape[0]
    offs, tk, ct = BatchSampler.penalty_csr(n, rep, pres, freq, lambda r: hist[r])
    want = apply_csr(logits, offs, tk, ct, rep, pres, freq)
    dev = torch.from_numpy(logits).cuda()
    C.apply_penalties(dev, torch.from_numpy(offs).cuda(), torch.from_numpy(tk).cuda(),
                      torch.from_numpy(ct).cuda(), torch.from_numpy(np.concatenate([rep, pres, freq])).cuda())
    torch.testing.assert_close(dev.cpu(), want, rtol=1e-6, atol=1e-6)


def test_index_guards_record_and_skip(C):
    # out-of-pool slots and block ids are never written: the kernels record
    # kErrBadIndex (3) in the status word and skip the access
    from swiftllm_b200.models.rope import cos_sin_table
    C.read_status(True)
    Hq, Hkv, D, bs, nb = 4, 2, 64, 16, 4
    qkv = bf(3, (Hq + 2 * Hkv) * D)
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    slots = torch.tensor([0, nb * bs + 5, 1], dtype=torch.int32, device="cuda")
    cs = cos_sin_table(D, 10000.0, 16, device="cuda")
    kv = torch.zeros(nb, 1, 2, Hkv, bs, D, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(3, Hq, D, dtype=torch.bfloat16, device="cuda")
    C.qkv_rope_cache(q, qkv, pos, cs, kv, 0, slots, Hq, Hkv, D, D, None)
    torch.cuda.synchronize()
    st = C.read_status(True)
    assert st[0] == 3 and st[1] == 101, st
    assert kv[:, :, :, :, 2:].abs().sum() == 0  # only slots 0 and 1 written
    kv2 = bf(6, 1, 2, 2, 16, 64)
    before = kv2.clone()
    C.copy_blocks(kv2, torch.tensor([[1, 6], [9, 2]], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    st = C.read_status(True)
    assert st[0] == 3 and st[1] == 110, st
    assert torch.equal(kv2, before)


@pytest.mark.parametrize("T,N,K", [(1, 4096, 4096), (37, 640, 256), (256, 12288, 4096),
                                   (700, 4096, 11008)])
def test_gemm_s8(C, T, N, K):
    # W8A8 on tcgen05 kind::i8: int32 accumulation is exact, so the result
    # matches the dequantised fp32 product up to the bf16 output rounding
    from swiftllm_b200 import ops
    x = bf(T, K, scale=0.5)
    w = bf(N, K, scale=0.05)
    xq, xs = ops.quantize_s8(x)
    wq, wsc = ops.quantize_s8(w)
    xs_ref = (x.float().abs().amax(-1) / 127).clamp_min(1e-12)
    torch.testing.assert_close(xs, xs_ref, rtol=1e-6, atol=0)
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    C.gemm_s8(out, xq, xs, wq, wsc, None)
    r = (xq.float() @ wq.float().t()) * xs[:, None] * wsc[None, :]
    torch.testing.assert_close(out.float(), r, rtol=1e-2, atol=1e-2)
    _status_ok(C)


def test_int8_model_gpu():
    from swiftllm_b200 import LLM, SamplingParams
    sp = SamplingParams(temperature=0, max_tokens=16, ignore_eos=True)
    llm = LLM("tiny-llama", load_format="dummy", dtype="bfloat16", gpu_memory_utilization=0.3,
              max_model_len=256, quantization="int8")
    out = llm.generate(prompt_token_ids=[list(range(100, 164))], sampling_params=sp, use_tqdm=False)
    assert len(out[0].outputs[0].token_ids) == 16
    llm.shutdown()


@pytest.mark.parametrize("Hq,Hkv,D", [(8, 8, 128), (8, 2, 128), (12, 4, 64)])
def test_alibi_decode_and_prefill(C, Hq, Hkv, D):
    # ALiBi: slope(head) * (key position - query position) added to every
    # score, in the decode kernel (split and unsplit) and the prefill kernel
    slopes = ref.alibi_slopes(Hq).float().cuda()
    lens = [37, 300, 1, 129]
    kv, bt, q_start, q, sl = _paged_setup(lens, [1] * len(lens), Hq, Hkv, D)
    scale = 1 / math.sqrt(D)
    r = ref.paged_attention(q.float().cpu(), kv[:, 1, 0].float().cpu(), kv[:, 1, 1].float().cpu(),
                            bt.cpu(), q_start.cpu(), sl.cpu(), scale, alibi_slopes=slopes.cpu())
    for splits in (1, 3):
        ws = torch.empty(len(lens) * Hq * splits * (D + 2), dtype=torch.float32, device="cuda")
        out = torch.empty_like(q)
        C.paged_decode(out, q, kv, 1, bt, sl, len(lens), splits, scale, 0, ws, slopes)
        torch.testing.assert_close(out.float().cpu(), r, rtol=2e-2, atol=2e-2)
    pairs = [(64, 64), (300, 45), (17, 17), (200, 129)]
    kv, bt, q_start, q, sl = _paged_setup([p[0] for p in pairs], [p[1] for p in pairs], Hq, Hkv, D)
    out = torch.zeros_like(q)
    C.paged_prefill(out, q, kv, 1, bt, q_start, sl, 0, len(pairs), 129, scale, 0, -1, slopes)
    r = ref.paged_attention(q.float().cpu(), kv[:, 1, 0].float().cpu(), kv[:, 1, 1].float().cpu(),
                            bt.cpu(), q_start.cpu(), sl.cpu(), scale, alibi_slopes=slopes.cpu())
    torch.testing.assert_close(out.float().cpu(), r, rtol=2e-2, atol=2e-2)
    _status_ok(C)


def test_spec_verify_greedy(C):
    # arg-max (lowest index on ties), accept flag and log-probabilities of
    # the draft and arg-max tokens against torch on the same rows
    V, R = 32003, 9
    logits = torch.randn(R, V, device="cuda") * 3
    logits[2, 100] = logits[2, 7] = 50.0  # tie: index 7 wins
    pos = torch.tensor([0, 2, 2, 5, 8, 8], dtype=torch.int64, device="cuda")
    am = logits.argmax(-1)
    draft = torch.stack([am[0], torch.tensor(100, device="cuda"), am[2], am[5] + 1,
                         am[8], torch.tensor(3, device="cuda")]).to(torch.int64)
    temp = torch.tensor([1.0, 1.0, 0.7, 1.0, 2.0, 1.0], device="cuda")
    out = torch.empty(4, 6, device="cuda")
    C.spec_verify_greedy(logits, pos, draft, temp, out)
    x = logits.index_select(0, pos) / temp[:, None]
    lsm = torch.log_softmax(x, -1)
    ref_am = x.argmax(-1)
    assert out[1].long().tolist() == ref_am.tolist() and ref_am[1].item() == 7
    assert (out[0] > 0.5).tolist() == (ref_am == draft).tolist()
    torch.testing.assert_close(out[2], lsm.gather(1, draft[:, None]).view(-1), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(out[3], lsm.gather(1, ref_am[:, None]).view(-1), rtol=1e-4, atol=1e-4)
    _status_ok(C)
