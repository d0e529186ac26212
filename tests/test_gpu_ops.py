"""Kernel-level parity: every CUDA kernel of the hot path against the CPU oracle, through the C ABI.

Integer / byte work (activation quantization, the Q8_0 GEMM's block sums, Q8_0 epilogues) must be
bit-exact. Float kernels restate the oracle's operation order where that is cheap (block-ordered
GEMM chains, double-accumulated dots, sequential prefill softmax) and are held to bit-exactness or to
a stated tolerance where the order legitimately differs (split-KV decode attention).
"""
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    import gsvcu
    c = gsvcu.Context(0)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def split_blocks(blocks, rows, K):
    """Raw Q8_0 blocks [rows][K/32][34] -> (qs int8 [rows][K], d uint16 [rows][K/32])."""
    b = np.asarray(blocks).reshape(rows, K // 32, 34)
    d = b[:, :, :2].copy().view(np.uint16).reshape(rows, K // 32)
    q = b[:, :, 2:].copy().view(np.int8).reshape(rows, K)
    return q, d


def rand_acts(rng, M, K):
    x = rng.standard_normal((M, K)).astype(np.float32)
    x *= rng.choice([1e-3, 0.3, 1.0, 40.0], size=(M, K // 32, 1)).astype(np.float32).repeat(32, axis=2).reshape(M, K)
    x[0, :32] = 0.0                      # all-zero block -> d = 0, id = 0
    if M > 1:
        x[1, 32:64] = np.arange(32) - 15.5   # exact .5 products
    return x


def test_quantize_bitexact(ctx):
    rng = np.random.default_rng(1)
    x = rand_acts(rng, 37, 2048)
    q = torch.empty((37, 2048), dtype=torch.int8, device="cuda")
    d = torch.empty((37, 64), dtype=torch.int16, device="cuda")
    ctx.op_quantize_q8_0(dev(x), q, d)
    ctx.sync()
    rq, rd = split_blocks(O.quantize_q8_0(x), 37, 2048)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), rd)


@pytest.mark.parametrize("M", [1, 8, 13, 64, 100, 257, 1000])
@pytest.mark.parametrize("NK", [(1536, 512), (512, 512), (2048, 512), (512, 2048)])
def test_q8_gemm_bitexact(ctx, M, NK):
    import gsvcu
    N, K = NK
    rng = np.random.default_rng(M * 7 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    raw = O.quantize_q8_0(W)                       # GGUF Q8_0 bytes [N][K/32][34]
    X = rand_acts(rng, M, K)
    xq, xd = split_blocks(O.quantize_q8_0(X), M, K)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    wq = torch.empty(N * K, dtype=torch.uint8, device="cuda")
    wd = torch.empty(N * K // 32, dtype=torch.int16, device="cuda")
    ctx.op_pack_q8_0(raw, N, K, wq, wd)
    Y = O.mul_mat(raw, 8, N, K, X)                 # ggml Q8_0 mul_mat semantics
    txq, txd = dev(xq), dev(xd.view(np.int16))
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ctx.op_q8_gemm(txq, txd, M, wq, wd, N, K, dev(bias), None, gsvcu.EPI_BIAS, y=y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), (Y + bias).view(np.uint32))
    ctx.op_q8_gemm(txq, txd, M, wq, wd, N, K, dev(bias), dev(resid), gsvcu.EPI_RESID, y=y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ((resid + Y) + bias).view(np.uint32))
    yq = torch.empty((M, N), dtype=torch.int8, device="cuda")
    yd = torch.empty((M, N // 32), dtype=torch.int16, device="cuda")
    ctx.op_q8_gemm(txq, txd, M, wq, wd, N, K, dev(bias), None, gsvcu.EPI_RELU_Q8, yq=yq, yd=yd)
    ctx.sync()
    rq, rd = split_blocks(O.quantize_q8_0(O.add_act(Y, bias, 1)), M, N)
    assert np.array_equal(yq.cpu().numpy(), rq)
    assert np.array_equal(yd.cpu().numpy().view(np.uint16), rd)


@pytest.mark.parametrize("M", [65, 128, 300, 1000, 4096])
@pytest.mark.parametrize("NK", [(1536, 512), (512, 512), (2048, 512), (512, 2048)])
def test_q8_gemm_tensor_cores_bitexact(ctx, M, NK):
    """The tcgen05 / TMEM / TMA prefill GEMM (gsvcu_op_q8_gemm_tc) equals the oracle's ggml Q8_0 mul_mat
    bit for bit in all three epilogues (ragged M: the tail tile's rows past M are zero-filled by TMA and
    not stored), and so equals the mma.sync kernels. The activations include blocks of +-127 everywhere,
    the largest integer sums a block can have."""
    import gsvcu
    N, K = NK
    rng = np.random.default_rng(M * 11 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[:3] = 0.02 * np.sign(rng.standard_normal((3, K)))            # rows of +-amax: all values +-127
    raw = O.quantize_q8_0(W)
    X = rand_acts(rng, M, K)
    X[: min(M, 5)] = np.sign(rng.standard_normal((min(M, 5), K))).astype(np.float32)
    xq, xd = split_blocks(O.quantize_q8_0(X), M, K)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    w16 = torch.empty(N * K, dtype=torch.float16, device="cuda")
    ctx.op_pack_q8_0_f16(raw, N, K, w16)
    wd = dev(split_blocks(raw, N, K)[1].view(np.int16))
    Y = O.mul_mat(raw, 8, N, K, X)
    txq, txd = dev(xq), dev(xd.view(np.int16))
    y = torch.full((M, N), -9.0, dtype=torch.float32, device="cuda")
    ctx.op_q8_gemm_tc(txq, txd, M, w16, wd, N, K, dev(bias), None, gsvcu.EPI_BIAS, y=y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), (Y + bias).view(np.uint32))
    ctx.op_q8_gemm_tc(txq, txd, M, w16, wd, N, K, dev(bias), dev(resid), gsvcu.EPI_RESID, y=y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ((resid + Y) + bias).view(np.uint32))
    yq = torch.empty((M, N), dtype=torch.int8, device="cuda")
    yd = torch.empty((M, N // 32), dtype=torch.int16, device="cuda")
    ctx.op_q8_gemm_tc(txq, txd, M, w16, wd, N, K, dev(bias), None, gsvcu.EPI_RELU_Q8, yq=yq, yd=yd)
    ctx.sync()
    rq, rd = split_blocks(O.quantize_q8_0(O.add_act(Y, bias, 1)), M, N)
    assert np.array_equal(yq.cpu().numpy(), rq)
    assert np.array_equal(yd.cpu().numpy().view(np.uint16), rd)


def test_layernorm_bitexact(ctx):
    rng = np.random.default_rng(3)
    rows = 300
    v = (rng.standard_normal((rows, 512)) * rng.choice([0.01, 1.0, 30.0], (rows, 1))).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(512)).astype(np.float32)
    b = (0.02 * rng.standard_normal(512)).astype(np.float32)
    y = torch.empty((rows, 512), dtype=torch.float32, device="cuda")
    yq = torch.empty((rows, 512), dtype=torch.int8, device="cuda")
    yd = torch.empty((rows, 16), dtype=torch.int16, device="cuda")
    ctx.op_layernorm_q8(dev(v), rows, dev(w), dev(b), y, yq, yd)
    ctx.sync()
    ref = O.ln_affine(v, None, None, w, b)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    rq, rd = split_blocks(O.quantize_q8_0(ref), rows, 512)
    assert np.array_equal(yq.cpu().numpy(), rq)
    assert np.array_equal(yd.cpu().numpy().view(np.uint16), rd)


@pytest.mark.parametrize("MNK", [(1, 1025, 512), (64, 1025, 512), (77, 512, 1025)])
def test_f32_gemm_double_accumulation(ctx, MNK):
    M, N, K = MNK
    rng = np.random.default_rng(M + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    add = rng.standard_normal((M, N)).astype(np.float32)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ctx.op_f32_gemm(dev(x), M, dev(w), N, K, dev(add), y)
    ctx.sync()
    ref = add + O.mul_mat(w, 0, N, K, x)
    got = y.cpu().numpy()
    # double accumulation in another order: equal after rounding to float except in rare ties
    mism = np.count_nonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert mism <= max(1, got.size // 100000), mism
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("wtype", [0, 1, 2])
@pytest.mark.parametrize("MNK", [(37, 1536, 512), (64, 512, 2048), (5, 1025, 512), (300, 2048, 512)])
def test_fx_gemm_bitexact(ctx, wtype, MNK):
    """F32 / F16 / BF16 layer matrices (exporter default / --f16 / --spec ...=bf16): equal, bit for bit, to
    the oracle's ggml FMA-vectorised dot (X rounded to F16 / BF16 for an F16 / BF16 W; 32 float chains
    folded pairwise), ragged M / N."""
    import gguf
    M, N, K = MNK
    rng = np.random.default_rng(M + N + K + wtype)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    if wtype == 2:
        wraw = gguf.quants.quantize(w, gguf.GGMLQuantizationType.BF16).view(np.int16)
    else:
        wraw = w.astype(np.float16) if wtype == 1 else w
    bias = (0.02 * rng.standard_normal(N)).astype(np.float32)
    tw = torch.from_numpy(wraw.view(np.int16) if wtype else wraw).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ref = O.mul_mat(wraw, {0: 0, 1: 1, 2: 30}[wtype], N, K, x, layer=True)
    ctx.op_fx_gemm(dev(x), M, tw, wtype, N, K, None, y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    ctx.op_fx_gemm(dev(x), M, tw, wtype, N, K, dev(bias), y)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), (ref + bias).view(np.uint32))


def paged_pool(rng, lens, n_layer, kv_dtype, npages_extra=3):
    """Random paged pool, pages permuted per sequence: (pool, block table, max_pages)."""
    PAGE, NH, HD = 64, 16, 32
    B = len(lens)
    maxp = max((l + PAGE - 1) // PAGE for l in lens) + 1
    npages = sum((l + PAGE - 1) // PAGE for l in lens) + npages_extra
    npdt = np.float16 if kv_dtype == 0 else np.float32
    pool = rng.standard_normal((npages, n_layer, 2, NH, PAGE, HD)).astype(npdt)
    perm = rng.permutation(npages)
    bt = np.zeros((B, maxp), np.int32)
    at = 0
    for b, l in enumerate(lens):
        for p in range((l + PAGE - 1) // PAGE):
            bt[b, p] = perm[at]
            at += 1
    return pool, bt, maxp


def gather_kv(pool, bt, lens, layer):
    B, Lmax = len(lens), max(lens)
    kk = np.zeros((B, Lmax, 16, 32), np.float32)
    vv = np.zeros((B, Lmax, 16, 32), np.float32)
    for b, l in enumerate(lens):
        for t in range(l):
            pg = bt[b, t // 64]
            kk[b, t] = pool[pg, layer, 0, :, t % 64, :].astype(np.float32)
            vv[b, t] = pool[pg, layer, 1, :, t % 64, :].astype(np.float32)
    return kk, vv


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_decode_attention_paged(ctx, kv_dtype):
    rng = np.random.default_rng(10 + kv_dtype)
    lens = [1, 2, 63, 64, 65, 255, 256, 257, 700, 1500, 2049, 5]
    n_layer, layer = 3, 1
    pool, bt, maxp = paged_pool(rng, lens, n_layer, kv_dtype)
    B = len(lens)
    q = rng.standard_normal((B, 1536)).astype(np.float32)   # q in the first 512 of a qkv row
    active = np.ones(B, np.int32)
    active[-1] = 0                                            # inactive slot is left untouched
    kvpos = np.array(lens, np.int32) - 1
    out_q = torch.full((B, 512), 77, dtype=torch.int8, device="cuda")
    out_d = torch.zeros((B, 16), dtype=torch.int16, device="cuda")
    out_f = torch.full((B, 512), -5.0, dtype=torch.float32, device="cuda")
    ctx.op_decode_attention(dev(q), 1536, dev(pool), kv_dtype, n_layer, layer, dev(bt), maxp, dev(kvpos), dev(active),
                            B, out_q, out_d, out_f)
    ctx.sync()
    got = out_f.cpu().numpy()
    kk, vv = gather_kv(pool, bt, lens, layer)
    ref = O.decode_attention(q[:, :512].reshape(B, 16, 32), kk, vv, np.array(lens, np.int32),
                             1.0 / np.sqrt(np.float32(32))).reshape(B, 512)
    # the same fixed float evaluation order on both sides: equal bit for bit
    mism = np.count_nonzero(got[:-1].view(np.uint32) != ref[:-1].view(np.uint32))
    assert mism == 0, (mism, np.abs(got[:-1] - ref[:-1]).max())
    assert np.all(got[-1] == -5.0) and np.all(out_q.cpu().numpy()[-1] == 77)
    rq, rd = split_blocks(O.quantize_q8_0(got[:-1]), B - 1, 512)
    assert np.array_equal(out_q.cpu().numpy()[:-1], rq)
    assert np.array_equal(out_d.cpu().numpy()[:-1].view(np.uint16), rd)


def test_prefill_attention_prefix_mask(ctx):
    rng = np.random.default_rng(5)
    shapes = [(1, 1), (5, 3), (64, 64), (100, 70), (300, 200), (513, 256), (130, 0)]
    seq_len = np.array([s for s, _ in shapes], np.int32)
    text_len = np.array([t for _, t in shapes], np.int32)
    start = np.concatenate([[0], np.cumsum(seq_len)[:-1]]).astype(np.int32)
    M = int(seq_len.sum())
    qkv = rng.standard_normal((M, 1536)).astype(np.float32)
    out_q = torch.empty((M, 512), dtype=torch.int8, device="cuda")
    out_d = torch.empty((M, 16), dtype=torch.int16, device="cuda")
    out_f = torch.empty((M, 512), dtype=torch.float32, device="cuda")
    ctx.op_prefill_attention(dev(qkv), start, seq_len, text_len, out_q, out_d, out_f)
    got = out_f.cpu().numpy()
    ref = O.prefill_attention(qkv, seq_len, text_len, 16, 32, 1.0 / np.sqrt(np.float32(32)))
    mism = np.count_nonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert mism <= 2, (mism, np.abs(got - ref).max())
    rq, rd = split_blocks(O.quantize_q8_0(got), M, 512)
    assert np.array_equal(out_q.cpu().numpy(), rq)


def test_sampler_against_reference_golden(ctx):
    """The compiled reference sampler's recorded outputs (tests/golden/sampler_golden.npz)."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "sampler_golden.npz"))
    n = len(g["token"])
    same_tok = same_state = 0
    for i in range(n):
        top_k, top_p, temp, rep = g["cfg"][i]
        prev = g["prev"][i][:g["n_prev"][i]]
        tok, st = ctx.op_sample(dev(g["logits"][i][None, :]), 1025, 1024, [20], [int(g["state0"][i])], prev=[prev],
                                top_k=int(top_k), top_p=float(top_p), temperature=float(temp), rep=float(rep))
        same_tok += int(tok[0] == g["token"][i])
        same_state += int(st[0] == g["state1"][i])
    assert same_state == n
    assert same_tok == n, f"{same_tok}/{n} tokens equal the reference sampler"


def test_sampler_random_vs_oracle(ctx):
    rng = np.random.default_rng(9)
    B, V = 64, 1025
    for trial in range(6):
        lg = (rng.standard_normal((B, V)) * [0.1, 0.45, 3.0][trial % 3]).astype(np.float32)
        steps = rng.integers(0, 30, B).astype(np.int32)          # some below 11: EOS masked
        states = rng.integers(1, 2**63, B, dtype=np.int64).astype(np.uint64)
        prev = [rng.integers(0, V, int(rng.integers(0, 5000)), dtype=np.int32) for _ in range(B)]
        cfg = [dict(top_k=15), dict(top_k=1), dict(top_k=15, top_p=0.8), dict(top_k=0, temperature=0.7),
               dict(top_k=15, rep=1.0), dict(top_k=50, top_p=0.95, temperature=1.3)][trial]
        tok, st = ctx.op_sample(dev(lg), V, 1024, steps, states, prev=prev, **cfg)
        for b in range(B):
            row = lg[b].copy()
            if steps[b] < 11:
                row[1024] = -np.inf
            probs = O.logits_to_probs(row, prev=prev[b][-4096:], top_k=cfg.get("top_k", 15),
                                      top_p=cfg.get("top_p", 1.0), temperature=cfg.get("temperature", 1.0),
                                      rep=cfg.get("rep", 1.35))
            t, s = O.sample(probs, int(states[b]))
            assert s == int(st[b])
            assert t == int(tok[b]), (trial, b)
