"""The oracle pinned: golden vectors of the reference's own code, and an independent float64 model.

* sampler: bit-exact against the compiled reference src/gsv_sampler.cpp (committed golden fixture,
  and live when oracle/_ref is built);
* Q8_0 activation quantization: bit-exact against gguf-py's quantizer (documented bit-exact with
  ggml's reference quantize_row_q8_0);
* add_act: the reference's own test inputs and tolerance (tests/test_add_act.cpp:64-65, 86-98);
* transformer semantics (prefix mask, post-LN layers, PE, BERT projection, KV-cached decode):
  against a float64 numpy restatement on a model with F32 matrices (no activation quantization);
* export formats: F16 embeddings widen exactly; Q8_0 logits bit-exact against a numpy restatement
  of ggml's Q8_0 dot with a correctly rounded fmaf.
"""
import os

import numpy as np
import pytest

import gsv_synth as S
import oracle as O
from conftest import gguf_retyped_copy, rel_l2

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_sampler_matches_reference_golden():
    g = np.load(os.path.join(GOLDEN, "sampler_golden.npz"))
    for i in range(len(g["token"])):
        top_k, top_p, temp, rep = g["cfg"][i]
        prev = g["prev"][i][:g["n_prev"][i]]
        probs = O.logits_to_probs(g["logits"][i], top_k=int(top_k), top_p=float(top_p), temperature=float(temp),
                                  rep=float(rep), prev=prev)
        assert np.array_equal(probs.view(np.uint32), g["probs"][i].view(np.uint32)), i
        tok, st = O.sample(probs, int(g["state0"][i]))
        assert tok == g["token"][i] and st == int(g["state1"][i]), i


@pytest.mark.skipif(not os.path.exists(O.REF_SAMPLER_PATH), reason="reference sampler not built (make -C oracle ref)")
def test_sampler_matches_live_reference():
    ref = O.RefSampler()
    rng = np.random.default_rng(0)
    for it in range(400):
        lg = (rng.standard_normal(1025) * rng.choice([0.1, 0.45, 3.0])).astype(np.float32)
        if it % 7 == 0:
            lg = (np.round(lg * 4) / 4).astype(np.float32)
        cfg = dict(top_k=int(rng.choice([0, 1, 5, 15, 1025])), top_p=float(rng.choice([1.0, 0.9, 0.5])),
                   temperature=float(rng.choice([1.0, 0.7, 1.3])), rep=float(rng.choice([1.35, 1.0, 2.0])))
        prev = rng.integers(0, 1025, int(rng.integers(0, 300)), dtype=np.int32)
        p1 = ref.logits_to_probs(lg, prev=prev, **cfg)
        p2 = O.logits_to_probs(lg, prev=prev, **cfg)
        assert np.array_equal(p1.view(np.uint32), p2.view(np.uint32))
        st = int(rng.integers(1, 2**63))
        assert ref.sample(p1, st) == O.sample(p2, st)
        assert ref.rng_init(0) == O.rng_init(0) == 1


def test_q8_0_quantizer_golden_and_gguf():
    import gguf
    g = np.load(os.path.join(GOLDEN, "q8_0_golden.npz"))
    assert np.array_equal(O.quantize_q8_0(g["x"]), g["blocks"].ravel())
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(32 * 2048) * rng.choice([1e-3, 1.0, 50.0], 32 * 2048)).astype(np.float32)
    ref = gguf.quants.quantize(x.reshape(-1, 32), gguf.GGMLQuantizationType.Q8_0).ravel()
    assert np.array_equal(O.quantize_q8_0(x), ref)


def test_add_act_reference_test_inputs():
    """tests/test_add_act.cpp:15-16,64-65 inputs; ReLU (act 1) and identity within its 2e-3 bar."""
    NE0, NR = 64, 7
    i = np.arange(NE0 * NR)
    a = (0.02 * ((i * 37 % 101) - 50) + 0.5).astype(np.float32).reshape(NR, NE0)
    b = (0.01 * ((np.arange(NE0) * 13) % 29 - 14)).astype(np.float32)
    for act in (0, 1):
        ref = a + b if act == 0 else np.maximum(a + b, 0)
        assert np.abs(O.add_act(a, b, act) - ref).max() <= 2e-3
        assert np.array_equal(O.add_act(a, b, act), ref.astype(np.float32))
    # act 2, GELU (erf form): the test's formula in float64 within its 2e-3 bar, and the oracle's own
    # float evaluation ((0.5 v) (1 + erf(v / sqrt 2)), erf in double) bit for bit
    import math
    v = (a + b).astype(np.float32)
    ref = np.array([0.5 * x * (1.0 + math.erf(x / math.sqrt(2.0))) for x in v.astype(np.float64).ravel()]).reshape(v.shape)
    got = O.add_act(a, b, 2)
    assert np.abs(got - ref).max() <= 2e-3
    e = np.array([math.erf(float(np.float32(x) * np.float32(0.70710678118654752440))) for x in v.ravel()],
                 np.float64).astype(np.float32).reshape(v.shape)
    assert np.array_equal(got, (np.float32(0.5) * v) * (np.float32(1.0) + e))


def test_layernorm_vs_float64():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((50, 512)).astype(np.float32) * 3
    r = rng.standard_normal((50, 512)).astype(np.float32)
    bias = rng.standard_normal(512).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    b = rng.standard_normal(512).astype(np.float32)
    y = O.ln_affine(x, r, bias, w, b)
    v = x.astype(np.float64) + r + bias
    ref = (v - v.mean(1, keepdims=True)) / np.sqrt(v.var(1, keepdims=True) + 1e-5) * w + b
    assert np.abs(y - ref).max() < 1e-5


def test_decode_attention_canonical_vs_float64():
    """The page-split float evaluation (own exp, fixed order) is softmax(q.K) V to float accuracy,
    including single-key, partial-page and many-page rows and large score ranges."""
    rng = np.random.default_rng(12)
    lens = np.array([1, 2, 63, 64, 65, 130, 700, 2049], np.int32)
    B, L = len(lens), int(lens.max())
    q = (rng.standard_normal((B, 16, 32)) * 2).astype(np.float32)
    k = rng.standard_normal((B, L, 16, 32)).astype(np.float32)
    v = rng.standard_normal((B, L, 16, 32)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(32.0))
    got = O.decode_attention(q, k, v, lens, scale)
    for b in range(B):
        n = lens[b]
        s = np.einsum("hd,thd->ht", q[b].astype(np.float64), k[b, :n].astype(np.float64)) * float(scale)
        w = np.exp(s - s.max(1, keepdims=True))
        ref = np.einsum("ht,thd->hd", w / w.sum(1, keepdims=True), v[b, :n].astype(np.float64))
        assert np.abs(got[b] - ref).max() < 2e-5 * max(1.0, np.abs(ref).max()), b


def test_q8_mul_mat_vs_dequantized_float64():
    """Q8_0 mul_mat equals the float64 product of the dequantized operands up to float rounding."""
    rng = np.random.default_rng(3)
    N, K, M = 64, 512, 5
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    wb, xb = O.quantize_q8_0(W).reshape(N, K // 32, 34), O.quantize_q8_0(X).reshape(M, K // 32, 34)

    def deq(b):
        d = b[..., :2].copy().view(np.float16).astype(np.float64)
        q = b[..., 2:].copy().view(np.int8).astype(np.float64)
        return (q * d).reshape(b.shape[0], -1)

    ref = deq(xb) @ deq(wb).T
    got = O.mul_mat(O.quantize_q8_0(W), 8, N, K, X)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


# ------------------------------------------------------------------ float64 model restatement
def _np_model(path):
    import gguf
    rd = gguf.GGUFReader(path)
    T = {t.name: np.array(t.data, dtype=np.float64) for t in rd.tensors}
    return T


def _np_pe(n, D=512):
    pe = np.zeros((n, D), np.float64)
    pos = np.arange(n)[:, None]
    div = np.exp(np.arange(0, D, 2) * -(np.log(10000.0) / D))
    pe[:, 0::2] = np.sin(pos * div)
    pe[:, 1::2] = np.cos(pos * div)
    return pe


def _np_layer(T, li, x, att_fn):
    p = f"transformer.block{li}."
    qkv = x @ T[p + "qkv_w"].reshape(1536, 512).T + T[p + "qkv_b"]
    o = att_fn(qkv) @ T[p + "out_w"].reshape(512, 512).T
    v = x + o + T[p + "out_b"]
    n1 = (v - v.mean(-1, keepdims=True)) / np.sqrt(v.var(-1, keepdims=True) + 1e-5) * T[p + "norm1_w"] + T[p + "norm1_b"]
    h = np.maximum(n1 @ T[p + "ffn1_w"].reshape(2048, 512).T + T[p + "ffn1_b"], 0)
    v2 = n1 + h @ T[p + "ffn2_w"].reshape(512, 2048).T + T[p + "ffn2_b"]
    return (v2 - v2.mean(-1, keepdims=True)) / np.sqrt(v2.var(-1, keepdims=True) + 1e-5) * T[p + "norm2_w"] + \
        T[p + "norm2_b"], qkv


def _np_attend(q, k, v, mask):
    s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(32.0)
    s = np.where(mask[None], s, -np.inf)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", p, v)


def _np_trace(T, req, forced, NL):
    """float64 prefill + teacher-forced decode of one sequence -> logits per step."""
    Tn, P = len(req.phones), len(req.prompt)
    S = Tn + P
    pe = _np_pe(P + len(forced) + S + 1)
    x = np.concatenate([T["ar.text_emb"].reshape(-1, 512)[req.phones] + pe[:Tn],
                        T["ar.audio_emb"].reshape(-1, 512)[req.prompt] + pe[:P]])
    feat = np.asarray(req.bert, np.float64).T
    proj = feat @ T["ar.bert_proj"].reshape(512, 1024).T + T["ar.bert_proj_b"]
    x[:Tn] += proj
    qi = np.arange(S)[:, None]
    ki = np.arange(S)[None, :]
    mask = np.where(qi < Tn, ki < Tn, ki <= qi)
    Ks, Vs = [], []
    for li in range(NL):
        def att(qkv):
            q, k, v = (qkv[:, j * 512:(j + 1) * 512].reshape(S, 16, 32) for j in range(3))
            Ks.append(k)
            Vs.append(v)
            return _np_attend(q, k, v, mask).reshape(S, 512)
        x, _ = _np_layer(T, li, x, att)
    pred = T["ar.predict"].reshape(-1, 512)
    out = [x[-1] @ pred.T]
    for s, tok in enumerate(forced):
        y = T["ar.audio_emb"].reshape(-1, 512)[tok] + pe[P + s]
        y = y[None]
        for li in range(NL):
            def att(qkv):
                q, k, v = (qkv[:, j * 512:(j + 1) * 512].reshape(1, 16, 32) for j in range(3))
                Ks[li] = np.concatenate([Ks[li], k])
                Vs[li] = np.concatenate([Vs[li], v])
                return _np_attend(q, Ks[li], Vs[li], np.ones((1, Ks[li].shape[0]), bool)).reshape(1, 512)
            y, _ = _np_layer(T, li, y, att)
        out.append(y[0] @ pred.T)
    return np.array(out)


def test_oracle_transformer_vs_float64(model_f32_small):
    orc = O.OracleModel(model_f32_small)
    T = _np_model(model_f32_small)
    rng = np.random.default_rng(4)
    reqs = [S.make_request(rng, 37, 11), S.make_request(rng, 20, 0)]
    forced = rng.integers(0, 1024, (2, 5)).astype(np.int32)
    lg = orc.decode_trace(reqs, forced)
    for b in range(2):
        ref = _np_trace(T, reqs[b], forced[b], orc.NL)
        for s in range(ref.shape[0]):
            assert rel_l2(lg[s, b], ref[s]) < 2e-5, (b, s)


def test_oracle_generate_rules(model_small):
    """gsv_ar::generate rules: EOS never before step 11, teacher forcing, EOS finish and lens order."""
    orc = O.OracleModel(model_small)
    rng = np.random.default_rng(5)
    reqs = [S.make_request(rng, 12, 6) for _ in range(3)]
    forced = rng.integers(0, 1024, 20).astype(np.int32)
    forced[13] = 1024
    toks, lens = orc.generate(reqs, max_steps=20, oracle_tokens=forced, seed_base=3)
    assert lens == [13, 13, 13]
    for t in toks:
        assert len(t) == 6 + 13 and np.array_equal(t[6:], forced[:13])
    # early stop keyed on sequence 0: generated count > early_stop finishes every unfinished sequence
    toks, lens = orc.generate(reqs, max_steps=40, early_stop=7, seed_base=3)
    assert lens == [7, 7, 7] and all(len(t) == 6 + 7 for t in toks)
    # max_steps: the whole stream is kept
    toks, lens = orc.generate(reqs[:1], max_steps=9, top_k=1)
    assert lens == [9] and len(toks[0]) == 6 + 9
    assert 1024 not in toks[0][6:6 + 11]


def test_oracle_batch_equals_single(model_small):
    orc = O.OracleModel(model_small)
    reqs = S.ragged_requests(6, 3, lo=20, hi=60)
    seeds = [11, 12, 13]
    tb, _ = orc.generate(reqs, seeds=seeds, max_steps=25)
    for b in range(3):
        ts, _ = orc.generate([reqs[b]], seeds=[seeds[b]], max_steps=25)
        assert np.array_equal(tb[b], ts[0])


@pytest.mark.parametrize("emb_type", ["f16", "bf16"])
def test_oracle_f16_embeddings_widen_exactly(tmp_path, emb_type):
    """F16 / BF16 text/audio embeddings (exporter --spec emb=f16 / bf16) are widened exactly: the oracle
    gives the same logits, bit for bit, as for a twin file storing those values as F32."""
    e16 = S.write_model(str(tmp_path / "e16.gguf"), seed=21, dims=S.Dims(NL=2), emb_type=emb_type)
    import gguf
    F32 = gguf.GGMLQuantizationType.F32
    e32 = gguf_retyped_copy(e16, str(tmp_path / "e32.gguf"), {"ar.text_emb": F32, "ar.audio_emb": F32})
    rng = np.random.default_rng(21)
    reqs = [S.make_request(rng, 23, 9), S.make_request(rng, 14, 0)]
    forced = rng.integers(0, 1024, (2, 4)).astype(np.int32)
    a = O.OracleModel(e16).decode_trace(reqs, forced)
    b = O.OracleModel(e32).decode_trace(reqs, forced)
    assert np.array_equal(a, b)


def _fmaf(a, b, c):
    """Correctly rounded float32 fma of float32 arrays whose product a*b is exact in float64.

    The float64 sum s = a*b + c is rounded once; TwoSum gives its exact residual e. Rounding s to
    float32 is then wrong only when s lies exactly halfway between two float32 values and e != 0:
    the exact value lies on e's side of that midpoint."""
    p = np.asarray(a, np.float64) * np.asarray(b, np.float64)
    c = np.asarray(c, np.float64)
    s = p + c
    bv = s - p
    e = (p - (s - bv)) + (c - bv)
    f = s.astype(np.float32)
    g = np.nextafter(f, np.where(s > f, np.inf, -np.inf).astype(np.float32))
    mid = (f.astype(np.float64) + g.astype(np.float64)) * 0.5 == s
    up, dn = np.maximum(f, g), np.minimum(f, g)
    return np.where(mid & (e > 0), up, np.where(mid & (e < 0), dn, f))


def test_oracle_q8_0_logits_restated(tmp_path):
    """Q8_0 ar.predict (exporter --spec predict=q8_0): the logits equal, bit for bit, a numpy
    restatement of ggml's Q8_0 mul_mat -- the hidden state quantized by gguf-py's Q8_0 quantizer,
    exact integer block dots, float accumulation acc = fmaf(isum, d_w * d_x, acc) in block order."""
    import gguf
    path = S.write_model(str(tmp_path / "p8.gguf"), seed=22, dims=S.Dims(NL=2), predict_type="q8_0")
    orc = O.OracleModel(path)
    rng = np.random.default_rng(22)
    reqs = [S.make_request(rng, 31, 7), S.make_request(rng, 12, 20)]
    logits, dump = orc.first_logits(reqs, dump=True)
    W = next(t for t in gguf.GGUFReader(path).tensors if t.name == "ar.predict")
    wb = np.array(W.data).reshape(orc.V, orc.D // 32, 34)
    dw = wb[..., :2].copy().view(np.float16)[..., 0].astype(np.float32)
    qw = wb[..., 2:].copy().view(np.int8).astype(np.int32)
    for b in range(len(reqs)):
        x = dump[b, orc.NL - 1, 3]          # last layer's output at the last position
        xb = gguf.quants.quantize(x.reshape(1, orc.D), gguf.GGMLQuantizationType.Q8_0).reshape(-1, 34)
        dx = xb[:, :2].copy().view(np.float16)[:, 0].astype(np.float32)
        qx = xb[:, 2:].copy().view(np.int8).astype(np.int32)
        isum = (qw * qx[None]).sum(-1).astype(np.float32)
        d = dw * dx[None]                    # exact: two 11-bit significands
        acc = np.zeros(orc.V, np.float32)
        for ib in range(orc.D // 32):
            acc = _fmaf(isum[:, ib], d[:, ib], acc)
        assert np.array_equal(acc, logits[b]), b


def _round_bf16(x):
    """float32 -> bfloat16 -> float32, round to nearest even (finite values)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("wtype,K", [(0, 512), (1, 512), (1, 2048), (30, 512)])
def test_oracle_float_layer_mul_mat_restated(wtype, K):
    """F32 / F16 layer matrices (exporter default / --f16): the oracle's mul_mat equals, bit for bit, a
    numpy restatement of ggml's FMA-vectorised dot -- src1 rounded to F16 for an F16 matrix, 32 float
    FMA chains (chain c takes k = c, c+32, ...), chains folded pairwise as c^16, ^8, ^4, ^1, ^2."""
    rng = np.random.default_rng(31 + K + wtype)
    N, M = 40, 5
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    if wtype == 1:
        wraw = W.astype(np.float16)
        wf, xr = wraw.astype(np.float32), X.astype(np.float16).astype(np.float32)
    elif wtype == 30:   # BF16: gguf-py's converter (round to nearest even), src1 rounded the same way
        import gguf
        wraw = gguf.quants.quantize(W, gguf.GGMLQuantizationType.BF16)
        wf, xr = _round_bf16(W), _round_bf16(X)
        assert np.array_equal(wraw.view(np.uint16).astype(np.uint32) << 16, wf.view(np.uint32))
    else:
        wraw, wf, xr = W, W, X
    got = O.mul_mat(wraw, wtype, N, K, X, layer=True)
    s = np.zeros((M, N, 32), np.float32)
    for t in range(K // 32):
        s = _fmaf(wf[None, :, 32 * t:32 * t + 32], xr[:, None, 32 * t:32 * t + 32], s)
    for off in (16, 8, 4, 1, 2):
        lo = [c for c in range(32) if not c & off]
        s[..., lo] = s[..., lo] + s[..., [c | off for c in lo]]
    assert np.array_equal(got, s[..., 0])
    if wtype == 0:   # not the predict / BERT projection order (exact products, double sums)
        assert not np.array_equal(got, O.mul_mat(wraw, 0, N, K, X))


@pytest.mark.parametrize("wtype", [2, 6, 20])
def test_oracle_q4_0_q5_0_iq4_nl_as_q8_0_blocks(wtype):
    """Q4_0 / Q5_0 / IQ4_NL matrices (--spec ...=q4_0 / q5_0, tools/quantize_gguf.cpp iq4_nl): the oracle's
    mul_mat equals, bit for bit, the Q8_0 mul_mat of blocks holding gguf-py's dequantized values divided
    by the block scale (ggml's dot of these types against Q8_0 activations is the integer dot of those
    values scaled by d_w * d_x)."""
    import gguf
    ty = gguf.GGMLQuantizationType(wtype)
    rng = np.random.default_rng(40 + wtype)
    N, K, M = 48, 512, 6
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    raw = S.iq4_nl_blocks(W) if wtype == 20 else gguf.quants.quantize(W, ty)
    deq = gguf.quants.dequantize(raw, ty).reshape(N, K // 32, 32)
    bs = 22 if wtype == 6 else 18
    d = raw.reshape(N, K // 32, bs)[..., :2].copy().view(np.float16).astype(np.float32)
    assert (d != 0).all()
    q = deq / d                                   # exact: deq is d * (an integer of at most 8 bits)
    assert np.array_equal(q, np.round(q)) and np.abs(q).max() <= {2: 8, 6: 16, 20: 127}[wtype]
    q8 = np.zeros((N, K // 32, 34), np.uint8)
    q8[..., :2] = raw.reshape(N, K // 32, bs)[..., :2]
    q8[..., 2:] = q.astype(np.int8).view(np.uint8)
    got = O.mul_mat(raw, wtype, N, K, X)
    assert np.array_equal(got, O.mul_mat(q8, 8, N, K, X))
    ref = X.astype(np.float64) @ deq.reshape(N, K).astype(np.float64).T
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()   # Q8_0 activation rounding only


@pytest.mark.parametrize("wtype", [3, 7])
def test_oracle_q4_1_q5_1_restated(wtype):
    """Q4_1 / Q5_1 matrices (exporter --spec ...=q4_1 / q5_1): the oracle's mul_mat equals, bit for bit, a
    numpy restatement of ggml's portable Q4_1 / Q5_1 x Q8_1 dot -- src1 quantized to Q8_1 (Q8_0 values
    and scale, s = fp16(sum * d)), per block the integer dot sumi of the unsigned weight values with
    them, sumf = sumf + fma(d_w*d_x, sumi, m_w*s_x) in block order. The weight values are unpacked
    independently and checked against gguf-py's dequantizer."""
    import gguf
    ty = gguf.GGMLQuantizationType(wtype)
    rng = np.random.default_rng(50 + wtype)
    N, K, M = 40, 512, 5
    nb = K // 32
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    raw = gguf.quants.quantize(W, ty)
    blk = raw.reshape(N, nb, 20 if wtype == 3 else 24)
    d = blk[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    mn = blk[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    qs = blk[..., 4:20] if wtype == 3 else blk[..., 8:24]
    q = np.concatenate([qs & 15, qs >> 4], -1).astype(np.int64)
    if wtype == 7:
        qh = blk[..., 4:8].copy().view("<u4")[..., 0]
        q += ((qh[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int64) * 16
    deq = gguf.quants.dequantize(raw, ty).reshape(N, nb, 32)
    assert np.array_equal(d[..., None] * q.astype(np.float32) + mn[..., None], deq)
    xb = X.reshape(M, nb, 32)
    dx = (np.abs(xb).max(-1) / np.float32(127)).astype(np.float32)
    idx = np.where(dx != 0, np.float32(1) / np.where(dx != 0, dx, np.float32(1)), np.float32(0)).astype(np.float32)
    v = (xb * idx[..., None]).astype(np.float32)
    qx = (np.sign(v) * np.floor(np.abs(v).astype(np.float64) + 0.5)).astype(np.int64)     # roundf
    assert np.array_equal(qx.astype(np.int8).view(np.uint8),
                          O.quantize_q8_0(X).reshape(M, nb, 34)[..., 2:])
    sx = (qx.sum(-1).astype(np.float32) * dx).astype(np.float16).astype(np.float32)
    dxr = dx.astype(np.float16).astype(np.float32)
    sumi = np.einsum("nbj,mbj->mnb", q, qx).astype(np.float32)
    acc = np.zeros((M, N), np.float32)
    for b in range(nb):
        dd = (d[None, :, b] * dxr[:, None, b]).astype(np.float32)
        ms = (mn[None, :, b] * sx[:, None, b]).astype(np.float32)
        acc = (acc + _fmaf(dd, sumi[..., b], ms)).astype(np.float32)
    assert np.array_equal(O.mul_mat(raw, wtype, N, K, X), acc)


def _kquant_unpack(raw, kind, nsb):
    """(values, per-value scale, d, dmin, mins) of K-quant blocks, unpacked in numpy."""
    if kind == "q6_k":
        b = raw.reshape(nsb, 210)
        ql, qh = b[:, :128].astype(np.int64), b[:, 128:192].astype(np.int64)
        q = np.zeros((nsb, 256), np.int64)
        for hh in range(2):
            for k in range(4):
                lo = ql[:, 64 * hh + (k & 1) * 32: 64 * hh + (k & 1) * 32 + 32]
                nib = lo & 15 if k < 2 else lo >> 4
                q[:, 128 * hh + 32 * k: 128 * hh + 32 * k + 32] = (nib | (((qh[:, 32 * hh: 32 * hh + 32] >> (2 * k)) & 3) << 4)) - 32
        sc = np.repeat(b[:, 192:208].copy().view(np.int8).astype(np.int64), 16, axis=1)
        d = b[:, 208:210].copy().view(np.float16)[:, 0].astype(np.float32)
        return q, sc, d, None, None
    b = raw.reshape(nsb, 144 if kind == "q4_k" else 176)
    d = b[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float32)
    s = b[:, 4:16].astype(np.int64)
    sc = np.zeros((nsb, 8), np.int64)
    mn = np.zeros((nsb, 8), np.int64)
    for j in range(8):
        if j < 4:
            sc[:, j], mn[:, j] = s[:, j] & 63, s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    qs = b[:, 16:144] if kind == "q4_k" else b[:, 48:176]
    q = np.zeros((nsb, 256), np.int64)
    for g in range(4):
        q[:, 64 * g: 64 * g + 32] = qs[:, 32 * g: 32 * g + 32] & 15
        q[:, 64 * g + 32: 64 * g + 64] = qs[:, 32 * g: 32 * g + 32] >> 4
        if kind == "q5_k":
            qh = b[:, 16:48].astype(np.int64)
            q[:, 64 * g: 64 * g + 32] += ((qh >> (2 * g)) & 1) * 16
            q[:, 64 * g + 32: 64 * g + 64] += ((qh >> (2 * g + 1)) & 1) * 16
    return q, np.repeat(sc, 32, axis=1), d, dmin, mn


@pytest.mark.parametrize("kind,wtype", [("q4_k", 12), ("q5_k", 13), ("q6_k", 14)])
def test_oracle_kquant_restated(kind, wtype):
    """K-quant matrices (exporter --spec ...=q4_k / q5_k / q6_k): the oracle's mul_mat equals, bit for bit, a
    numpy restatement of ggml's portable K-quant x Q8_K dot -- src1 quantized to Q8_K per 256 values
    (iscale = -127/max, round half to even, d = 1/iscale, sums of 16), eight integer lane sums per
    super-block (value e to lane e mod 8, times its sub-block scale), sums[l] = fma(d_w*d_x, lane, sums[l]),
    for Q4_K / Q5_K sumf = fma(-dmin_w*d_x, sum of bsums*mins, sumf), then sumf + sums[0] + ... + sums[7].
    The unpacked weights are checked against gguf-py's dequantizer."""
    import gguf
    ty = gguf.GGMLQuantizationType(wtype)
    rng = np.random.default_rng(60 + wtype)
    N, K, M = 24, 512, 5
    nsb = K // 256
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    X[1, :256] = 0.0                                  # an all-zero activation super-block
    raw = S.kquant_blocks(W, kind)
    q, sc, d, dmin, mn = _kquant_unpack(raw, kind, N * nsb)
    deq = gguf.quants.dequantize(raw, ty).reshape(N * nsb, 256)
    w = (d[:, None] * sc.astype(np.float32)).astype(np.float32) * q.astype(np.float32)
    if dmin is not None:
        w = w - np.repeat((dmin[:, None] * mn.astype(np.float32)).astype(np.float32), 32, axis=1)
    np.testing.assert_allclose(w, deq, rtol=0, atol=1e-6 * np.abs(deq).max())
    # Q8_K of the activations
    xb = X.reshape(M * nsb, 256)
    mx = xb[np.arange(M * nsb), np.abs(xb).argmax(-1)]
    iscale = np.where(mx != 0, np.float32(-127) / np.where(mx != 0, mx, np.float32(1)), np.float32(0)).astype(np.float32)
    qx = np.minimum(127, np.rint((iscale[:, None] * xb).astype(np.float32))).astype(np.int64)
    dx = np.where(mx != 0, np.float32(1) / np.where(iscale != 0, iscale, np.float32(1)), np.float32(0)).astype(np.float32)
    bs = qx.reshape(M * nsb, 16, 16).sum(-1)
    q, sc = q.reshape(N, nsb, 256), sc.reshape(N, nsb, 256)
    qx, dx, bs = qx.reshape(M, nsb, 256), dx.reshape(M, nsb), bs.reshape(M, nsb, 16)
    sums = np.zeros((M, N, 8), np.float32)
    sumf = np.zeros((M, N), np.float32)
    for s_ in range(nsb):
        prod = np.einsum("ne,me->mne", sc[:, s_] * q[:, s_], qx[:, s_])
        lanes = prod.reshape(M, N, 32, 8).sum(2).astype(np.float32)      # value e -> lane e % 8
        dd = (d.reshape(N, nsb)[None, :, s_] * dx[:, None, s_]).astype(np.float32)
        sums = _fmaf(dd[..., None], lanes, sums).astype(np.float32)
        if dmin is not None:
            sumi = (bs[:, None, s_, :] * np.repeat(mn.reshape(N, nsb, 8)[None, :, s_, :], 2, axis=-1)).sum(-1)
            dm = (dmin.reshape(N, nsb)[None, :, s_] * dx[:, None, s_]).astype(np.float32)
            sumf = _fmaf(-dm, sumi.astype(np.float32), sumf).astype(np.float32)
    for l in range(8):
        sumf = (sumf + sums[..., l]).astype(np.float32)
    assert np.array_equal(O.mul_mat(raw, wtype, N, K, X), sumf)


# ------------------------------------------------------------------ BERT feature producer
def _np_bert(path, ids, n_layers):
    """float64 numpy BERT (HF BertModel semantics, post-LN, GELU erf) over the GGUF weights -> [D][T]."""
    import gguf
    from scipy.special import erf
    rd = gguf.GGUFReader(path)
    kv = {f.name: f.parts[f.data[0]][0] for f in rd.fields.values() if f.name.startswith("bert.")}
    D, NH, FF, eps = int(kv["bert.hidden"]), int(kv["bert.head"]), int(kv["bert.inter"]), float(kv["bert.ln_eps"])
    HD = D // NH
    T = {t.name: np.array(t.data, dtype=np.float64) for t in rd.tensors}

    def ln(v, w, b):
        return (v - v.mean(-1, keepdims=True)) / np.sqrt(v.var(-1, keepdims=True) + eps) * w + b

    S = len(ids)
    x = T["bert.word_emb"].reshape(-1, D)[ids] + T["bert.pos_emb"].reshape(-1, D)[:S] + T["bert.type_emb"].reshape(-1, D)[0]
    x = ln(x, T["bert.emb_ln_w"], T["bert.emb_ln_b"])
    for li in range(n_layers):
        p = f"bert.l{li}."
        qkv = x @ T[p + "qkv_w"].reshape(3 * D, D).T + T[p + "qkv_b"]
        q, k, v = (qkv[:, i * D:(i + 1) * D].reshape(S, NH, HD) for i in range(3))
        s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(HD)
        a = np.exp(s - s.max(-1, keepdims=True))
        att = np.einsum("hqk,khd->qhd", a / a.sum(-1, keepdims=True), v).reshape(S, D)
        x = ln(x + att @ T[p + "attn_out_w"].reshape(D, D).T + T[p + "attn_out_b"], T[p + "attn_ln_w"], T[p + "attn_ln_b"])
        hpre = x @ T[p + "ff1_w"].reshape(FF, D).T + T[p + "ff1_b"]
        h = 0.5 * hpre * (1.0 + erf(hpre / np.sqrt(2.0)))
        x = ln(x + h @ T[p + "ff2_w"].reshape(D, FF).T + T[p + "ff2_b"], T[p + "out_ln_w"], T[p + "out_ln_b"])
    return x.T


@pytest.mark.parametrize("mat_type,tol", [("f32", 1e-6), ("f16", 2e-4)])
def test_bert_oracle_vs_float64(tmp_path, mat_type, tol):
    """The BERT feature producer (src/gsv_bert.cpp): embeddings + LayerNorm, post-LN layers with GELU-erf
    FFN, only bert.layers_used layers run; [D][T] features, encode_feat drops [CLS] / [SEP]. Against an
    independent float64 numpy BERT on the same GGUF: F32 matrices within float accumulation, F16 matrices
    within the F16 rounding of the activations (ggml's vec_dot_type)."""
    dims = S.BertDims(D=128, NH=2, FF=512, NL=5, VOCAB=300, MAXPOS=48)
    path = S.write_bert_model(str(tmp_path / f"bert_{mat_type}.gguf"), seed=7, dims=dims, mat_type=mat_type)
    orc = O.BertOracle(path)
    assert orc.NL == 3 and orc.D == 128
    rng = np.random.default_rng(8)
    ids = rng.integers(0, 300, 37).astype(np.int32)
    for k in (0, 1, 3):
        got = orc.encode(ids, n_layers=k)
        assert got.shape == (128, 37)
        assert rel_l2(got, _np_bert(path, ids, k)) < (5e-7 if k == 0 else tol), k
    full = orc.encode(ids)
    assert np.array_equal(full, orc.encode(ids, n_layers=3))
    assert np.array_equal(orc.encode_feat(ids), full[:, 1:-1])
    feats, per = orc.encode_layers(ids)
    assert len(per) == 4 and np.array_equal(feats, full) and np.array_equal(per[1], orc.encode(ids, n_layers=1))
    lens = [37, 5, 2]
    flat = np.concatenate([ids, ids[:5], ids[:2]] + [np.zeros(0, np.int32)])
    slots = np.zeros(3 * 40, np.int32)
    for b, (o, n) in enumerate(zip([0, 37, 42], lens)):
        slots[b * 40: b * 40 + n] = flat[o: o + n]
    bat = orc.encode_feat_batch(slots, lens, 40)
    assert np.array_equal(bat[0], orc.encode_feat(ids)) and bat[1].shape == (128, 3) and bat[2].shape == (128, 0)


def test_bert_oracle_vs_transformers(tmp_path):
    """The BERT restatement against Hugging Face's BertModel (the model GPT-SoVITS takes hidden_states[-3]
    from) in float64, with the synthetic GGUF weights mapped back the way tools/export_gguf/convert_bert.py
    wrote them (q|k|v rows concatenated): embeddings, post-LN layers, GELU (erf), and layers_used =
    n_layer - 2 = hidden_states[-3]."""
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    import gguf
    dims = S.BertDims(D=128, NH=2, FF=512, NL=5, VOCAB=300, MAXPOS=48)
    path = S.write_bert_model(str(tmp_path / "bert_hf.gguf"), seed=11, dims=dims)
    T = {t.name: torch.from_numpy(np.array(t.data, dtype=np.float64)) for t in gguf.GGUFReader(path).tensors}
    D = dims.D
    cfg = transformers.BertConfig(vocab_size=dims.VOCAB, hidden_size=D, num_hidden_layers=dims.NL,
                                  num_attention_heads=dims.NH, intermediate_size=dims.FF,
                                  max_position_embeddings=dims.MAXPOS, type_vocab_size=2, layer_norm_eps=1e-12,
                                  hidden_act="gelu", hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    model = transformers.BertModel(cfg, add_pooling_layer=False).double().eval()
    sd = {"embeddings.word_embeddings.weight": T["bert.word_emb"].reshape(-1, D),
          "embeddings.position_embeddings.weight": T["bert.pos_emb"].reshape(-1, D),
          "embeddings.token_type_embeddings.weight": T["bert.type_emb"].reshape(-1, D),
          "embeddings.LayerNorm.weight": T["bert.emb_ln_w"], "embeddings.LayerNorm.bias": T["bert.emb_ln_b"]}
    for li in range(dims.NL):
        p, h = f"bert.l{li}.", f"encoder.layer.{li}."
        w, b = T[p + "qkv_w"].reshape(3 * D, D), T[p + "qkv_b"]
        for i, n in enumerate(("query", "key", "value")):
            sd[h + f"attention.self.{n}.weight"] = w[i * D:(i + 1) * D]
            sd[h + f"attention.self.{n}.bias"] = b[i * D:(i + 1) * D]
        sd[h + "attention.output.dense.weight"] = T[p + "attn_out_w"].reshape(D, D)
        sd[h + "attention.output.dense.bias"] = T[p + "attn_out_b"]
        sd[h + "attention.output.LayerNorm.weight"] = T[p + "attn_ln_w"]
        sd[h + "attention.output.LayerNorm.bias"] = T[p + "attn_ln_b"]
        sd[h + "intermediate.dense.weight"] = T[p + "ff1_w"].reshape(dims.FF, D)
        sd[h + "intermediate.dense.bias"] = T[p + "ff1_b"]
        sd[h + "output.dense.weight"] = T[p + "ff2_w"].reshape(D, dims.FF)
        sd[h + "output.dense.bias"] = T[p + "ff2_b"]
        sd[h + "output.LayerNorm.weight"] = T[p + "out_ln_w"]
        sd[h + "output.LayerNorm.bias"] = T[p + "out_ln_b"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("position_ids" in k or "token_type_ids" in k for k in missing), missing
    ids = np.random.default_rng(12).integers(0, dims.VOCAB, 29).astype(np.int32)
    with torch.no_grad():
        hs = model(torch.from_numpy(ids.astype(np.int64))[None], output_hidden_states=True).hidden_states
    ref = hs[-3][0].numpy().T                                          # [D][T]
    assert rel_l2(O.BertOracle(path).encode(ids), ref) < 1e-6


def test_oracle_serving_equals_generate(model_small):
    """The oracle's continuous-batching loop (OracleServer: the CPU arm of the serving benchmark and the
    reference for the library's gsvcu_serve_*): sequences admitted into refilled slots, with different
    sampler settings and an early-stop limit, each produce exactly the tokens of generate alone."""
    orc = O.OracleModel(model_small)
    reqs = S.ragged_requests(55, 6, lo=40, hi=120)
    seeds = [500 + i for i in range(6)]
    steps = [40, 40, 40, 40, 68, 75]
    cfgs = [dict(), dict(top_k=5, top_p=0.8, temperature=0.7, rep=1.1), dict(top_k=1),
            dict(top_k=30, top_p=0.95, temperature=1.3), dict(), dict(top_k=3)]
    early = [-1, 30, -1, -1, 50, -1]
    alone = []
    for i in range(6):
        t, _ = orc.generate([reqs[i]], seeds=[seeds[i]], max_steps=steps[i], early_stop=early[i], **cfgs[i])
        alone.append(t[0][len(reqs[i].prompt):])
    srv = O.OracleServer(orc, 4, 512)
    for i in range(4):
        srv.admit([reqs[i]], [seeds[i]], [i], max_steps=steps[i], early_stop=early[i], **cfgs[i])
    served, pending = {}, 4
    for _ in range(200):
        if len(served) == 6:
            break
        for f in srv.step(8, tok_cap=100000):
            served[f["tag"]] = f
            if pending < 6:
                srv.admit([reqs[pending]], [seeds[pending]], [pending], max_steps=steps[pending],
                          early_stop=early[pending], **cfgs[pending])
                pending += 1
    assert len(served) == 6 and srv.active() == 0
    for i in range(6):
        assert np.array_equal(served[i]["tokens"], alone[i]), i
        kind = served[i]["finish_kind"]
        assert served[i]["n_generated"] == (steps[i] if kind == 2 else len(alone[i]))
    assert srv.tokens_total() == sum(len(a) for a in alone)
