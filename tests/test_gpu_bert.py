"""The BERT feature producer on B200 (gsvcu_bert_*, the role of gsv.cpp's gsv_bert, src/gsv_bert.cpp)
against the CPU restatement (oracle BertOracle, itself pinned to Hugging Face's BertModel in float64).

The GPU evaluates the oracle's arithmetic operation for operation (ggml's FMA-vectorised dot order for
F32 / F16 matrices, exact integer block dots for Q8_0, LayerNorm sums in double, attention in double
rounded once, GELU with erf in double), so features are compared bit for bit; the double sums of
LayerNorm and attention may round differently at a tie, so a handful of 1-ulp differences is allowed.
"""
import numpy as np
import pytest

import gsv_synth as S
import oracle as O
from conftest import MODEL_CACHE, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _model(tmp_path_factory, name, dims, mat_type):
    p = tmp_path_factory.mktemp("bert") / f"{name}.gguf"
    return S.write_bert_model(str(p), seed=13, dims=dims, mat_type=mat_type)


def _ulps(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def _close(got, ref):
    """Equal but for rare 1-ulp differences (double sums rounding differently at a tie)."""
    u = _ulps(got, ref)
    assert u.max() <= 4 and np.count_nonzero(u) <= max(2, u.size // 100000), (u.max(), np.count_nonzero(u))
    assert rel_l2(got, ref) < 1e-6


SMALL = S.BertDims(D=256, NH=4, FF=512, NL=4, VOCAB=500, MAXPOS=128)


@pytest.mark.parametrize("mat_type", ["f32", "f16", "q8_0"])
def test_bert_encode_layers_match_oracle(tmp_path_factory, mat_type):
    """encode / encode_layers: every layer's [D][T] output (0 = embedding LayerNorm) for F32, F16 and Q8_0
    matrices."""
    import gsvcu
    path = _model(tmp_path_factory, f"small_{mat_type}", SMALL, mat_type)
    orc = O.BertOracle(path)
    g = gsvcu.Bert(path)
    assert (g.hp.hidden, g.hp.n_head, g.hp.inter, g.hp.layers_used) == (256, 4, 512, 2)
    rng = np.random.default_rng(3)
    for T in (1, 7, 64, 65, 128):
        ids = rng.integers(0, 500, T).astype(np.int32)
        for k in range(g.hp.layers_used + 1):
            _close(g.encode(ids, n_layers=k), orc.encode(ids, n_layers=k))
    g.close()


def test_bert_feat_batch_matches_single_and_oracle(tmp_path_factory):
    """encode_feat_batch: sequences of different lengths in slots of Tmax (padding ignored), each equal to
    its own encode_feat and to the oracle; short sequences (<= 2 ids) give empty features; features can
    be written to device memory for the AR prefill."""
    import gsvcu
    path = _model(tmp_path_factory, "small_f32", SMALL, "f32")
    orc = O.BertOracle(path)
    g = gsvcu.Bert(path)
    rng = np.random.default_rng(4)
    lens = [5, 2, 40, 17, 64, 3]
    tmax = 64
    ids = rng.integers(0, 500, (len(lens), tmax)).astype(np.int32)
    feats = g.encode_feat_batch(ids.ravel(), lens, tmax)
    ref = orc.encode_feat_batch(ids.ravel(), lens, tmax)
    for b, l in enumerate(lens):
        assert feats[b].shape == (256, max(l - 2, 0))
        single = g.encode_feat_batch(ids[b], [l], tmax)[0]
        assert np.array_equal(feats[b].view(np.uint32), single.view(np.uint32)), b
        if l > 2:
            _close(feats[b], ref[b])
    total = sum(256 * max(l - 2, 0) for l in lens)
    dev = torch.empty(total, dtype=torch.float32, device="cuda")
    g.encode_feat_batch(ids.ravel(), lens, tmax, out=dev)
    flat = np.concatenate([f.ravel() for f in feats])
    assert np.array_equal(dev.cpu().numpy().view(np.uint32), flat.view(np.uint32))
    g.close()


def test_bert_published_shape_matches_oracle(tmp_path_factory):
    """The published chinese-roberta-wwm-ext-large shape (hidden 1024, 16 heads of 64, FFN 4096), F16
    matrices as the exporter's --spec writes them, two layers: features equal the oracle's."""
    import gsvcu
    dims = S.BertDims(D=1024, NH=16, FF=4096, NL=4, VOCAB=21128, MAXPOS=512)
    path = _model(tmp_path_factory, "large_f16", dims, "f16")
    orc = O.BertOracle(path)
    g = gsvcu.Bert(path)
    rng = np.random.default_rng(5)
    ids = np.concatenate([[101], rng.integers(672, 8000, 38), [102]]).astype(np.int32)
    _close(g.encode(ids), orc.encode(ids))
    _close(g.encode_feat_batch(ids, [ids.size], ids.size)[0], orc.encode_feat(ids))
    g.close()


def test_bert_rejects_bad_inputs(tmp_path_factory):
    import gsvcu
    path = _model(tmp_path_factory, "small_f32", SMALL, "f32")
    g = gsvcu.Bert(path)
    with pytest.raises(gsvcu.GsvcuError):
        g.encode(np.array([1, 600, 2], np.int32))           # id beyond the vocabulary
    with pytest.raises(gsvcu.GsvcuError):
        g.encode(np.zeros(129, np.int32))                   # longer than max_pos
    with pytest.raises(gsvcu.GsvcuError):
        g.encode_feat_batch(np.zeros(8, np.int32), [5, 9], 4)   # length beyond its slot
    g.close()


def test_cpp_dropin_bert_class(tmp_path_factory, tmp_path):
    """The C++ `class gsv_bert` shim (include/gsv_bert.h, csrc/gsv_bert.cpp) gives the C ABI's features:
    encode_feat_batch, encode_feat and encode_feat_cached agree per sequence, the LRU counts hits and
    misses as the reference's (src/gsv_bert.cpp:241-266), encode_layers returns layers_used + 1 arrays."""
    import json
    import os
    import struct
    import subprocess
    import gsvcu
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = os.path.join(root, "tests", "cpp", "bin", "gsv_bert_smoke")
    assert os.path.exists(exe), "build with `make -C tests/cpp`"
    path = _model(tmp_path_factory, "small_f16", SMALL, "f16")
    rng = np.random.default_rng(6)
    lens, tmax = [9, 30, 2, 17], 32
    ids = rng.integers(0, 500, (len(lens), tmax)).astype(np.int32)
    f = tmp_path / "ids.bin"
    with open(f, "wb") as fh:
        fh.write(struct.pack("<ii", len(lens), tmax))
        fh.write(np.array(lens, np.int32).tobytes())
        fh.write(ids.tobytes())
    out = subprocess.run([exe, path, str(f)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    lines = [json.loads(x) for x in out.stdout.strip().splitlines()]
    assert (lines[0]["hidden"], lines[0]["layers_used"], lines[0]["max_pos"]) == (256, 2, 128)
    g = gsvcu.Bert(path)
    feats = g.encode_feat_batch(ids.ravel(), lens, tmax)
    w = lambda a: float((a.ravel().astype(np.float64) * ((np.arange(a.size) % 7) + 1)).sum())
    for b in range(len(lens)):
        rec = lines[1 + b]
        assert rec["n"] == feats[b].size
        assert rec["batch"] == rec["single"] == rec["cached"]
        np.testing.assert_allclose(rec["batch"], w(feats[b]), rtol=1e-9, atol=1e-9)
    last = lines[-1]
    assert (last["hits"], last["misses"]) == (0, 5)   # sequence 0 was evicted by the 2-entry LRU
    assert last["layers"] == 3
    np.testing.assert_allclose(last["full"], w(g.encode(ids[0, :lens[0]])), rtol=1e-9)
    g.close()
