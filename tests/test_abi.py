"""The C ABI surface on the CPU: the library loads, exports every entry point the header declares,
validates GGUF files on the host (corrupt files, wrong dtypes, missing tensors -> error codes, no
crash), and refuses cleanly without an sm_100 GPU. No GPU work is launched here."""
import ctypes as C
import os
import shutil

import numpy as np
import pytest

import gsvcu

HAVE_GPU = False
try:
    import torch
    HAVE_GPU = torch.cuda.is_available()
except Exception:
    pass


def test_every_declared_symbol_is_exported():
    lib = gsvcu.load_library()
    declared = gsvcu.declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
        assert name in gsvcu.SIGNATURES, f"{name} has no ctypes signature"


def test_inspect_valid_model(model_small):
    rc, hp, msg = gsvcu.inspect_gguf(model_small)
    assert rc == gsvcu.OK, msg
    assert (hp.hidden_dim, hp.n_head, hp.n_layer, hp.vocab_size, hp.eos, hp.bert_dim) == (512, 16, 2, 1025, 1024, 1024)
    assert hp.text_pe_alpha == 1.0 and hp.audio_pe_alpha == 1.0


def test_inspect_rejects_bad_files(model_small, model_f32_small, tmp_path):
    rc, _, msg = gsvcu.inspect_gguf(str(tmp_path / "missing.gguf"))
    assert rc == -4 and "cannot open" in msg
    data = open(model_small, "rb").read()
    bad = tmp_path / "bad_magic.gguf"
    bad.write_bytes(b"XXXX" + data[4:])
    assert gsvcu.inspect_gguf(str(bad))[0] == -4
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(data[: len(data) // 2])
    rc, _, msg = gsvcu.inspect_gguf(str(trunc))
    assert rc == -4 and "out of file bounds" in msg
    hdr = tmp_path / "hdr.gguf"
    hdr.write_bytes(data[:40])
    assert gsvcu.inspect_gguf(str(hdr))[0] == -4
    # layer matrices Q8_0, F32 or F16: F32 matrices load
    rc, _, msg = gsvcu.inspect_gguf(model_f32_small)
    assert rc == gsvcu.OK, msg


@pytest.mark.parametrize("mat_type,ffn_type,predict_type,emb_type", [
    ("q8_0", "q8_0", "q8_0", "f32"), ("q8_0", "q8_0", "f32", "f16"), ("f16", "f16", "f16", "f16"),
    ("f32", "f32", "f32", "f32"), ("q8_0", "f16", "f32", "f32"), ("f16", "q8_0", "f32", "f32"),
    ("q4_0", "q4_0", "q4_0", "f32"), ("q8_0", "q5_0", "q5_0", "f16"), ("q8_0", "iq4_nl", "iq4_nl", "f32"),
    ("bf16", "bf16", "bf16", "bf16"), ("q4_1", "q4_1", "q4_1", "f32"), ("q8_0", "q5_1", "q5_1", "f16"),
    ("q8_0", "q6_k", "f16", "f16"), ("q4_k", "q5_k", "q6_k", "f32")])
def test_inspect_export_formats(mat_type, ffn_type, predict_type, emb_type):
    """The exporter's formats: Q8_0 / Q4_0 / Q5_0 / F16 predict, F16 embeddings, F32 / F16 / Q4_0 / Q5_0
    attention and FFN matrices and mixed attn / ffn groups are accepted (GPU parity:
    tests/test_gpu_model.py::test_export_formats_match_oracle)."""
    import gsv_synth as S
    from conftest import MODEL_CACHE
    rc, hp, msg = gsvcu.inspect_gguf(S.cached_model(MODEL_CACHE, seed=9, n_layer=2, mat_type=mat_type,
                                                    predict_type=predict_type, emb_type=emb_type,
                                                    ffn_type=ffn_type))
    assert rc == gsvcu.OK, msg
    assert hp.vocab_size == 1025


def test_inspect_rejects_unsupported_matrix_types(model_small, tmp_path):
    """ffn1_w and ffn2_w of a layer are one group (Q8_0-class, or float-input: F32 / F16 / BF16 / Q4_1 /
    Q5_1 / K-quants); ggml types no reference tool writes (Q2_K, Q3_K, the IQ2 / IQ3 family) are refused
    with the tensor named."""
    import gguf
    from conftest import gguf_retyped_copy
    T = gguf.GGMLQuantizationType
    mixed = gguf_retyped_copy(model_small, str(tmp_path / "mixed.gguf"), {"transformer.block1.ffn2_w": T.F32})
    rc, _, msg = gsvcu.inspect_gguf(mixed)
    assert rc == -5 and "transformer.block1.ffn1_w / ffn2_w" in msg
    q2k = gguf_retyped_copy(model_small, str(tmp_path / "q2k.gguf"), {"transformer.block0.out_w": T.Q2_K})
    rc, _, msg = gsvcu.inspect_gguf(q2k)
    assert rc == -5 and "transformer.block0.out_w has ggml type 10" in msg


def test_inspect_missing_tensor(tmp_path):
    import gguf
    w = gguf.GGUFWriter(str(tmp_path / "partial.gguf"), "gsv.ar")
    w.add_uint32("ar.n_layer", 1)
    w.add_tensor("ar.text_emb", np.zeros((732, 512), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    rc, _, msg = gsvcu.inspect_gguf(str(tmp_path / "partial.gguf"))
    assert rc == -5 and "missing tensor" in msg


@pytest.mark.skipif(HAVE_GPU, reason="checks the no-GPU refusal")
def test_create_without_gpu_is_a_clean_error():
    lib = gsvcu.load_library()
    h = C.c_void_p()
    assert lib.gsvcu_create(0, C.byref(h)) == -7
    assert not h.value
    with pytest.raises(gsvcu.GsvcuError):
        gsvcu.Context(0)


def test_null_arguments_are_rejected():
    lib = gsvcu.load_library()
    assert lib.gsvcu_create(0, None) == -1
    assert lib.gsvcu_first_logits(None, None, 1, None) == -1
    assert lib.gsvcu_generate(None, None, 1, None, 0, -1, 10, None, 0, None, 0, None, None, None, 0,
                              gsvcu.PROGRESS_FN(), None) == -1
    assert lib.gsvcu_serve_step(None, 1, None, 0, None, 0) == -1
    assert lib.gsvcu_inspect_gguf(None, None, None, 0) == -1
    assert lib.gsvcu_last_error(None) == b"null context"


def test_dit_and_bert_null_arguments_are_rejected():
    """The DiT and BERT entry points validate their pointers on the host before any device work."""
    lib = gsvcu.load_library()
    h = C.c_void_p()
    assert lib.gsvcu_dit_load(0, None, C.byref(h)) == -1
    assert lib.gsvcu_dit_load(0, b"x.gguf", None) == -1
    assert lib.gsvcu_bert_load(0, None, C.byref(h)) == -1
    assert lib.gsvcu_bert_load(0, b"x.gguf", None) == -1
    buf = (C.c_float * 256)()
    assert lib.gsvcu_dit_velocity(None, buf, C.c_float(0.5), 0, buf) == -1
    assert lib.gsvcu_dit_set_alg(None, 1) == -1
    assert lib.gsvcu_dit_set_dbcache(None, 1, C.c_float(0.1), 0, 0, -1, -1, C.c_float(-1.0), 1) == -1
    assert lib.gsvcu_bert_encode(None, None, 1, 0, None) == -1
    assert lib.gsvcu_dit_last_error(None) == b"null DiT context"
    assert lib.gsvcu_bert_last_error(None) == b"null BERT context"


@pytest.mark.skipif(HAVE_GPU, reason="checks the no-GPU refusal")
def test_dit_and_bert_load_without_gpu_is_a_clean_error(tmp_path):
    lib = gsvcu.load_library()
    h = C.c_void_p()
    assert lib.gsvcu_dit_load(0, str(tmp_path / "none.gguf").encode(), C.byref(h)) == -7
    assert not h.value
    assert lib.gsvcu_bert_load(0, str(tmp_path / "none.gguf").encode(), C.byref(h)) == -7
    assert not h.value


def test_dit_time_sin_is_host_code_matching_the_restatement():
    """gsvcu_dit_time_sin (the DiT's sinusoidal time input, `gsv_dit::time_sin` at src/gsv_dit.cpp:754-768,
    host code in both) runs without a GPU; it equals the restatement's formula to float rounding."""
    import dit_oracle as O
    lib = gsvcu.load_library()
    out = np.zeros(256, np.float32)
    for t in (0.0, 0.03125, 0.5, 0.96875, 1.0):
        lib.gsvcu_dit_time_sin(C.c_float(t), out.ctypes.data_as(C.c_void_p))
        assert np.allclose(out, O.time_sin(t), rtol=0, atol=2e-4), t
    lib.gsvcu_dit_time_sin(C.c_float(0.25), None)   # a null output is ignored


def test_bench_weight_bytes_per_format(tmp_path):
    """bench.py's per-format weight bytes per decode step equal the GGUF bytes of the matrices the step reads
    (24 layers of attention / FFN matrices, their F32 biases and LayerNorms, the predict matrix)."""
    import importlib.util
    import gguf
    import gsv_synth as S
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    for name, (kw, nbytes, _) in bench.FORMATS.items():
        path = S.write_model(str(tmp_path / f"{name}.gguf"), seed=1, dims=S.Dims(NL=1), **kw)
        t = {x.name: int(x.n_bytes) for x in gguf.GGUFReader(path).tensors}
        layer = sum(v for k, v in t.items() if k.startswith("transformer.block0."))
        assert 24 * layer + t["ar.predict"] == nbytes, name
