"""Shared test setup: paths, the `gpu` marker, synthetic models.

CPU tests (`-m "not gpu"`) cover the oracle against golden vectors, host logic and the C ABI
surface. GPU tests (`-m gpu`) compare the CUDA library with the oracle through the C ABI.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "gsv.cpp_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_CACHE = os.environ.get("GSVCU_MODEL_CACHE", "/tmp/gsvcu_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def model_small():
    """2-layer synthetic Q8_0 model (fast oracle)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=11, n_layer=2)


@pytest.fixture(scope="session")
def model_full():
    """Full 24-layer synthetic Q8_0 model (BASELINE dims)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=0, n_layer=24)


@pytest.fixture(scope="session")
def model_f32_small():
    """2-layer model whose attention/FFN matrices are F32 (no activation quantization)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=5, n_layer=2, mat_type="f32")


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-30))


def gguf_retyped_copy(src, dst, retype):
    """Rewrite a GGUF file with tensor `name` stored as ggml type retype[name] (its values converted
    through float32: exact when widening to F32)."""
    import gguf
    F32, F16 = gguf.GGMLQuantizationType.F32, gguf.GGMLQuantizationType.F16
    rd = gguf.GGUFReader(src)
    w = gguf.GGUFWriter(dst, str(rd.fields["general.architecture"].contents()))
    for f in rd.fields.values():
        if f.name.startswith("ar."):
            if f.types[0] == gguf.GGUFValueType.UINT32:
                w.add_uint32(f.name, int(f.contents()))
            else:
                w.add_float32(f.name, float(f.contents()))
    for t in rd.tensors:
        data = np.array(t.data)
        if t.name in retype:
            arr, ty = gguf.quants.dequantize(data, t.tensor_type).astype(np.float32), retype[t.name]
            if ty == F32:
                w.add_tensor(t.name, arr, raw_dtype=F32)
            elif ty == F16:
                w.add_tensor(t.name, arr.astype(np.float16), raw_dtype=F16)
            else:
                try:
                    w.add_tensor(t.name, gguf.quants.quantize(arr, ty), raw_dtype=ty)
                except NotImplementedError:   # no gguf-py quantizer (K-quants): all-zero blocks
                    bs, ts = gguf.GGML_QUANT_SIZES[ty]
                    w.add_tensor(t.name, np.zeros((arr.shape[0], arr.shape[1] // bs * ts), np.uint8), raw_dtype=ty)
        else:
            w.add_tensor(t.name, data, raw_dtype=t.tensor_type)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return dst
