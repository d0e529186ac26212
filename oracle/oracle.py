"""ctypes binding of the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / --impl reference leg import
this module. It checks the CUDA library; it is never a fallback for it.

Model weights are read from a GGUF file with gguf-py (the reader of the reference exporter's
ecosystem, tools/export_gguf/convert_ar.py) and handed to the C++ restatement as raw tensor bytes,
so the oracle and the CUDA library consume identical bytes.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_SAMPLER_PATH = os.path.join(HERE, "_ref", "libgsv_sampler_ref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def _load():
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"oracle library missing: {LIB_PATH} (run `make -C oracle`)")
    lib = C.CDLL(LIB_PATH)
    lib.orc_set_threads.argtypes = [C.c_int]
    lib.orc_get_threads.restype = C.c_int
    lib.orc_fp32_to_fp16.argtypes = [_f32p, _u16p, C.c_int64]
    lib.orc_fp16_to_fp32.argtypes = [_u16p, _f32p, C.c_int64]
    lib.orc_quantize_q8_0.argtypes = [_f32p, C.c_int64, _u8p]
    lib.orc_mul_mat.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, _f32p, C.c_int64, _f32p, C.c_int]
    lib.orc_mul_mat.restype = C.c_int
    lib.orc_ln_affine.argtypes = [_f32p, C.c_void_p, C.c_void_p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_float, _f32p]
    lib.orc_add_act.argtypes = [_f32p, _f32p, C.c_int64, C.c_int64, C.c_int, _f32p]
    lib.orc_decode_attention.argtypes = [_f32p, _f32p, _f32p, _i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _f32p]
    lib.orc_prefill_attention.argtypes = [_f32p, _i32p, _i32p, C.c_int, C.c_int, C.c_int, C.c_float, _f32p]
    lib.orc_logits_to_probs.argtypes = [C.c_int, C.c_float, C.c_float, C.c_float, _f32p, C.c_int, C.c_void_p, C.c_int, _f32p]
    lib.orc_rng_init.argtypes = [C.c_uint64]
    lib.orc_rng_init.restype = C.c_uint64
    lib.orc_sample.argtypes = [_f32p, C.c_int, C.POINTER(C.c_uint64)]
    lib.orc_sample.restype = C.c_int
    lib.orc_model_new.argtypes = [C.c_int] * 7
    lib.orc_model_new.restype = C.c_void_p
    lib.orc_model_free.argtypes = [C.c_void_p]
    lib.orc_model_error.argtypes = [C.c_void_p]
    lib.orc_model_error.restype = C.c_char_p
    lib.orc_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
    lib.orc_model_set.restype = C.c_int
    lib.orc_model_finalize.argtypes = [C.c_void_p, C.c_int]
    lib.orc_model_finalize.restype = C.c_int
    lib.orc_bert_new.argtypes = [C.c_int] * 6 + [C.c_float]
    lib.orc_bert_new.restype = C.c_void_p
    lib.orc_bert_free.argtypes = [C.c_void_p]
    lib.orc_bert_error.argtypes = [C.c_void_p]
    lib.orc_bert_error.restype = C.c_char_p
    lib.orc_bert_set.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
    lib.orc_bert_set.restype = C.c_int
    lib.orc_bert_finalize.argtypes = [C.c_void_p]
    lib.orc_bert_finalize.restype = C.c_int
    lib.orc_bert_run.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _f32p]
    lib.orc_bert_run.restype = C.c_int
    lib.orc_model_pe.argtypes = [C.c_void_p]
    lib.orc_model_pe.restype = C.POINTER(C.c_float)
    req = [C.c_void_p, C.c_int, _i32p, _i32p, _f32p, _i32p, _i32p]
    lib.orc_first_logits.argtypes = req + [C.c_int, _f32p, C.c_void_p]
    lib.orc_first_logits.restype = C.c_int
    lib.orc_decode_trace.argtypes = req + [C.c_int, _i32p, C.c_int, _f32p, C.c_void_p]
    lib.orc_decode_trace.restype = C.c_int
    lib.orc_generate.argtypes = req + [C.c_int, C.c_float, C.c_float, C.c_float, C.c_uint64, C.c_int, C.c_int,
                                       C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, _i32p, _i32p, _i32p,
                                       C.c_int, C.c_void_p]
    lib.orc_generate.restype = C.c_int
    lib.orc_last_generate_seconds.argtypes = [C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_int)]
    lib.orc_last_generate_seconds.restype = None
    lib.orc_serve_new.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
    lib.orc_serve_new.restype = C.c_void_p
    lib.orc_serve_free.argtypes = [C.c_void_p]
    lib.orc_serve_admit.argtypes = [C.c_void_p, C.c_int, _i32p, _i32p, _f32p, _i32p, _i32p, C.c_void_p, C.c_void_p,
                                    C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float]
    lib.orc_serve_admit.restype = C.c_int
    lib.orc_serve_step.argtypes = [C.c_void_p, C.c_int, _i32p, C.c_int, C.c_void_p, C.c_int]
    lib.orc_serve_step.restype = C.c_int
    lib.orc_serve_tokens_total.argtypes = [C.c_void_p]
    lib.orc_serve_tokens_total.restype = C.c_int64
    lib.orc_serve_reset.argtypes = [C.c_void_p]
    lib.orc_serve_active.argtypes = [C.c_void_p]
    lib.orc_serve_active.restype = C.c_int
    lib.orc_serve_seconds.argtypes = [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_int64)]
    lib.orc_serve_seconds.restype = None
    return lib


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        _LIB = _load()
    return _LIB


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return int(lib().orc_get_threads())


# ------------------------------------------------------------------ primitive ops
def fp32_to_fp16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    y = np.empty(x.size, np.uint16)
    lib().orc_fp32_to_fp16(x, y, x.size)
    return y


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Raw Q8_0 blocks (34 bytes per 32 values) of a float array whose size is a multiple of 32."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().orc_quantize_q8_0(x, x.size, out)
    return out


def mul_mat(w: np.ndarray, wtype: int, N: int, K: int, x: np.ndarray, layer: bool = False) -> np.ndarray:
    """Y[M][N] = W[N][K] . X[M][K]^T with ggml CPU semantics (wtype 8 / 2 / 6 = raw Q8_0 / Q4_0 / Q5_0
    bytes, 0 = F32, 1 = F16). layer: W is a layer matrix, so an F32 W takes the FMA-vectorised order of an
    F16 one."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.size // K
    y = np.empty((M, N), np.float32)
    w = np.ascontiguousarray(w)
    if lib().orc_mul_mat(wtype, w.ctypes.data, N, K, x, M, y, int(layer)):
        raise ValueError("orc_mul_mat failed")
    return y


def ln_affine(x, r, bias, w, b, eps=1e-5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = w.size
    rows = x.size // n
    y = np.empty_like(x)
    rp = np.ascontiguousarray(r, dtype=np.float32) if r is not None else None
    bp = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else None
    lib().orc_ln_affine(x, rp.ctypes.data if rp is not None else None, bp.ctypes.data if bp is not None else None,
                        np.ascontiguousarray(w, np.float32), np.ascontiguousarray(b, np.float32), rows, n, eps, y)
    return y


def add_act(a, b, act=1):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    y = np.empty_like(a)
    lib().orc_add_act(a, b, a.size // b.size, b.size, act, y)
    return y


def decode_attention(q, k, v, lens, scale):
    """q [B][NH][HD]; k/v [B][Lmax][NH][HD]; lens [B] -> out [B][NH][HD] (ggml flash_attn_ext semantics)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    B, NH, HD = q.shape
    out = np.empty_like(q)
    lib().orc_decode_attention(q, k, v, np.ascontiguousarray(lens, np.int32), B, k.shape[1], NH, HD, scale, out)
    return out


def prefill_attention(qkv, seq_len, text_len, NH, HD, scale):
    qkv = np.ascontiguousarray(qkv, np.float32)
    out = np.empty((qkv.shape[0], NH * HD), np.float32)
    lib().orc_prefill_attention(qkv, np.ascontiguousarray(seq_len, np.int32), np.ascontiguousarray(text_len, np.int32),
                                len(seq_len), NH, HD, scale, out)
    return out


def logits_to_probs(logits, top_k=15, top_p=1.0, temperature=1.0, rep=1.35, prev=None):
    lg = np.array(logits, dtype=np.float32, copy=True)
    probs = np.empty_like(lg)
    pv = np.ascontiguousarray(prev, np.int32) if prev is not None and len(prev) else None
    lib().orc_logits_to_probs(top_k, top_p, temperature, rep, lg, lg.size, pv.ctypes.data if pv is not None else None,
                              0 if pv is None else pv.size, probs)
    return probs


def rng_init(seed: int) -> int:
    return int(lib().orc_rng_init(seed))


def sample(probs, state: int):
    st = C.c_uint64(state)
    t = lib().orc_sample(np.ascontiguousarray(probs, np.float32), len(probs), C.byref(st))
    return t, int(st.value)


# ------------------------------------------------------------------ model
@dataclass
class Request:
    """gsv_ar_request (reference src/gsv_ar.h:13-17): phones, bert [1024][T] row-major, prompt codes."""
    phones: np.ndarray
    bert: np.ndarray
    prompt: np.ndarray


def pack_requests(reqs, bert_dim=1024):
    phones = np.ascontiguousarray(np.concatenate([np.asarray(r.phones, np.int32) for r in reqs]), np.int32)
    n_ph = np.array([len(r.phones) for r in reqs], np.int32)
    bert = np.ascontiguousarray(np.concatenate([np.asarray(r.bert, np.float32).reshape(bert_dim, len(r.phones)).ravel()
                                                for r in reqs]), np.float32)
    prompts = np.ascontiguousarray(np.concatenate([np.asarray(r.prompt, np.int32) for r in reqs]
                                                  + [np.zeros(0, np.int32)]), np.int32)
    n_pr = np.array([len(r.prompt) for r in reqs], np.int32)
    return phones, n_ph, bert, prompts, n_pr


class BertOracle:
    """CPU restatement of gsv_bert (reference src/gsv_bert.{h,cpp}) over a GGUF file of
    tools/export_gguf/convert_bert.py."""

    def __init__(self, gguf_path: str):
        import gguf  # gguf-py

        rd = gguf.GGUFReader(gguf_path)

        def kv(key, default, cast=int):
            f = rd.fields.get(key)
            return default if f is None else cast(f.parts[f.data[0]][0])

        self.D = kv("bert.hidden", 1024)
        self.NH = kv("bert.head", 16)
        self.FF = kv("bert.inter", 4096)
        self.NL = kv("bert.layers_used", 22)
        self.VOCAB = kv("bert.vocab", 21128)
        self.MAXPOS = kv("bert.max_pos", 512)
        self.EPS = kv("bert.ln_eps", 1e-12, float)
        L = lib()
        self._m = L.orc_bert_new(self.D, self.NH, self.FF, self.NL, self.VOCAB, self.MAXPOS, self.EPS)
        for t in rd.tensors:
            data = np.ascontiguousarray(t.data)
            if L.orc_bert_set(self._m, t.name.encode(), int(t.tensor_type), data.ctypes.data, data.nbytes) < 0:
                raise ValueError(L.orc_bert_error(self._m).decode())
        if L.orc_bert_finalize(self._m) != 0:
            raise ValueError(L.orc_bert_error(self._m).decode())

    def __del__(self):
        if getattr(self, "_m", None) and _LIB is not None:
            _LIB.orc_bert_free(self._m)
            self._m = None

    def encode(self, ids, n_layers=-1) -> np.ndarray:
        """gsv_bert::encode (n_layers < 0) / encode_layers: features [D][T]."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((self.D, ids.size), np.float32)
        if lib().orc_bert_run(self._m, ids, ids.size, n_layers, out):
            raise ValueError(lib().orc_bert_error(self._m).decode())
        return out

    def encode_feat(self, ids) -> np.ndarray:
        """gsv_bert::encode_feat: features without [CLS] / [SEP], [D][T-2]."""
        return self.encode(ids)[:, 1:-1].copy()

    def encode_layers(self, ids):
        """gsv_bert::encode_layers: (features, per_layer) with per_layer[0] the embedding LayerNorm output
        and per_layer[k] the output of layer k-1, layers_used + 1 entries."""
        per_layer = [self.encode(ids, n_layers=k) for k in range(self.NL + 1)]
        return per_layer[-1], per_layer

    def encode_feat_batch(self, ids_flat, lens, tmax):
        """gsv_bert::encode_feat_batch (src/gsv_bert.cpp:271-311): B sequences of lens[b] tokens in slots of
        tmax. The reference runs them as one block-diagonally masked sequence; here each row's dot and each
        masked attention row do not depend on the batch, so this equals encode_feat per sequence."""
        ids_flat = np.asarray(ids_flat, np.int32)
        if tmax < 3 or tmax > self.MAXPOS or len(lens) == 0 or ids_flat.size < len(lens) * tmax:
            raise ValueError("encode_feat_batch: bad args")
        return [self.encode_feat(ids_flat[b * tmax: b * tmax + lens[b]]) if lens[b] > 2 else
                np.zeros((self.D, 0), np.float32) for b in range(len(lens))]


class OracleModel:
    """CPU restatement of gsv_ar (reference src/gsv_ar.{h,cpp}) over a GGUF file."""

    def __init__(self, gguf_path: str, pe_max: int = 8192):
        import gguf  # gguf-py

        rd = gguf.GGUFReader(gguf_path)

        def kv(key, default):
            f = rd.fields.get(key)
            if f is None:
                return default
            return int(f.parts[f.data[0]][0])

        self.D = kv("ar.hidden_dim", 512)
        self.NH = kv("ar.head", 16)
        self.NL = kv("ar.n_layer", 24)
        self.V = kv("ar.vocab_size", 1025)
        self.PV = kv("ar.phoneme_vocab_size", 732)
        self.EOS = kv("ar.eos", 1024)
        self.BERT = 1024
        self.HD = self.D // self.NH
        L = lib()
        self._m = L.orc_model_new(self.D, self.NH, self.NL, self.V, self.PV, self.EOS, self.BERT)
        for t in rd.tensors:
            data = np.ascontiguousarray(t.data)
            if L.orc_model_set(self._m, t.name.encode(), int(t.tensor_type), data.ctypes.data, data.nbytes) < 0:
                raise ValueError(L.orc_model_error(self._m).decode())
        if L.orc_model_finalize(self._m, pe_max) != 0:
            raise ValueError(L.orc_model_error(self._m).decode())
        self.pe_max = pe_max

    def __del__(self):
        if getattr(self, "_m", None) and _LIB is not None:
            _LIB.orc_model_free(self._m)
            self._m = None

    def pe(self) -> np.ndarray:
        p = lib().orc_model_pe(self._m)
        return np.ctypeslib.as_array(p, shape=(self.pe_max, self.D)).copy()

    def _err(self):
        return ValueError(lib().orc_model_error(self._m).decode())

    def first_logits(self, reqs, kv_f16=False, dump=False):
        ph, nph, bert, pr, npr = pack_requests(reqs, self.BERT)
        B = len(reqs)
        out = np.empty((B, self.V), np.float32)
        d = np.empty((B, self.NL, 4, self.D), np.float32) if dump else None
        if lib().orc_first_logits(self._m, B, ph, nph, bert, pr, npr, int(kv_f16), out,
                                  d.ctypes.data if d is not None else None):
            raise self._err()
        return (out, d) if dump else out

    def decode_trace(self, reqs, forced, kv_f16=False, dump=False):
        """Teacher-forced trace: logits [n+1][B][V] (row 0 = prefill), optional dumps [n][B][NL][4][D]."""
        ph, nph, bert, pr, npr = pack_requests(reqs, self.BERT)
        B = len(reqs)
        forced = np.ascontiguousarray(forced, np.int32).reshape(B, -1)
        n = forced.shape[1]
        out = np.empty((n + 1, B, self.V), np.float32)
        d = np.empty((n, B, self.NL, 4, self.D), np.float32) if dump else None
        if lib().orc_decode_trace(self._m, B, ph, nph, bert, pr, npr, int(kv_f16), forced, n, out,
                                  d.ctypes.data if d is not None else None):
            raise self._err()
        return (out, d) if dump else out

    def generate(self, reqs, top_k=15, top_p=1.0, temperature=1.0, rep=1.35, seed_base=1, early_stop=-1,
                 max_steps=1500, oracle_tokens=None, seeds=None, kv_f16=False, with_first_logits=False):
        """gsv_ar::generate semantics. Returns (tokens list per seq, lens in finish order)."""
        ph, nph, bert, pr, npr = pack_requests(reqs, self.BERT)
        B = len(reqs)
        cap = int(max(npr)) + max_steps + 1
        toks = np.zeros((B, cap), np.int32)
        ntok = np.zeros(B, np.int32)
        lens = np.zeros(B, np.int32)
        ot = np.ascontiguousarray(oracle_tokens, np.int32) if oracle_tokens is not None else None
        sd = np.ascontiguousarray(seeds, np.uint64) if seeds is not None else None
        fl = np.empty((B, self.V), np.float32) if with_first_logits else None
        if lib().orc_generate(self._m, B, ph, nph, bert, pr, npr, top_k, top_p, temperature, rep, seed_base,
                              early_stop, max_steps, ot.ctypes.data if ot is not None else None,
                              0 if ot is None else ot.size, sd.ctypes.data if sd is not None else None,
                              0 if sd is None else sd.size, int(kv_f16), toks, ntok, lens, cap,
                              fl.ctypes.data if fl is not None else None):
            raise self._err()
        out = [toks[b, :ntok[b]].copy() for b in range(B)]
        if with_first_logits:
            return out, lens.tolist(), fl
        return out, lens.tolist()


class OracleServer:
    """CPU restatement of the continuous-batching entry (gsvcu_serve_*; the role of svc::ArBatcher,
    reference tools/svc_core.h:1244-1340): `slots` sequence slots over one OracleModel; every admitted
    sequence decodes exactly as OracleModel.generate of that sequence alone."""

    def __init__(self, model: "OracleModel", slots: int, max_ctx: int, kv_f16: bool = False):
        self.model = model
        self.slots = slots
        self._s = lib().orc_serve_new(model._m, slots, max_ctx, int(kv_f16))
        if not self._s:
            raise ValueError("orc_serve_new failed")

    def close(self):
        if getattr(self, "_s", None) and _LIB is not None:
            _LIB.orc_serve_free(self._s)
            self._s = None

    __del__ = close

    def admit(self, reqs, seeds, tags=None, max_steps=1500, early_stop=-1, top_k=15, top_p=1.0, temperature=1.0,
              rep=1.35):
        ph, nph, bert, pr, npr = pack_requests(reqs, self.model.BERT)
        sd = np.ascontiguousarray(seeds, np.uint64)
        tg = np.ascontiguousarray(tags if tags is not None else range(len(reqs)), np.int32)
        if lib().orc_serve_admit(self._s, len(reqs), ph, nph, bert, pr, npr, sd.ctypes.data, tg.ctypes.data,
                                 max_steps, early_stop, top_k, top_p, temperature, rep):
            raise self.model._err()

    def step(self, n_steps, max_done=None, tok_cap=0):
        """Run n_steps iterations; returns the finished sequences as dicts (slot, tag, finish_kind,
        n_generated, tokens)."""
        max_done = self.slots if max_done is None else max_done
        done = np.zeros((max(max_done, 1), 5), np.int32)
        toks = np.zeros(max(tok_cap, 1), np.int32) if tok_cap else None
        nd = lib().orc_serve_step(self._s, n_steps, done, max_done, toks.ctypes.data if toks is not None else None,
                                  tok_cap)
        out, at = [], 0
        for i in range(nd):
            k = int(done[i, 4])
            out.append(dict(slot=int(done[i, 0]), tag=int(done[i, 1]), finish_kind=int(done[i, 2]),
                            n_generated=int(done[i, 3]), tokens=toks[at:at + k].copy() if toks is not None else None))
            at += k
        return out

    def tokens_total(self) -> int:
        return int(lib().orc_serve_tokens_total(self._s))

    def active(self) -> int:
        return int(lib().orc_serve_active(self._s))

    def reset(self):
        lib().orc_serve_reset(self._s)

    def seconds(self):
        """(prefill seconds, decode seconds, decoded rows) since creation."""
        p, d, n = C.c_double(), C.c_double(), C.c_int64()
        lib().orc_serve_seconds(self._s, C.byref(p), C.byref(d), C.byref(n))
        return p.value, d.value, n.value


def last_generate_seconds():
    """(prefill seconds, decode seconds, decode steps) of the last OracleModel.generate on this thread."""
    p, d, n = C.c_double(), C.c_double(), C.c_int()
    lib().orc_last_generate_seconds(C.byref(p), C.byref(d), C.byref(n))
    return p.value, d.value, n.value


# ------------------------------------------------------------------ the reference's own sampler
class RefSampler:
    """The reference's src/gsv_sampler.cpp, compiled in place into oracle/_ref/ (see oracle/Makefile)."""

    def __init__(self):
        if not os.path.exists(REF_SAMPLER_PATH):
            raise RuntimeError(f"reference sampler not built: {REF_SAMPLER_PATH}")
        self.lib = C.CDLL(REF_SAMPLER_PATH)
        self.lib.ref_logits_to_probs.argtypes = [C.c_int, C.c_float, C.c_float, C.c_float, _f32p, C.c_int, C.c_void_p,
                                                 C.c_int, _f32p]
        self.lib.ref_rng_init.argtypes = [C.c_uint64]
        self.lib.ref_rng_init.restype = C.c_uint64
        self.lib.ref_sample.argtypes = [_f32p, C.c_int, C.POINTER(C.c_uint64)]
        self.lib.ref_sample.restype = C.c_int

    def logits_to_probs(self, logits, top_k=15, top_p=1.0, temperature=1.0, rep=1.35, prev=None):
        lg = np.array(logits, dtype=np.float32, copy=True)
        probs = np.empty_like(lg)
        pv = np.ascontiguousarray(prev, np.int32) if prev is not None and len(prev) else None
        self.lib.ref_logits_to_probs(top_k, top_p, temperature, rep, lg, lg.size,
                                     pv.ctypes.data if pv is not None else None, 0 if pv is None else pv.size, probs)
        return probs

    def rng_init(self, seed):
        return int(self.lib.ref_rng_init(seed))

    def sample(self, probs, state):
        st = C.c_uint64(state)
        t = self.lib.ref_sample(np.ascontiguousarray(probs, np.float32), len(probs), C.byref(st))
        return t, int(st.value)
