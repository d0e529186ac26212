"""ctypes binding of libgsvcu.so (include/gsvcu.h), the B200 library of the AR hot path.

The Python-side counterpart of the C++ drop-in (csrc/gsv_ar.cpp): it calls the same C ABI entry
points with plain pointers and sizes. The library must have been built in-tree
(`make -C gsv.cpp_b200`); there is no fallback of any kind when it is missing.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libgsvcu.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "gsvcu.h")

OK = 0
ERR = {-1: "ARG", -2: "CUDA", -3: "OOM", -4: "IO", -5: "FORMAT", -6: "STATE", -7: "DEVICE"}
KV_F16, KV_F32 = 0, 1
EPI_BIAS, EPI_RESID, EPI_RELU_Q8 = 0, 1, 2


class GsvcuError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"gsvcu error {code} ({ERR.get(code, '?')}): {msg}")
        self.code = code


class Request(C.Structure):
    _fields_ = [("phones", C.POINTER(C.c_int32)), ("n_phones", C.c_int32), ("bert", C.POINTER(C.c_float)),
                ("prompt", C.POINTER(C.c_int32)), ("n_prompt", C.c_int32)]


class SamplerCfg(C.Structure):
    _fields_ = [("top_k", C.c_int32), ("top_p", C.c_float), ("temperature", C.c_float),
                ("repetition_penalty", C.c_float)]


class HParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden_dim", "n_head", "head_dim", "n_layer", "vocab_size",
                                           "phoneme_vocab_size", "eos", "bert_dim", "ffn_dim")] + \
               [("text_pe_alpha", C.c_float), ("audio_pe_alpha", C.c_float)]


class Finished(C.Structure):
    _fields_ = [("slot", C.c_int32), ("tag", C.c_int32), ("finish_kind", C.c_int32), ("n_generated", C.c_int32),
                ("n_tokens", C.c_int32)]


PROGRESS_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int32)

_P, _I, _U64 = C.c_void_p, C.c_int32, C.c_uint64
# exported C entry points and their ctypes signatures
SIGNATURES = {
    "gsvcu_create": ([C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "gsvcu_destroy": ([_P], None),
    "gsvcu_last_error": ([_P], C.c_char_p),
    "gsvcu_load_gguf": ([_P, C.c_char_p], C.c_int),
    "gsvcu_get_hparams": ([_P, C.POINTER(HParams)], C.c_int),
    "gsvcu_kv_reserve": ([_P, _I, _I, _I], C.c_int),
    "gsvcu_release_cache": ([_P], C.c_int),
    "gsvcu_inspect_gguf": ([C.c_char_p, C.POINTER(HParams), C.c_char_p, _I], C.c_int),
    "gsvcu_first_logits": ([_P, C.POINTER(Request), _I, _P], C.c_int),
    "gsvcu_generate": ([_P, C.POINTER(Request), _I, C.POINTER(SamplerCfg), _U64, _I, _I, _P, _I, _P, _I, _P, _P, _P,
                        _I, PROGRESS_FN, _P], C.c_int),
    "gsvcu_debug_trace": ([_P, C.POINTER(Request), _I, _P, _I, _P, _P], C.c_int),
    "gsvcu_serve_admit": ([_P, C.POINTER(Request), _I, C.POINTER(SamplerCfg), _P, _P, _I, _I], C.c_int),
    "gsvcu_serve_step": ([_P, _I, C.POINTER(Finished), _I, _P, _I], C.c_int),
    "gsvcu_serve_active": ([_P], C.c_int),
    "gsvcu_serve_tokens_total": ([_P], C.c_int64),
    "gsvcu_op_quantize_q8_0": ([_P, _P, _I, _I, _P, _P], C.c_int),
    "gsvcu_op_pack_q8_0": ([_P, _P, _I, _I, _P, _P], C.c_int),
    "gsvcu_op_q8_gemm": ([_P, _P, _P, _I, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P], C.c_int),
    "gsvcu_op_layernorm_q8": ([_P, _P, _I, _P, _P, _P, _P, _P], C.c_int),
    "gsvcu_op_f32_gemm": ([_P, _P, _I, _P, _I, _I, _P, _P], C.c_int),
    "gsvcu_op_fx_gemm": ([_P, _P, _I, _P, _I, _I, _I, _P, _P], C.c_int),
    "gsvcu_op_decode_attention": ([_P, _P, _I, _P, _I, _I, _I, _P, _I, _P, _P, _I, _P, _P, _P], C.c_int),
    "gsvcu_op_prefill_attention": ([_P, _P, _I, _P, _P, _P, _P, _P, _P], C.c_int),
    "gsvcu_op_sample": ([_P, _P, _I, _I, _I, C.POINTER(SamplerCfg), _P, _P, _I, _P, _P, _P], C.c_int),
    "gsvcu_sync": ([_P], C.c_int),
    "gsvcu_serve_reset": ([_P], C.c_int),
    "gsvcu_step_profile": ([_P, _I, _P, _P], C.c_int),
    "gsvcu_kernel_launches": ([_P], C.c_int64),
    "gsvcu_stream": ([_P], C.c_void_p),
    "gsvcu_op_decode_attention_noalloc": ([_P, _P, _I, _P, _I, _I, _I, _P, _I, _P, _P, _I, _P, _P, _P], C.c_int),
    "gsvcu_set_fused_decode": ([_P, _I], C.c_int),
    "gsvcu_set_serve_lookahead": ([_P, _I], C.c_int),
    "gsvcu_fused_decode": ([_P], C.c_int),
    "gsvcu_set_wait_fault": ([_P, _I], C.c_int),
    "gsvcu_set_prefill_gemm": ([_P, _I], C.c_int),
    "gsvcu_op_q8_gemm_tc": ([_P, _P, _P, _I, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P], C.c_int),
    "gsvcu_op_pack_q8_0_f16": ([_P, _P, _I, _I, _P], C.c_int),
}

class BertHParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "n_head", "inter", "layers_used", "vocab", "max_pos")] + \
               [("ln_eps", C.c_float)]


SIGNATURES.update({
    "gsvcu_bert_load": ([C.c_int, C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "gsvcu_bert_destroy": ([_P], None),
    "gsvcu_bert_last_error": ([_P], C.c_char_p),
    "gsvcu_bert_get_hparams": ([_P, C.POINTER(BertHParams)], C.c_int),
    "gsvcu_bert_encode": ([_P, _P, _I, _I, _P], C.c_int),
    "gsvcu_bert_encode_feat_batch": ([_P, _I, _P, _P, _I, _P, _I], C.c_int),
})

class DitHParams(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("dim", "depth", "heads", "dim_head", "ff_mult", "mel_dim", "text_dim")]


SIGNATURES.update({
    "gsvcu_dit_load": ([C.c_int, C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "gsvcu_dit_destroy": ([_P], None),
    "gsvcu_dit_last_error": ([_P], C.c_char_p),
    "gsvcu_dit_get_hparams": ([_P, C.POINTER(DitHParams)], C.c_int),
    "gsvcu_dit_set_condition": ([_P, _P, _P, _I, _I], C.c_int),
    "gsvcu_dit_velocity": ([_P, _P, C.c_float, _I, _P], C.c_int),
    "gsvcu_dit_sample": ([_P, _P, _I, _I, C.c_float, _I, _P], C.c_int),
    "gsvcu_dit_op_hidden": ([_P, _P, C.c_float, _I, _P], C.c_int),
    "gsvcu_dit_stream": ([_P, C.POINTER(C.c_void_p)], C.c_int),
    "gsvcu_dit_prepare": ([_P, _P, _P, _I, _I], C.c_int),
    "gsvcu_dit_sample_full": ([_P, _P, _P, _I, _I, _I, C.c_float, C.c_uint64, _P, _I, _P], C.c_int),
    "gsvcu_dit_op_condition": ([_P, _P], C.c_int),
    "gsvcu_dit_set_alg": ([_P, _I], C.c_int),
    "gsvcu_dit_set_dbcache": ([_P, _I, C.c_float, _I, _I, _I, _I, C.c_float, _I], C.c_int),
    "gsvcu_dit_db_set_step": ([_P, _I], C.c_int),
    "gsvcu_dit_db_get_stats": ([_P, _P, _P, _P, _P, _P], C.c_int),
    "gsvcu_dit_get_alg": ([_P, C.POINTER(C.c_int32)], C.c_int),
    "gsvcu_dit_synthesize": ([_P, _P, _I, _P, _I, _P, _I, _I, C.c_float, C.c_uint64, _I, _P, _I, _I, _P], C.c_int),
    "gsvcu_dit_time_sin": ([C.c_float, _P], None),
    "gsvcu_dit_get_inv_freq": ([_P, _P], C.c_int),
})

PROF_CLASSES = ["sampler", "step_prep", "qkv_gemm", "decode_attn", "out_gemm", "layernorm", "ffn1_gemm", "ffn2_gemm",
                "predict", "dense_fused"]

_LIB = None


def load_library(path: str = LIB_PATH):
    """Load libgsvcu.so and bind every entry point; raises if the library or a symbol is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"libgsvcu.so not built at {path} (run `make -C gsv.cpp_b200`)")
    lib = C.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _LIB = lib
    return lib


def declared_symbols(header: str = HEADER):
    """Function names declared in include/gsvcu.h."""
    txt = open(header).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(gsvcu_[a-z0-9_]+)\s*\(", txt)))


def inspect_gguf(path: str):
    """Validate an AR GGUF on the host (no GPU needed). Returns (code, hparams or None, message)."""
    lib = load_library()
    hp = HParams()
    err = C.create_string_buffer(512)
    rc = lib.gsvcu_inspect_gguf(path.encode(), C.byref(hp), err, 512)
    return rc, (hp if rc == OK else None), err.value.decode(errors="replace")


def _ptr(a):
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


class _Reqs:
    """Keeps numpy buffers alive while the C array of gsvcu_request points into them."""

    def __init__(self, reqs, bert_dim=1024):
        self.keep = []
        arr = (Request * len(reqs))()
        for i, r in enumerate(reqs):
            ph = np.ascontiguousarray(r.phones, np.int32)
            pr = np.ascontiguousarray(r.prompt, np.int32)
            if hasattr(r.bert, "data_ptr"):      # device tensor (float32, contiguous, on the context's GPU)
                be = r.bert
                if be.numel() != bert_dim * ph.size or not be.is_contiguous():
                    raise ValueError("bert must hold bert_dim x n_phones contiguous values")
                bptr = C.cast(C.c_void_p(be.data_ptr()), C.POINTER(C.c_float))
            else:
                be = np.ascontiguousarray(r.bert, np.float32).reshape(-1)
                if be.size != bert_dim * ph.size:
                    raise ValueError("bert must hold bert_dim x n_phones values")
                bptr = be.ctypes.data_as(C.POINTER(C.c_float))
            self.keep += [ph, be, pr]
            arr[i].phones = ph.ctypes.data_as(C.POINTER(C.c_int32))
            arr[i].n_phones = ph.size
            arr[i].bert = bptr
            arr[i].prompt = pr.ctypes.data_as(C.POINTER(C.c_int32)) if pr.size else None
            arr[i].n_prompt = pr.size
        self.arr = arr
        self.n = len(reqs)


class Context:
    """One gsvcu context (one CUDA device, one stream)."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        h = C.c_void_p()
        rc = self.lib.gsvcu_create(device, C.byref(h))
        if rc != OK:
            raise GsvcuError(rc, f"cannot open CUDA device {device} (needs an sm_100 GPU)")
        self.h = h
        self.hp = None

    def close(self):
        if getattr(self, "h", None):
            self.lib.gsvcu_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != OK:
            raise GsvcuError(rc, self.lib.gsvcu_last_error(self.h).decode(errors="replace"))
        return rc

    def load(self, path: str):
        self._check(self.lib.gsvcu_load_gguf(self.h, path.encode()))
        hp = HParams()
        self._check(self.lib.gsvcu_get_hparams(self.h, C.byref(hp)))
        self.hp = hp
        return hp

    def kv_reserve(self, max_slots: int, max_ctx: int, kv_dtype: int = KV_F16):
        self._check(self.lib.gsvcu_kv_reserve(self.h, max_slots, max_ctx, kv_dtype))

    def release_cache(self):
        self._check(self.lib.gsvcu_release_cache(self.h))

    def sync(self):
        self._check(self.lib.gsvcu_sync(self.h))

    def first_logits(self, reqs):
        r = _Reqs(reqs)
        out = np.empty((r.n, self.hp.vocab_size), np.float32)
        self._check(self.lib.gsvcu_first_logits(self.h, r.arr, r.n, _ptr(out)))
        return out

    def generate(self, reqs, top_k=15, top_p=1.0, temperature=1.0, rep=1.35, seed_base=1, early_stop=-1,
                 max_steps=1500, oracle_tokens=None, seeds=None, progress=None):
        r = _Reqs(reqs)
        cap = max(len(x.prompt) for x in reqs) + max_steps
        toks = np.zeros((r.n, cap), np.int32)
        ntok = np.zeros(r.n, np.int32)
        lens = np.zeros(r.n, np.int32)
        sc = SamplerCfg(top_k, top_p, temperature, rep)
        ot = np.ascontiguousarray(oracle_tokens, np.int32) if oracle_tokens is not None else None
        sd = np.ascontiguousarray(seeds, np.uint64) if seeds is not None else None
        cb = PROGRESS_FN(lambda u, n: progress(n)) if progress else PROGRESS_FN()
        self._check(self.lib.gsvcu_generate(self.h, r.arr, r.n, C.byref(sc), seed_base, early_stop, max_steps,
                                            _ptr(ot), 0 if ot is None else ot.size, _ptr(sd),
                                            0 if sd is None else sd.size, _ptr(toks), _ptr(ntok), _ptr(lens), cap,
                                            cb, None))
        return [toks[b, :ntok[b]].copy() for b in range(r.n)], lens.tolist()

    def debug_trace(self, reqs, forced, dump=False):
        r = _Reqs(reqs)
        forced = np.ascontiguousarray(forced, np.int32).reshape(r.n, -1)
        n = forced.shape[1]
        V, NL, Dm = self.hp.vocab_size, self.hp.n_layer, self.hp.hidden_dim
        lg = np.empty((n + 1, r.n, V), np.float32)
        d = np.zeros((n + 1, r.n, NL, 4, Dm), np.float32) if dump else None
        self._check(self.lib.gsvcu_debug_trace(self.h, r.arr, r.n, _ptr(forced), n, _ptr(lg), _ptr(d)))
        return (lg, d) if dump else lg

    # continuous batching
    def serve_admit(self, reqs, seeds, tags, max_steps, early_stop=-1, top_k=15, top_p=1.0, temperature=1.0,
                    rep=1.35):
        r = _Reqs(reqs)
        sd = np.ascontiguousarray(seeds, np.uint64)
        tg = np.ascontiguousarray(tags, np.int32)
        sc = SamplerCfg(top_k, top_p, temperature, rep)
        self._check(self.lib.gsvcu_serve_admit(self.h, r.arr, r.n, C.byref(sc), _ptr(sd), _ptr(tg), max_steps,
                                               early_stop))

    def serve_step(self, n_steps, max_done=4096, tok_cap=0):
        done = (Finished * max_done)()
        toks = np.zeros(max(tok_cap, 1), np.int32)
        n = self.lib.gsvcu_serve_step(self.h, n_steps, done, max_done, _ptr(toks) if tok_cap else None, tok_cap)
        if n < 0:
            self._check(n)
        out, at = [], 0
        for i in range(n):
            f = done[i]
            out.append(dict(slot=f.slot, tag=f.tag, finish_kind=f.finish_kind, n_generated=f.n_generated,
                            tokens=toks[at:at + f.n_tokens].copy()))
            at += f.n_tokens
        return out

    def serve_reset(self):
        self._check(self.lib.gsvcu_serve_reset(self.h))

    def step_profile(self, n_steps):
        ms = np.zeros(len(PROF_CLASSES), np.float32)
        by = C.c_int64(0)
        self._check(self.lib.gsvcu_step_profile(self.h, n_steps, _ptr(ms), C.byref(by)))
        return dict(zip(PROF_CLASSES, ms.tolist())), int(by.value)

    def kernel_launches(self):
        return int(self.lib.gsvcu_kernel_launches(self.h))

    def set_serve_lookahead(self, on):
        self._check(self.lib.gsvcu_set_serve_lookahead(self.h, 1 if on else 0))

    def set_fused_decode(self, mode):
        """mode: 0 unfused, 1 fused one group, 2 fused two slot groups (True -> 2, False -> 0)."""
        mode = 2 if mode is True else 0 if mode is False else int(mode)
        self._check(self.lib.gsvcu_set_fused_decode(self.h, mode))

    def fused_decode(self):
        return int(self.lib.gsvcu_fused_decode(self.h))

    def set_prefill_gemm(self, mode):
        """1: prefill Q8_0 GEMMs on tcgen05 (default); 0: on mma.sync tiles (gsvcu_set_prefill_gemm)."""
        self._check(self.lib.gsvcu_set_prefill_gemm(self.h, int(mode)))

    def set_wait_fault(self, on):
        """Test-only: make this context's decode-attention page waits run out (gsvcu_set_wait_fault)."""
        self._check(self.lib.gsvcu_set_wait_fault(self.h, 1 if on else 0))

    def stream_handle(self):
        return int(self.lib.gsvcu_stream(self.h) or 0)

    def serve_active(self):
        return self.lib.gsvcu_serve_active(self.h)

    def serve_tokens_total(self):
        return int(self.lib.gsvcu_serve_tokens_total(self.h))

    # kernel-level entry points (torch CUDA tensors)
    def op_quantize_q8_0(self, x, q, d):
        self._check(self.lib.gsvcu_op_quantize_q8_0(self.h, _ptr(x), x.shape[0], x.shape[1], _ptr(q), _ptr(d)))

    def op_pack_q8_0(self, raw: np.ndarray, N: int, K: int, wq, wd):
        raw = np.ascontiguousarray(raw, np.uint8)
        self._check(self.lib.gsvcu_op_pack_q8_0(self.h, _ptr(raw), N, K, _ptr(wq), _ptr(wd)))

    def op_q8_gemm(self, xq, xd, M, wq, wd, N, K, bias, resid, epi, y=None, yq=None, yd=None):
        self._check(self.lib.gsvcu_op_q8_gemm(self.h, _ptr(xq), _ptr(xd), M, _ptr(wq), _ptr(wd), N, K, _ptr(bias),
                                              _ptr(resid), epi, _ptr(y), _ptr(yq), _ptr(yd)))

    def op_q8_gemm_tc(self, xq, xd, M, w16, wd, N, K, bias, resid, epi, y=None, yq=None, yd=None):
        self._check(self.lib.gsvcu_op_q8_gemm_tc(self.h, _ptr(xq), _ptr(xd), M, _ptr(w16), _ptr(wd), N, K, _ptr(bias),
                                                 _ptr(resid), epi, _ptr(y), _ptr(yq), _ptr(yd)))

    def op_pack_q8_0_f16(self, raw: np.ndarray, N: int, K: int, w16):
        raw = np.ascontiguousarray(raw, np.uint8)
        self._check(self.lib.gsvcu_op_pack_q8_0_f16(self.h, raw.ctypes.data, N, K, _ptr(w16)))

    def op_layernorm_q8(self, v, rows, w, b, y, yq, yd):
        self._check(self.lib.gsvcu_op_layernorm_q8(self.h, _ptr(v), rows, _ptr(w), _ptr(b), _ptr(y), _ptr(yq),
                                                   _ptr(yd)))

    def op_f32_gemm(self, x, M, w, N, K, add, y):
        self._check(self.lib.gsvcu_op_f32_gemm(self.h, _ptr(x), M, _ptr(w), N, K, _ptr(add), _ptr(y)))

    def op_fx_gemm(self, x, M, w, wtype, N, K, bias, y):
        self._check(self.lib.gsvcu_op_fx_gemm(self.h, _ptr(x), M, _ptr(w), wtype, N, K, _ptr(bias), _ptr(y)))

    def op_decode_attention(self, q, q_stride, pool, kv_dtype, n_layer, layer, block_table, max_pages, kvpos, active,
                            B, out_q, out_d, out_f32=None):
        self._check(self.lib.gsvcu_op_decode_attention(self.h, _ptr(q), q_stride, _ptr(pool), kv_dtype, n_layer, layer,
                                                       _ptr(block_table), max_pages, _ptr(kvpos), _ptr(active), B,
                                                       _ptr(out_q), _ptr(out_d), _ptr(out_f32)))

    def op_prefill_attention(self, qkv, seq_start, seq_len, text_len, out_q, out_d, out_f32=None):
        ss = np.ascontiguousarray(seq_start, np.int32)
        sl = np.ascontiguousarray(seq_len, np.int32)
        tl = np.ascontiguousarray(text_len, np.int32)
        self._check(self.lib.gsvcu_op_prefill_attention(self.h, _ptr(qkv), ss.size, _ptr(ss), _ptr(sl), _ptr(tl),
                                                        _ptr(out_q), _ptr(out_d), _ptr(out_f32)))

    def op_sample(self, logits, V, eos, steps, rng_states, prev=None, top_k=15, top_p=1.0, temperature=1.0, rep=1.35):
        """logits: torch CUDA [B][V]; prev: list of int arrays (repetition windows). Returns (tokens, new states)."""
        B = logits.shape[0]
        sc = SamplerCfg(top_k, top_p, temperature, rep)
        st = np.ascontiguousarray(steps, np.int32)
        rs = np.ascontiguousarray(rng_states, np.uint64).copy()
        tok = np.zeros(B, np.int32)
        if prev is not None:
            stride = max(1, max(len(p) for p in prev))
            pv = np.zeros((B, stride), np.int32)
            npv = np.zeros(B, np.int32)
            for b, p in enumerate(prev):
                pv[b, :len(p)] = p
                npv[b] = len(p)
        else:
            stride, pv, npv = 0, None, None
        self._check(self.lib.gsvcu_op_sample(self.h, _ptr(logits), B, V, eos, C.byref(sc), _ptr(pv), _ptr(npv),
                                             stride, _ptr(st), _ptr(rs), _ptr(tok)))
        return tok, rs


class Bert:
    """The BERT feature producer on the GPU (gsvcu_bert_*; the role of gsv.cpp's gsv_bert)."""

    def __init__(self, path: str, device: int = 0):
        self.lib = load_library()
        h = C.c_void_p()
        rc = self.lib.gsvcu_bert_load(device, path.encode(), C.byref(h))
        if rc != OK:
            raise GsvcuError(rc, "gsvcu_bert_load failed (see stderr)")
        self.h = h
        hp = BertHParams()
        self.lib.gsvcu_bert_get_hparams(self.h, C.byref(hp))
        self.hp = hp

    def close(self):
        if getattr(self, "h", None):
            self.lib.gsvcu_bert_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != OK:
            raise GsvcuError(rc, self.lib.gsvcu_bert_last_error(self.h).decode(errors="replace"))

    def encode(self, ids, n_layers=-1) -> np.ndarray:
        """gsv_bert::encode / encode_layers: [hidden][T]."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((self.hp.hidden, ids.size), np.float32)
        self._check(self.lib.gsvcu_bert_encode(self.h, ids.ctypes.data, ids.size, n_layers, out.ctypes.data))
        return out

    def encode_feat_batch(self, ids_flat, lens, tmax, out=None):
        """gsv_bert::encode_feat_batch: a list of [hidden][lens[b] - 2] arrays (empty for lens[b] <= 2); with
        out (a device tensor) the features are written there, concatenated, and out is returned."""
        ids_flat = np.ascontiguousarray(ids_flat, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        D = self.hp.hidden
        sizes = [D * max(int(l) - 2, 0) for l in lens]
        if out is not None:
            self._check(self.lib.gsvcu_bert_encode_feat_batch(self.h, len(lens), ids_flat.ctypes.data, lens.ctypes.data,
                                                              tmax, _ptr(out), 1))
            return out
        flat = np.empty(max(sum(sizes), 1), np.float32)
        self._check(self.lib.gsvcu_bert_encode_feat_batch(self.h, len(lens), ids_flat.ctypes.data, lens.ctypes.data,
                                                          tmax, flat.ctypes.data, 0))
        res, at = [], 0
        for l, n in zip(lens, sizes):
            res.append(flat[at:at + n].reshape(D, max(int(l) - 2, 0)).copy())
            at += n
        return res


class Dit:
    """The DiT / CFM velocity estimator on the GPU (gsvcu_dit_*; the role of gsv.cpp's gsv_dit)."""

    def __init__(self, path: str, device: int = 0):
        self.lib = load_library()
        h = C.c_void_p()
        rc = self.lib.gsvcu_dit_load(device, path.encode(), C.byref(h))
        if rc != OK:
            raise GsvcuError(rc, "gsvcu_dit_load failed (see stderr)")
        self.h = h
        hp = DitHParams()
        self.lib.gsvcu_dit_get_hparams(self.h, C.byref(hp))
        self.hp = hp
        self.T = 0

    def close(self):
        if getattr(self, "h", None):
            self.lib.gsvcu_dit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != OK:
            raise GsvcuError(rc, self.lib.gsvcu_dit_last_error(self.h).decode(errors="replace"))

    def set_condition(self, cond, neg, x_lens=0):
        """The static cache of gsv_dit::prepare: condition / negative-condition rows [T][1024]."""
        cond = np.ascontiguousarray(cond, np.float32)
        neg = np.ascontiguousarray(neg, np.float32)
        assert cond.shape == neg.shape and cond.shape[1] == self.hp.dim
        self._check(self.lib.gsvcu_dit_set_condition(self.h, cond.ctypes.data, neg.ctypes.data, cond.shape[0], x_lens))
        self.T = cond.shape[0]

    def prepare(self, prompt_mel, mu, x_lens=0):
        """gsv_dit::prepare: the static cache from prompt_mel [100][T] and mu [512][T]."""
        prompt_mel = np.ascontiguousarray(prompt_mel, np.float32)
        mu = np.ascontiguousarray(mu, np.float32)
        self._check(self.lib.gsvcu_dit_prepare(self.h, prompt_mel.ctypes.data, mu.ctypes.data, mu.shape[1], x_lens))
        self.T = mu.shape[1]

    def condition(self) -> np.ndarray:
        """The condition rows [2][T][1024] (condition, negative) in use."""
        out = np.empty((2, self.T, self.hp.dim), np.float32)
        self._check(self.lib.gsvcu_dit_op_condition(self.h, out.ctypes.data))
        return out

    def sample_full(self, mu, prompt, steps, cfg, seed=1, x0=None, skip_steps=0) -> np.ndarray:
        """gsv_dit::sample: mu [512][T], prompt [100][P] -> mel [100][T - P] (seeded noise when x0 is None)."""
        mu = np.ascontiguousarray(mu, np.float32)
        prompt = np.ascontiguousarray(prompt, np.float32)
        T, P = mu.shape[1], prompt.shape[1]
        x0p = None if x0 is None else np.ascontiguousarray(x0, np.float32)
        out = np.empty((100, T - P), np.float32)
        self._check(self.lib.gsvcu_dit_sample_full(self.h, mu.ctypes.data, prompt.ctypes.data, P, T, steps, float(cfg),
                                                   seed, None if x0p is None else x0p.ctypes.data, skip_steps,
                                                   out.ctypes.data))
        self.T = T
        return out

    def synthesize(self, fea_ref, fea_todo, mel_ref, steps, cfg, seed=1, block_override=0, skip_steps=0) -> np.ndarray:
        """gsv_dit::synthesize: fea_ref [512][R], fea_todo [512][N], mel_ref [100][mel_ref_T] -> mel [100][N]."""
        fea_ref = np.ascontiguousarray(fea_ref, np.float32)
        fea_todo = np.ascontiguousarray(fea_todo, np.float32)
        mel_ref = np.ascontiguousarray(mel_ref, np.float32)
        out = np.empty((100, fea_todo.shape[1]), np.float32)
        self._check(self.lib.gsvcu_dit_synthesize(self.h, fea_ref.ctypes.data, fea_ref.shape[1], fea_todo.ctypes.data,
                                                  fea_todo.shape[1], mel_ref.ctypes.data, mel_ref.shape[1], steps,
                                                  float(cfg), seed, block_override, None, 0, skip_steps,
                                                  out.ctypes.data))
        return out

    def set_dbcache(self, fn, threshold=0.08, warmup=8, warmup_interval=1, max_cached=-1, max_cont=-1,
                    max_accum=0.0, downsample=4):
        """cache-dit (DBCache) settings (gsv_dit_cfg::dbcache_*); fn = 0 turns it off."""
        self._check(self.lib.gsvcu_dit_set_dbcache(self.h, fn, float(threshold), warmup, warmup_interval, max_cached,
                                                   max_cont, float(max_accum), downsample))

    def db_stats(self):
        """(steps, hits [2], misses [2], last_fd [2], acc [2])."""
        st = np.zeros(1, np.int32)
        h, m = np.zeros(2, np.int32), np.zeros(2, np.int32)
        fd, acc = np.zeros(2, np.float32), np.zeros(2, np.float32)
        self._check(self.lib.gsvcu_dit_db_get_stats(self.h, st.ctypes.data, h.ctypes.data, m.ctypes.data, fd.ctypes.data,
                                                    acc.ctypes.data))
        return int(st[0]), h, m, fd, acc

    def set_alg(self, uncond_reuse: int):
        """gsv_dit::set_alg: uncond_reuse 0, 1 (reuse on odd steps) or 2 (extrapolate on odd steps)."""
        self._check(self.lib.gsvcu_dit_set_alg(self.h, uncond_reuse))

    def velocity(self, x_mel, t, negative=False) -> np.ndarray:
        """gsv_dit::velocity: x_mel [100][T] -> vel [100][T]."""
        x_mel = np.ascontiguousarray(x_mel, np.float32)
        vel = np.empty_like(x_mel)
        self._check(self.lib.gsvcu_dit_velocity(self.h, x_mel.ctypes.data, float(t), int(bool(negative)), vel.ctypes.data))
        return vel

    def sample(self, x0, P, steps, cfg, skip_steps=0) -> np.ndarray:
        """gsv_dit::sample's CFM loop on the set condition: x0 [100][T] -> mel [100][T - P]."""
        x0 = np.ascontiguousarray(x0, np.float32)
        out = np.empty((x0.shape[0], x0.shape[1] - P), np.float32)
        self._check(self.lib.gsvcu_dit_sample(self.h, x0.ctypes.data, P, steps, float(cfg), skip_steps, out.ctypes.data))
        return out

    def hidden(self, x_mel, t, n_blocks) -> np.ndarray:
        """Hidden state [2][T][1024] (conditioned, negative) after the trunk and n_blocks blocks."""
        x_mel = np.ascontiguousarray(x_mel, np.float32)
        out = np.empty((2, self.T, self.hp.dim), np.float32)
        self._check(self.lib.gsvcu_dit_op_hidden(self.h, x_mel.ctypes.data, float(t), n_blocks, out.ctypes.data))
        return out

    def stream_handle(self) -> int:
        s = C.c_void_p()
        self._check(self.lib.gsvcu_dit_stream(self.h, C.byref(s)))
        return s.value or 0
