"""Seeded synthetic AR weights and requests (no checkpoints or datasets exist offline).

`write_model` writes a GGUF file with the tensor names, shapes, dtypes and KV keys of the
reference exporter (tools/export_gguf/convert_ar.py:91-130, dtype policy :76-89): attention and
FFN matrices Q8_0 (``--spec attn=q8_0,ffn=q8_0``), everything else F32. Values are random:
matrices and embeddings N(0, 0.02), LayerNorm weight 1 + N(0, 0.02), biases N(0, 0.02),
PE alphas 1.0. Requests follow the benchmark shapes of the reference (tests/bench_ar_width.cpp:43-55):
uniform phone ids in [0, 731], BERT features N(0, 1) laid out [1024][T], prompt codes in [0, 1023].
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np


@dataclass
class Dims:
    D: int = 512
    NH: int = 16
    NL: int = 24
    V: int = 1025
    PV: int = 732
    EOS: int = 1024
    BERT: int = 1024


def iq4_nl_blocks(arr: np.ndarray) -> np.ndarray:
    """IQ4_NL blocks of a float [N][K] array from a plain quantizer (not ggml's scale search): per 32
    values d = fp16(amax / 127) and each value the nearest entry of the IQ4_NL table, codes packed as
    block_iq4_nl (fp16 d, then values 0..15 in the low nibbles and 16..31 in the high ones)."""
    from gguf import quants
    table = np.array(quants.IQ4_NL.kvalues, np.float32)
    N, K = arr.shape
    b = arr.reshape(N, K // 32, 32)
    d = (np.abs(b).max(-1, keepdims=True) / 127).astype(np.float16)
    df = d.astype(np.float32)
    df[df == 0] = 1
    idx = np.abs(b[..., None] / df[..., None] - table).argmin(-1).astype(np.uint8)
    qs = idx[..., :16] | (idx[..., 16:] << 4)
    return np.concatenate([d.view(np.uint8).reshape(N, K // 32, 2), qs], axis=-1).reshape(N, K // 32 * 18)


def kquant_blocks(arr: np.ndarray, kind: str) -> np.ndarray:
    """Q4_K / Q5_K / Q6_K blocks of a float [N][K] array (K % 256 == 0) from a plain quantizer (not ggml's
    scale search), packed as block_q4_K {fp16 d, dmin; 12 bytes of 6-bit scales / mins; 128 bytes of
    nibbles}, block_q5_K {d, dmin, scales, 32 bytes of fifth bits, nibbles}, block_q6_K {128 bytes of low
    nibbles; 64 bytes of 2-bit highs; 16 int8 scales; fp16 d}."""
    N, K = arr.shape
    sb = arr.reshape(N * K // 256, 256).astype(np.float64)
    nsb = sb.shape[0]
    if kind == "q6_k":
        sub = sb.reshape(nsb, 16, 16)
        s = np.abs(sub).max(-1) / 31.0
        d = (np.abs(s).max(-1) / 127.0).astype(np.float16)
        df = np.where(d.astype(np.float64) == 0, 1.0, d.astype(np.float64))
        sc = np.clip(np.round(s / df[:, None]), -128, 127).astype(np.int8)
        step = df[:, None] * np.where(sc == 0, 1, sc)
        q = (np.clip(np.round(sub / step[..., None]), -32, 31) + 32).astype(np.uint8).reshape(nsb, 256)
        out = np.zeros((nsb, 210), np.uint8)
        for hh in range(2):
            for k in range(4):
                v = q[:, 128 * hh + 32 * k: 128 * hh + 32 * k + 32]
                lo = v & 15
                col = 64 * hh + (k & 1) * 32
                out[:, col:col + 32] |= lo if k < 2 else (lo << 4)
                out[:, 128 + 32 * hh: 160 + 32 * hh] |= ((v >> 4) & 3) << (2 * k)
        out[:, 192:208] = sc.view(np.uint8)
        out[:, 208:210] = d.view(np.uint8).reshape(nsb, 2)
        return out.reshape(N, K // 256 * 210)
    top = 15 if kind == "q4_k" else 31
    sub = sb.reshape(nsb, 8, 32)
    mn = np.maximum(0.0, -sub.min(-1))
    s = (sub.max(-1) + mn) / top
    d = (s.max(-1) / 63.0).astype(np.float16)
    dmin = (mn.max(-1) / 63.0).astype(np.float16)
    df = np.where(d.astype(np.float64) == 0, 1.0, d.astype(np.float64))
    dmf = np.where(dmin.astype(np.float64) == 0, 1.0, dmin.astype(np.float64))
    sc = np.clip(np.round(s / df[:, None]), 1, 63).astype(np.uint8)
    mq = np.clip(np.round(mn / dmf[:, None]), 0, 63).astype(np.uint8)
    q = np.clip(np.round((sub + (dmf[:, None] * mq)[..., None]) / (df[:, None] * sc)[..., None]), 0, top)
    q = q.astype(np.uint8).reshape(nsb, 256)
    scales = np.zeros((nsb, 12), np.uint8)
    for j in range(8):
        if j < 4:
            scales[:, j] |= sc[:, j]
            scales[:, j + 4] |= mq[:, j]
        else:
            scales[:, j + 4] |= (sc[:, j] & 15) | ((mq[:, j] & 15) << 4)
            scales[:, j - 4] |= (sc[:, j] >> 4) << 6
            scales[:, j] |= (mq[:, j] >> 4) << 6
    qs = np.zeros((nsb, 128), np.uint8)
    qh = np.zeros((nsb, 32), np.uint8)
    for g in range(4):
        lo, hi = q[:, 64 * g: 64 * g + 32], q[:, 64 * g + 32: 64 * g + 64]
        qs[:, 32 * g: 32 * g + 32] = (lo & 15) | ((hi & 15) << 4)
        qh |= ((lo >> 4) & 1) << (2 * g)
        qh |= ((hi >> 4) & 1) << (2 * g + 1)
    hdr = np.concatenate([d.view(np.uint8).reshape(nsb, 2), dmin.view(np.uint8).reshape(nsb, 2), scales], -1)
    out = np.concatenate([hdr, qs] if kind == "q4_k" else [hdr, qh, qs], -1)
    return out.reshape(N, -1)


def write_model(path: str, seed: int = 0, dims: Dims | None = None, mat_type: str = "q8_0",
                ln_noise: float = 0.02, predict_type: str = "f32", emb_type: str = "f32",
                ffn_type: str | None = None) -> str:
    """mat_type is the type of the attention matrices (the exporter's --spec attn=...) and, unless
    ffn_type is given, of the FFN matrices (--spec ffn=...): "q8_0", "q4_0", "q4_1", "q5_0", "q5_1",
    "q4_k", "q5_k", "q6_k", "iq4_nl", "f16", "bf16" or "f32" (iq4_nl: the reference's
    tools/quantize_gguf.cpp tier, quantized by iq4_nl_blocks; K-quants by kquant_blocks). predict_type "f32" or any of those stores ar.predict in that type
    (--spec predict=...); emb_type "f16" / "bf16" stores the
    text / audio embeddings as F16 (--spec emb=f16). The exporter's --f16 preset is
    mat_type="f16", predict_type="f16", emb_type="f16"; its default (no flags) is mat_type="f32"."""
    import gguf

    d = dims or Dims()
    rng = np.random.default_rng(seed)
    D, FF = d.D, 4 * d.D
    types = {"q8_0": gguf.GGMLQuantizationType.Q8_0, "f32": gguf.GGMLQuantizationType.F32,
             "f16": gguf.GGMLQuantizationType.F16, "q4_0": gguf.GGMLQuantizationType.Q4_0,
             "q5_0": gguf.GGMLQuantizationType.Q5_0, "iq4_nl": gguf.GGMLQuantizationType.IQ4_NL,
             "bf16": gguf.GGMLQuantizationType.BF16, "q4_1": gguf.GGMLQuantizationType.Q4_1,
             "q5_1": gguf.GGMLQuantizationType.Q5_1, "q4_k": gguf.GGMLQuantizationType.Q4_K,
             "q5_k": gguf.GGMLQuantizationType.Q5_K, "q6_k": gguf.GGMLQuantizationType.Q6_K}
    qt = types[mat_type]
    ft = types[ffn_type or mat_type]

    def n(*shape, s=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    w = gguf.GGUFWriter(path, "gsv.ar")
    w.add_uint32("ar.hidden_dim", D)
    w.add_uint32("ar.head", d.NH)
    w.add_uint32("ar.n_layer", d.NL)
    w.add_uint32("ar.vocab_size", d.V)
    w.add_uint32("ar.phoneme_vocab_size", d.PV)
    w.add_uint32("ar.eos", d.EOS)
    w.add_float32("ar.bert_dim", float(d.BERT))

    def add(name, arr, dtype=gguf.GGMLQuantizationType.F32):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        if dtype == gguf.GGMLQuantizationType.F32:
            w.add_tensor(name, arr, raw_dtype=dtype)
        elif dtype == gguf.GGMLQuantizationType.F16:
            w.add_tensor(name, arr.astype(np.float16), raw_dtype=dtype)
        elif dtype == gguf.GGMLQuantizationType.IQ4_NL:
            w.add_tensor(name, iq4_nl_blocks(arr), raw_dtype=dtype)
        elif dtype in (gguf.GGMLQuantizationType.Q4_K, gguf.GGMLQuantizationType.Q5_K, gguf.GGMLQuantizationType.Q6_K):
            w.add_tensor(name, kquant_blocks(arr, dtype.name.lower()), raw_dtype=dtype)
        else:
            w.add_tensor(name, gguf.quants.quantize(arr, dtype), raw_dtype=dtype)

    et = {"f32": gguf.GGMLQuantizationType.F32, "f16": gguf.GGMLQuantizationType.F16,
          "bf16": gguf.GGMLQuantizationType.BF16}[emb_type]
    add("ar.text_emb", n(d.PV, D), et)
    add("ar.audio_emb", n(d.V, D), et)
    add("ar.bert_proj", n(D, d.BERT))
    add("ar.bert_proj_b", n(D))
    add("ar.text_pe_alpha", np.ones(1, np.float32))
    add("ar.audio_pe_alpha", np.ones(1, np.float32))
    add("ar.predict", n(d.V, D), types[predict_type])
    for li in range(d.NL):
        p = f"transformer.block{li}"
        add(f"{p}.qkv_w", n(3 * D, D), qt)
        add(f"{p}.qkv_b", n(3 * D))
        add(f"{p}.out_w", n(D, D), qt)
        add(f"{p}.out_b", n(D))
        add(f"{p}.norm1_w", 1.0 + n(D, s=ln_noise))
        add(f"{p}.norm1_b", n(D, s=ln_noise))
        add(f"{p}.ffn1_w", n(FF, D), ft)
        add(f"{p}.ffn1_b", n(FF))
        add(f"{p}.ffn2_w", n(D, FF), ft)
        add(f"{p}.ffn2_b", n(D))
        add(f"{p}.norm2_w", 1.0 + n(D, s=ln_noise))
        add(f"{p}.norm2_b", n(D, s=ln_noise))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def cached_model(cache_dir: str, seed: int = 0, n_layer: int = 24, mat_type: str = "q8_0",
                 predict_type: str = "f32", emb_type: str = "f32", ffn_type: str | None = None) -> str:
    """Write (once) and return the path of a synthetic model in cache_dir."""
    os.makedirs(cache_dir, exist_ok=True)
    suffix = ("" if predict_type == "f32" else f"_p{predict_type}") + ("" if emb_type == "f32" else f"_e{emb_type}")
    suffix += "" if ffn_type in (None, mat_type) else f"_f{ffn_type}"
    path = os.path.join(cache_dir, f"gsv_ar_synth_s{seed}_l{n_layer}_{mat_type}{suffix}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model(tmp, seed=seed, dims=Dims(NL=n_layer), mat_type=mat_type, predict_type=predict_type,
                    emb_type=emb_type, ffn_type=ffn_type)
        os.replace(tmp, path)
    return path


@dataclass
class Request:
    """gsv_ar_request (reference src/gsv_ar.h:13-17)."""
    phones: np.ndarray   # int32 [T]
    bert: np.ndarray     # float32 [1024][T]
    prompt: np.ndarray   # int32 [P]


def make_request(rng: np.random.Generator, n_phones: int, n_prompt: int, bert_dim: int = 1024,
                 phone_vocab: int = 732, code_max: int = 1023) -> Request:
    return Request(
        phones=rng.integers(0, phone_vocab, n_phones, dtype=np.int32),
        bert=rng.standard_normal((bert_dim, n_phones), dtype=np.float32),
        prompt=rng.integers(0, code_max + 1, n_prompt, dtype=np.int32),
    )


def ragged_requests(seed: int, B: int, lo: int = 80, hi: int = 400, text_frac: float = 0.7):
    """Prefixes P ~ U[lo, hi] split round(0.7 P) phones / rest prompt codes (BASELINE configs 1 and 4)."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(B):
        P = int(rng.integers(lo, hi + 1))
        T = int(round(text_frac * P))
        out.append(make_request(rng, T, P - T))
    return out


@dataclass
class BertDims:
    """Dims of a synthetic gsv BERT (chinese-roberta-wwm-ext-large: 1024 / 16 / 4096 / 24 layers, 22 used)."""
    D: int = 1024
    NH: int = 16
    FF: int = 4096
    NL: int = 24
    VOCAB: int = 21128
    MAXPOS: int = 512


def write_bert_model(path: str, seed: int = 0, dims: BertDims | None = None, mat_type: str = "f32") -> str:
    """Seeded synthetic BERT GGUF with the names, shapes, dtypes and KV keys of the reference exporter
    (tools/export_gguf/convert_bert.py:38-88): embeddings, norms and biases F32, attention / FFN
    matrices `mat_type` (its --spec attn=..,ffn=..). Values N(0, 0.02), LayerNorm weights 1 + N(0, 0.02)."""
    import gguf

    d = dims or BertDims()
    rng = np.random.default_rng(seed)
    types = {"f32": gguf.GGMLQuantizationType.F32, "f16": gguf.GGMLQuantizationType.F16,
             "q8_0": gguf.GGMLQuantizationType.Q8_0}

    def n(*shape, s=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    w = gguf.GGUFWriter(path, "gsv.bert")
    w.add_uint32("bert.n_layer", d.NL)
    w.add_uint32("bert.hidden", d.D)
    w.add_uint32("bert.head", d.NH)
    w.add_uint32("bert.inter", d.FF)
    w.add_float32("bert.ln_eps", 1e-12)
    w.add_uint32("bert.vocab", d.VOCAB)
    w.add_uint32("bert.max_pos", d.MAXPOS)
    w.add_uint32("bert.layers_used", d.NL - 2)

    def add(name, arr, qt=gguf.GGMLQuantizationType.F32):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        if qt == gguf.GGMLQuantizationType.F32:
            w.add_tensor(name, arr, raw_dtype=qt)
        elif qt == gguf.GGMLQuantizationType.F16:
            w.add_tensor(name, arr.astype(np.float16), raw_dtype=qt)
        else:
            w.add_tensor(name, gguf.quants.quantize(arr, qt), raw_dtype=qt)

    mt = types[mat_type]
    add("bert.word_emb", n(d.VOCAB, d.D))
    add("bert.pos_emb", n(d.MAXPOS, d.D))
    add("bert.type_emb", n(2, d.D))
    add("bert.emb_ln_w", 1.0 + n(d.D))
    add("bert.emb_ln_b", n(d.D))
    for li in range(d.NL):
        p = f"bert.l{li}."
        add(p + "qkv_w", n(3 * d.D, d.D), mt)
        add(p + "qkv_b", n(3 * d.D))
        add(p + "attn_out_w", n(d.D, d.D), mt)
        add(p + "attn_out_b", n(d.D))
        add(p + "attn_ln_w", 1.0 + n(d.D))
        add(p + "attn_ln_b", n(d.D))
        add(p + "ff1_w", n(d.FF, d.D), mt)
        add(p + "ff1_b", n(d.FF))
        add(p + "ff2_w", n(d.D, d.FF), mt)
        add(p + "ff2_b", n(d.D))
        add(p + "out_ln_w", 1.0 + n(d.D))
        add(p + "out_ln_b", n(d.D))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def write_dit_model(path: str, seed: int = 0, depth: int = 22, mat_type: str = "f16") -> str:
    """Seeded synthetic DiT GGUF with the names, shapes, dtypes and KV keys of the reference exporter
    (tools/export_gguf/convert_dit.py:40-152): 2D weights `mat_type` (its --spec lin=..), biases, norms and
    inv_freq F32; conv_pos weights in the exporter's [G][OCg][ICg * K] order (inner index ic * 31 + tap).
    Values N(0, 0.02); the AdaLN biases N(0, 0.3) so the gates and modulations are not negligible;
    inv_freq the fp16-stored 10000^(-2i/64); text_embed: freqs_cis by the exporter's formula, 4
    ConvNeXtV2 blocks (depthwise taps [7][512] as the exporter transposes them, N(0, 0.2); GRN gamma and
    beta N(0, 0.3))."""
    import gguf

    D, MEL = 1024, 100
    rng = np.random.default_rng(seed)
    qt = {"f32": gguf.GGMLQuantizationType.F32, "f16": gguf.GGMLQuantizationType.F16}[mat_type]

    def n(*shape, s=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    w = gguf.GGUFWriter(path, "gsv.dit")
    for k, v in (("dit.dim", D), ("dit.depth", depth), ("dit.heads", 16), ("dit.dim_head", 64), ("dit.ff_mult", 2),
                 ("dit.mel_dim", MEL), ("dit.text_dim", 512), ("dit.conv_layers", 4), ("dit.conv_pos_groups", 16),
                 ("dit.conv_pos_kernel", 31), ("dit.rope_dims", 64), ("dit.text_max_pos", 4096),
                 ("dit.time_freq_dim", 256)):
        w.add_uint32(k, v)
    w.add_float32("dit.norm_eps", 1e-6)

    def add(name, arr, mat=False):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        if mat and qt == gguf.GGMLQuantizationType.F16:
            w.add_tensor(name, arr.astype(np.float16), raw_dtype=qt)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType.F32)

    add("dit.time_embed.time_mlp.0.weight", n(D, 256), True)
    add("dit.time_embed.time_mlp.0.bias", n(D))
    add("dit.time_embed.time_mlp.2.weight", n(D, D), True)
    add("dit.time_embed.time_mlp.2.bias", n(D))
    freqs = (np.float32(1.0) / (np.float32(10000.0) ** (np.arange(0, 512, 2, dtype=np.float32) / np.float32(512))))
    ang = np.outer(np.arange(4096, dtype=np.float32), freqs).astype(np.float32)
    add("dit.text_embed.freqs_cis", np.concatenate([np.cos(ang), np.sin(ang)], axis=1))
    for bi in range(4):
        p = f"dit.text_embed.text_blocks.{bi}."
        add(p + "dwconv.weight", n(7, 512, s=0.2))
        add(p + "dwconv.bias", n(512))
        add(p + "norm.weight", 1.0 + n(512))
        add(p + "norm.bias", n(512))
        add(p + "pwconv1.weight", n(1024, 512), True)
        add(p + "pwconv1.bias", n(1024))
        add(p + "grn.gamma", n(1, 1, 1024, s=0.3))
        add(p + "grn.beta", n(1, 1, 1024, s=0.3))
        add(p + "pwconv2.weight", n(512, 1024), True)
        add(p + "pwconv2.bias", n(512))
    add("dit.input_embed.proj.weight_mel", n(D, MEL), True)
    add("dit.input_embed.proj.weight_ctx", n(D, 612), True)
    add("dit.input_embed.proj.bias", n(D))
    for li in (0, 2):
        add(f"dit.input_embed.conv_pos_embed.conv1d.{li}.weight", n(16, 64, 64 * 31), True)
        add(f"dit.input_embed.conv_pos_embed.conv1d.{li}.bias", n(D))
    inv = (1.0 / (10000.0 ** (np.arange(0, 64, 2, dtype=np.float32) / 64.0))).astype(np.float16).astype(np.float32)
    add("dit.rotary_embed.inv_freq", inv)
    for li in range(depth):
        p = f"dit.transformer_blocks.{li}."
        add(p + "attn_norm.linear.weight", n(6 * D, D), True)
        add(p + "attn_norm.linear.bias", n(6 * D, s=0.3))
        for m in ("to_q", "to_k", "to_v"):
            add(p + f"attn.{m}.weight", n(D, D), True)
            add(p + f"attn.{m}.bias", n(D))
        add(p + "attn.to_out.0.weight", n(D, D), True)
        add(p + "attn.to_out.0.bias", n(D))
        add(p + "ff.ff.0.0.weight", n(2048, D), True)
        add(p + "ff.ff.0.0.bias", n(2048))
        add(p + "ff.ff.2.weight", n(D, 2048), True)
        add(p + "ff.ff.2.bias", n(D))
    add("dit.norm_out.linear.weight", n(2 * D, D), True)
    add("dit.norm_out.linear.bias", n(2 * D, s=0.3))
    add("dit.proj_out.weight", n(MEL, D), True)
    add("dit.proj_out.bias", n(MEL))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def cached_dit_model(cache_dir: str, seed: int = 0, depth: int = 22, mat_type: str = "f16") -> str:
    """Path of a synthetic DiT GGUF, written once per (seed, depth, mat_type) under cache_dir."""
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"dit_s{seed}_d{depth}_{mat_type}_te.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_dit_model(tmp, seed, depth, mat_type)
        os.replace(tmp, path)
    return path
