"""CPU restatement of gsv.cpp's DiT / CFM velocity estimator -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / --impl reference leg use this
module; it checks the CUDA library and is never a fallback for it.

It follows the reference graph (src/gsv_dit.cpp) op by op in numpy:
  time_sin              :755-769   SinusPositionEmbedding(256), float32 expf / sinf / cosf
  time_embed            :278-284   Linear 256 -> 1024, SiLU, Linear 1024 -> 1024
  build_trunk           :533-549   x = proj_mel(x_mel) + condition; conv_pos twice (grouped conv1d,
                                   k = 31, 16 groups, zero padding 15, bias + Mish), * mask, + x
  dit_block             :407-433   AdaLN-Zero modulation, LN * (1 + scale) + shift (layernorm_affine,
                                   eps 1e-6), to_q / to_k / to_v, RoPE of head 0 (:191-200: adjacent
                                   pairs, angle n * inv_freq[i]), flash attention with the key padding
                                   mask (:333-346), to_out * mask, gated residual, FFN with GELU (tanh),
                                   gated residual
  build_head            :563-576   norm_out (scale, shift) + proj_out
  sample                :1410-1478 Euler steps t = j / steps with guidance v + (v - v_neg) * cfg, the
                                   prompt frames zeroed; x0 = randn * 0.875 from gsv_rng (:1403-1408)
  prepare / build_prepare :486-531 text path: mu^T + freqs_cis, 4 ConvNeXtV2 blocks (:242-275: depthwise
                                   conv k = 7 in tap order, LayerNorm with affine, pwconv1, GELU (erf), GRN
                                   (:222-241), pwconv2, residual); condition = proj_ctx([prompt_x | text]) + b,
                                   negative = proj_ctx([0 | text]) + b
  synthesize            :1480-1581 chunks of <= 640 frames after the last 500 reference frames, the prompt
                                   of later chunks ending in the previous chunk's last 32 frames
Numerics: ggml's mul_mat with F16 weights converts the activations to F16 before the dot products,
so every matrix product here takes f16-rounded activations against the f16 weights, summed in
float64 and rounded to float32 once; everything else is float32 (LayerNorm statistics float64).
GELU is evaluated with the tanh formula in float32 (torch's approximate="tanh"), not with ggml's
fp16 lookup table. Parity with the CUDA path is a relative-L2 tolerance, not bitwise.
Parity unpinned: the reference DiT needs ggml (absent here) and ships no DiT golden vectors, so this
restatement is checked against the reference's formulas only, not against a run of the reference.
"""
from __future__ import annotations

import numpy as np

D, NH, HD, MEL, FF = 1024, 16, 64, 100, 2048
KCP, GCP, ICG = 31, 16, 64


def load(path: str) -> dict:
    """Tensors of a DiT GGUF as float32 numpy arrays (shapes in torch order: [out][in])."""
    from gguf import GGUFReader

    r = GGUFReader(path)
    W = {}
    for t in r.tensors:
        a = np.asarray(t.data)
        shape = tuple(int(x) for x in reversed(t.shape.tolist()))
        W[t.name] = a.astype(np.float32).reshape(shape)
    depth = 0
    while f"dit.transformer_blocks.{depth}.attn.to_q.weight" in W:
        depth += 1
    W["depth"] = depth
    return W


def f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def mm(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    """ggml mul_mat with an F16 weight: x [R][K] (f16-rounded) . w[N][K]^T, double sums, + bias."""
    y = (f16(x).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
    return y + b.astype(np.float32) if b is not None else y


def silu(x):
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def mish(x):
    x = np.asarray(x, dtype=np.float32)
    sp = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)
    return (x * np.tanh(sp)).astype(np.float32)


def gelu_tanh(x):
    x = np.asarray(x, dtype=np.float32)
    u = np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x * x * x)
    return (np.float32(0.5) * x * (np.float32(1) + np.tanh(u))).astype(np.float32)


def time_sin(t: float) -> np.ndarray:
    e = np.float32(np.log(10000.0) / 127.0)
    freq = np.exp(-e * np.arange(128, dtype=np.float32)).astype(np.float32)
    a = (np.float32(1000.0) * np.float32(t) * freq).astype(np.float32)
    return np.concatenate([np.sin(a), np.cos(a)]).astype(np.float32)


def layernorm_mod(x: np.ndarray, scale: np.ndarray, shift: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    mean = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mean) ** 2).mean(axis=-1, keepdims=True)
    y = ((x64 - mean) / np.sqrt(var + 1e-6)).astype(np.float32)
    return (y * (np.float32(1) + scale) + shift).astype(np.float32)


def rope_tables(inv_freq: np.ndarray, T: int):
    a = (np.arange(T, dtype=np.float32)[:, None] * inv_freq[None, :].astype(np.float32)).astype(np.float32)
    return np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)


def rope64(x: np.ndarray, cs: np.ndarray, sn: np.ndarray) -> np.ndarray:
    """Adjacent pairs (2i, 2i + 1) of the first 64 columns rotated by angle t * inv_freq[i]."""
    y = x.copy()
    x0, x1 = x[:, 0:64:2], x[:, 1:64:2]
    y[:, 0:64:2] = x0 * cs - x1 * sn
    y[:, 1:64:2] = x0 * sn + x1 * cs
    return y


def conv_pos(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Grouped conv1d (16 groups of 64 channels, 31 taps, zero padding 15) of x [T][1024], + bias.
    w: the exporter's [G][OCg][ICg * 31] with inner index ic * 31 + tap."""
    T = x.shape[0]
    xp = np.zeros((T + KCP - 1, D), dtype=np.float32)
    xp[KCP // 2:KCP // 2 + T] = f16(x)
    out = np.empty((T, D), dtype=np.float32)
    idx = np.arange(T)[:, None] + np.arange(KCP)[None, :]   # [T][31]
    for g in range(GCP):
        win = xp[:, g * ICG:(g + 1) * ICG][idx]                # [T][31][64]
        cols = win.transpose(0, 2, 1).reshape(T, ICG * KCP)   # inner index ic * 31 + tap
        out[:, g * ICG:(g + 1) * ICG] = (cols.astype(np.float64) @ w[g].astype(np.float64).T).astype(np.float32)
    return out + b


def attention(q, k, v, x_lens):
    """Softmax(q k^T / 8) v per head over keys < x_lens; q, k, v [T][1024] -> [T][1024]."""
    T = q.shape[0]
    out = np.empty((T, D), dtype=np.float32)
    for h in range(NH):
        sl = slice(h * HD, (h + 1) * HD)
        s = (q[:, sl].astype(np.float64) @ k[:x_lens, sl].astype(np.float64).T) * 0.125
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, sl] = (p @ v[:x_lens, sl].astype(np.float64)).astype(np.float32)
    return out


def time_embed(W, t: float) -> np.ndarray:
    h = silu(mm(time_sin(t)[None, :], W["dit.time_embed.time_mlp.0.weight"], W["dit.time_embed.time_mlp.0.bias"]))
    return mm(h, W["dit.time_embed.time_mlp.2.weight"], W["dit.time_embed.time_mlp.2.bias"])[0]


def trunk(W, x_mel: np.ndarray, cond: np.ndarray, x_lens: int) -> np.ndarray:
    """build_trunk (src/gsv_dit.cpp:533-549): x_mel [100][T], cond [T][1024] -> hidden [T][1024]."""
    T = x_mel.shape[1]
    mask = (np.arange(T) < x_lens).astype(np.float32)[:, None]
    x = mm(x_mel.T, W["dit.input_embed.proj.weight_mel"]) + cond
    cp = mish(conv_pos(x * mask, W["dit.input_embed.conv_pos_embed.conv1d.0.weight"],
                       W["dit.input_embed.conv_pos_embed.conv1d.0.bias"]))
    cp = mish(conv_pos(cp, W["dit.input_embed.conv_pos_embed.conv1d.2.weight"],
                       W["dit.input_embed.conv_pos_embed.conv1d.2.bias"])) * mask
    return (x + cp).astype(np.float32)


def blocks(W, x: np.ndarray, t: float, x_lens: int, l0: int, l1: int) -> np.ndarray:
    """DiT blocks l0 .. l1 - 1 (dit_block, src/gsv_dit.cpp:407-433) on hidden x [T][1024]."""
    T = x.shape[0]
    mask = (np.arange(T) < x_lens).astype(np.float32)[:, None]
    st = silu(time_embed(W, t))[None, :]
    cs, sn = rope_tables(W["dit.rotary_embed.inv_freq"], T)
    for li in range(l0, l1):
        p = f"dit.transformer_blocks.{li}."
        m = mm(st, W[p + "attn_norm.linear.weight"], W[p + "attn_norm.linear.bias"])[0].reshape(6, D)
        xn = layernorm_mod(x, m[1], m[0])
        q = rope64(mm(xn, W[p + "attn.to_q.weight"], W[p + "attn.to_q.bias"]), cs, sn)
        k = rope64(mm(xn, W[p + "attn.to_k.weight"], W[p + "attn.to_k.bias"]), cs, sn)
        v = mm(xn, W[p + "attn.to_v.weight"], W[p + "attn.to_v.bias"])
        a = mm(attention(q, k, v, x_lens), W[p + "attn.to_out.0.weight"], W[p + "attn.to_out.0.bias"]) * mask
        x = (x + a * m[2]).astype(np.float32)
        xn2 = layernorm_mod(x, m[4], m[3])
        f = mm(gelu_tanh(mm(xn2, W[p + "ff.ff.0.0.weight"], W[p + "ff.ff.0.0.bias"])),
               W[p + "ff.ff.2.weight"], W[p + "ff.ff.2.bias"])
        x = (x + f * m[5]).astype(np.float32)
    return x


def head_out(W, x: np.ndarray, t: float) -> np.ndarray:
    """build_head (src/gsv_dit.cpp:563-576): hidden [T][1024] -> vel [100][T]."""
    st = silu(time_embed(W, t))[None, :]
    e2 = mm(st, W["dit.norm_out.linear.weight"], W["dit.norm_out.linear.bias"])[0]
    xo = layernorm_mod(x, e2[:D], e2[D:])
    return mm(xo, W["dit.proj_out.weight"], W["dit.proj_out.bias"]).T.copy()


def branch(W, x_mel: np.ndarray, t: float, cond: np.ndarray, x_lens: int, n_blocks: int | None = None,
           head: bool = True) -> np.ndarray:
    """One estimator pass of one branch: x_mel [100][T] and cond [T][1024] -> vel [100][T] (with the head) or
    the hidden state [T][1024] after n_blocks blocks."""
    depth = W["depth"] if n_blocks is None else min(n_blocks, W["depth"])
    x = blocks(W, trunk(W, x_mel, cond, x_lens), t, x_lens, 0, depth)
    return head_out(W, x, t) if head else x


class DbCache:
    """cache-dit (DBCache) of gsv_dit (src/gsv_dit.cpp:1124-1323): settings, per-branch gates and state."""

    def __init__(self, fn, thr=0.08, warmup=8, warmup_interval=1, max_cached=-1, max_cont=-1, max_accum=0.0, ds=4):
        self.fn, self.thr, self.warmup, self.iv = fn, np.float32(thr), warmup, warmup_interval
        self.max_cached, self.max_cont, self.max_accum, self.ds = max_cached, max_cont, np.float32(max_accum), ds
        self.r_prev = [None, None]
        self.mr_prev = [None, None]
        self.step = 0
        self.reset()

    def reset(self):
        self.b = [dict(cached=0, cont=0, hits=0, misses=0, valid=False, acc=np.float32(0), last_fd=np.float32(0))
                  for _ in range(2)]
        self.step = 0


def branch_cached(W, db: DbCache, bi: int, x_mel, t, cond, x_lens):
    """run_step_cached (src/gsv_dit.cpp:1250-1323) of branch bi -> vel [100][T]."""
    T = x_mel.shape[1]
    xt = trunk(W, x_mel, cond, x_lens)
    xf = blocks(W, xt, t, x_lens, 0, db.fn)
    ds = db.ds if (db.ds >= 1 and T % db.ds == 0) else 1
    rflat = (xf - xt).astype(np.float32).ravel()
    Tds = T // ds
    if ds > 1:   # the reference's view: row stride of ds floats over the flat residual
        idx = (np.arange(Tds)[:, None] * ds + np.arange(D)[None, :]).ravel()
        r_cur = rflat[idx]
    else:
        r_cur = rflat
    if db.r_prev[bi] is None or db.r_prev[bi].size != r_cur.size:
        db.r_prev[bi] = np.zeros_like(r_cur)
    rp = db.r_prev[bi]
    fd = np.float32(np.float32(np.abs(r_cur.astype(np.float64) - rp).sum()) /
                    (np.float32(np.abs(rp.astype(np.float64)).sum()) + np.float32(1e-6)))
    d = db.b[bi]
    d["last_fd"] = fd
    hit = False
    warm = db.step < db.warmup and db.step % max(db.iv, 1) == 0
    if d["valid"] and db.thr > 0 and not warm:
        ok = fd < db.thr
        if ok and db.max_cached >= 0 and d["cached"] >= db.max_cached:
            ok = False
        if ok and db.max_cont >= 0 and d["cont"] >= db.max_cont:
            ok = False
            d["cont"] = 0
        if ok and db.max_accum > 0 and d["acc"] >= db.max_accum:
            ok = False
        hit = ok
    if fd > 0:
        d["acc"] = np.float32(d["acc"] + fd)
    if hit:
        xm = (xf + db.mr_prev[bi]).astype(np.float32)
        d["hits"] += 1
        d["cached"] += 1
        d["cont"] += 1
    else:
        xm = blocks(W, xf, t, x_lens, db.fn, W["depth"])
        db.mr_prev[bi] = (xm - xf).astype(np.float32)
        db.r_prev[bi] = r_cur.copy()
        d["misses"] += 1
        d["valid"] = True
        d["cont"] = 0
    return head_out(W, xm, t)


def sample(W, x0: np.ndarray, cond: np.ndarray, neg: np.ndarray, P: int, steps: int, cfg: float,
           uncond_reuse: int = 0, skip_steps: int = 0, db: DbCache | None = None) -> np.ndarray:
    """The CFM Euler loop on set conditions: x0 [100][T] -> mel [100][T - P]; uncond_reuse as the reference's
    alg (src/gsv_dit.cpp:1449-1468): 1 reuses the last computed negative velocity on odd steps, 2
    extrapolates 2 neg[k-1] - neg[k-2]."""
    x = x0.astype(np.float32).copy()
    T = x.shape[1]
    x[:, :P] = 0
    dt = np.float32(1.0) / np.float32(steps)
    p1 = p2 = None
    count = 0
    if db is not None:
        db.reset()
    vfun = (lambda bi, xx, tt, cc: branch_cached(W, db, bi, xx, tt, cc, T)) if db is not None else \
        (lambda bi, xx, tt, cc: branch(W, xx, tt, cc, T))
    for j in range(steps):
        if db is not None:
            db.step = j
        if j < skip_steps:   # src/gsv_dit.cpp:1444-1448: no model call, x unchanged
            continue
        t = float(np.float32(j) * dt)
        vel = vfun(0, x, t, cond)
        if cfg > 1e-5:
            odd = (j & 1) == 1
            if odd and uncond_reuse == 1 and count >= 1:
                ng = p1
            elif odd and uncond_reuse == 2 and count >= 2:
                ng = (np.float32(2.0) * p1 - p2).astype(np.float32)
            else:
                ng = vfun(1, x, t, neg)
                count += 1
                p2, p1 = p1, ng
            vel = (vel + (vel - ng) * np.float32(cfg)).astype(np.float32)
        x = (x + dt * vel).astype(np.float32)
        x[:, :P] = 0
    return x[:, P:].copy()


def gelu_erf(x):
    from scipy.special import erf
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(0.5) * x * (np.float32(1) + erf(x / np.float32(np.sqrt(2.0))).astype(np.float32))).astype(np.float32)


def text_embed(W, mu: np.ndarray) -> np.ndarray:
    """The text path of the static cache: mu [512][T] -> [T][512]."""
    T = mu.shape[1]
    x = (mu.T.astype(np.float32) + W["dit.text_embed.freqs_cis"][:T]).astype(np.float32)
    for bi in range(4):
        p = f"dit.text_embed.text_blocks.{bi}."
        w = W[p + "dwconv.weight"].reshape(7, 512)
        xp = np.zeros((T + 6, 512), dtype=np.float32)
        xp[3:3 + T] = x
        y = xp[0:T] * w[0]
        for kw in range(1, 7):
            y = (y + xp[kw:kw + T] * w[kw]).astype(np.float32)
        y = (y + W[p + "dwconv.bias"]).astype(np.float32)
        y64 = y.astype(np.float64)
        mean = y64.mean(axis=1, keepdims=True)
        var = ((y64 - mean) ** 2).mean(axis=1, keepdims=True)
        y = (((y64 - mean) / np.sqrt(var + 1e-6)).astype(np.float32) * W[p + "norm.weight"] + W[p + "norm.bias"]).astype(np.float32)
        h = gelu_erf(mm(y, W[p + "pwconv1.weight"], W[p + "pwconv1.bias"]))
        gx = np.sqrt((h.astype(np.float64) ** 2).sum(axis=0)).astype(np.float32)
        nx = (gx / (np.float32(gx.astype(np.float64).mean()) + np.float32(1e-6))).astype(np.float32)
        g = W[p + "grn.gamma"].reshape(-1)
        bt = W[p + "grn.beta"].reshape(-1)
        h = (g * (h * nx) + bt + h).astype(np.float32)
        x = (x + mm(h, W[p + "pwconv2.weight"], W[p + "pwconv2.bias"])).astype(np.float32)
    return x


def prepare(W, prompt_x: np.ndarray, mu: np.ndarray):
    """The static cache: condition and negative condition rows [T][1024] from prompt_x [100][T], mu [512][T]."""
    tx = text_embed(W, mu)
    T = tx.shape[0]
    wc, bc = W["dit.input_embed.proj.weight_ctx"], W["dit.input_embed.proj.bias"]
    cat = np.concatenate([prompt_x.T.astype(np.float32), tx], axis=1)
    zcat = np.concatenate([np.zeros((T, 100), np.float32), tx], axis=1)
    return mm(cat, wc, bc), mm(zcat, wc, bc)


class Rng:
    """gsv_rng (src/gsv_sampler.h:33-40): xorshift64*, uniform01 = (next >> 40) / 2^24."""

    def __init__(self, seed: int):
        self.s = seed if seed else 1

    def next(self) -> int:
        s = self.s
        s ^= s >> 12
        s ^= (s << 25) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 27
        self.s = s
        return (s * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF

    def uniform01(self) -> np.float32:
        return np.float32((self.next() >> 40) * (1.0 / 16777216.0))


def noise(seed: int, n: int) -> np.ndarray:
    """randn01 * 0.875 for n values (src/gsv_dit.cpp:1403-1408, 1436-1438): Box-Muller in float."""
    r = Rng(seed if seed else 1)
    out = np.empty(n, np.float32)
    for i in range(n):
        u1 = r.uniform01()
        u2 = r.uniform01()
        if u1 < np.float32(1e-30):
            u1 = np.float32(1e-30)
        v = np.sqrt(np.float32(-2.0) * np.log(u1)) * np.cos(np.float32(6.283185307179586) * u2)
        out[i] = np.float32(v) * np.float32(0.875)
    return out


def sample_full(W, mu, prompt, P, steps, cfg, seed, x0=None, skip_steps=0):
    """gsv_dit::sample: mu [512][T], prompt [100][P] -> mel [100][T - P]."""
    T = mu.shape[1]
    prompt_x = np.zeros((100, T), np.float32)
    prompt_x[:, :P] = prompt
    cond, neg = prepare(W, prompt_x, mu)
    if x0 is None:
        x0 = noise(seed, 100 * T).reshape(100, T)
    return sample(W, x0, cond, neg, P, steps, cfg, skip_steps=skip_steps)


def synthesize(W, fea_ref, fea_todo, mel_ref, steps, cfg, seed, block_override=0, skip_steps=0):
    """gsv_dit::synthesize (src/gsv_dit.cpp:1480-1581): chunked sampling with a rolling prompt -> mel [100][N]."""
    REF, TAIL, TOTAL, MAXCHUNK = 500, 32, 1000, 640
    R, N, MT = fea_ref.shape[1], fea_todo.shape[1], mel_ref.shape[1]
    common = min(MT, R)
    off = common - REF if common > REF else 0
    rf = common - off
    chunk = min(TOTAL - rf, block_override if block_override > 0 else MAXCHUNK)
    mel_s = mel_ref[:, off:off + rf].astype(np.float32)
    fea_s = fea_ref[:, off:off + rf].astype(np.float32)
    roll_mel, roll_fea = mel_s, fea_s
    out = np.zeros((100, N), np.float32)
    cseed = seed
    for start in range(0, N, chunk):
        tlen = min(chunk, N - start)
        if start == 0:
            prompt, feat = mel_s, fea_s
        else:
            tail = min(TAIL, rf, roll_mel.shape[1], roll_fea.shape[1])
            prompt = np.concatenate([mel_s[:, :rf - tail], roll_mel[:, roll_mel.shape[1] - tail:]], axis=1)
            feat = np.concatenate([fea_s[:, :rf - tail], roll_fea[:, roll_fea.shape[1] - tail:]], axis=1)
        mu = np.concatenate([feat, fea_todo[:, start:start + tlen]], axis=1).astype(np.float32)
        gen = sample_full(W, mu, prompt, rf, steps, cfg, cseed, skip_steps=skip_steps if start == 0 else 0)
        cseed = (cseed * 6364136223846793005 + 1442695040888963407) % 2 ** 64
        out[:, start:start + tlen] = gen
        keep = min(rf, tlen)
        roll_mel = gen[:, tlen - keep:]
        roll_fea = fea_todo[:, start + tlen - keep:start + tlen].astype(np.float32)
    return out


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
