"""CPU checks of the DiT restatement (oracle/dit_oracle.py) against the reference's formulas
(src/gsv_dit.cpp, tools/export_gguf/convert_dit.py). The reference DiT needs ggml and ships no golden
vectors, so these pin the restatement to the formulas, not to a run of the reference."""
import math

import numpy as np
import pytest

import dit_oracle as O
import gsv_synth as S


def test_time_sin_formula():
    """SinusPositionEmbedding(256) as src/gsv_dit.cpp:755-769 evaluates it (float32 e, expf, sinf, cosf)."""
    e = np.float32(math.log(10000.0) / 127.0)
    for t in (0.0, 0.25, 0.875):
        ref = np.empty(256, np.float32)
        for i in range(128):
            a = np.float32(np.float32(1000.0) * np.float32(t)) * np.float32(math.exp(-float(e) * i))
            ref[i], ref[128 + i] = math.sin(a), math.cos(a)
        # arguments reach 1000 rad, where one float ulp is 6e-5: libm and numpy may differ by that much
        assert np.allclose(O.time_sin(t), ref, rtol=0, atol=2e-4)
    assert np.array_equal(O.time_sin(0.0)[:128], np.zeros(128, np.float32))


def test_conv_pos_matches_direct_convolution():
    """The grouped conv (16 groups of 64, 31 taps, zero padding 15) with the exporter's weight order
    (inner index ic * 31 + tap) equals torch's conv1d formula evaluated directly."""
    rng = np.random.default_rng(0)
    T = 23
    x = O.f16(rng.standard_normal((T, 1024)).astype(np.float32))
    w = rng.standard_normal((16, 64, 64 * 31)).astype(np.float32)
    b = rng.standard_normal(1024).astype(np.float32)
    got = O.conv_pos(x, w, b)
    wt = w.reshape(16, 64, 64, 31)   # [g][o][ic][tap], torch [OC][ICg][K]
    for g, o in ((0, 0), (5, 17), (15, 63)):
        for t in (0, 7, T - 1):
            acc = 0.0
            for ic in range(64):
                for k in range(31):
                    s = t + k - 15
                    if 0 <= s < T:
                        acc += float(wt[g, o, ic, k]) * float(x[s, g * 64 + ic])
            assert abs(got[t, g * 64 + o] - (acc + b[g * 64 + o])) < 1e-3


def test_rope_rotates_adjacent_pairs_of_head0():
    """RoPE (src/gsv_dit.cpp:191-200): pairs (2i, 2i+1) of the first 64 columns rotated by t * inv_freq[i];
    norms of pairs preserved, identity at t = 0, other heads untouched."""
    rng = np.random.default_rng(1)
    T = 9
    x = rng.standard_normal((T, 1024)).astype(np.float32)
    inv = (1.0 / (10000.0 ** (np.arange(0, 64, 2) / 64.0))).astype(np.float32)
    cs, sn = O.rope_tables(inv, T)
    y = O.rope64(x, cs, sn)
    assert np.array_equal(y[0], x[0]) and np.array_equal(y[:, 64:], x[:, 64:])
    n0 = x[:, 0:64:2] ** 2 + x[:, 1:64:2] ** 2
    n1 = y[:, 0:64:2] ** 2 + y[:, 1:64:2] ** 2
    assert np.allclose(n0, n1, rtol=1e-5)
    t, i = 5, 3
    a = t * inv[i]
    assert np.isclose(y[t, 2 * i], x[t, 2 * i] * math.cos(a) - x[t, 2 * i + 1] * math.sin(a), atol=1e-5)


def test_attention_ignores_padding_keys():
    rng = np.random.default_rng(2)
    T, xl = 40, 29
    q, k, v = (rng.standard_normal((T, 1024)).astype(np.float32) for _ in range(3))
    a = O.attention(q, k, v, xl)
    k2, v2 = k.copy(), v.copy()
    k2[xl:] = 100.0
    v2[xl:] = -100.0
    assert np.array_equal(a, O.attention(q, k2, v2, xl))


def test_synthetic_dit_has_exporter_layout(tmp_path):
    """The synthetic file carries the exporter's names, shapes (torch order) and KV keys for every tensor
    the estimator reads (tools/export_gguf/convert_dit.py:120-150)."""
    p = S.write_dit_model(str(tmp_path / "d.gguf"), seed=3, depth=1)
    W = O.load(p)
    assert W["depth"] == 1
    assert W["dit.input_embed.proj.weight_mel"].shape == (1024, 100)
    assert W["dit.input_embed.conv_pos_embed.conv1d.0.weight"].shape == (16, 64, 64 * 31)
    assert W["dit.transformer_blocks.0.attn_norm.linear.weight"].shape == (6144, 1024)
    assert W["dit.transformer_blocks.0.ff.ff.2.weight"].shape == (1024, 2048)
    assert W["dit.norm_out.linear.weight"].shape == (2048, 1024)
    assert W["dit.proj_out.weight"].shape == (100, 1024)
    assert W["dit.rotary_embed.inv_freq"].shape == (32,)


@pytest.mark.parametrize("cfg", [0.0, 1.5])
def test_sample_zeroes_prompt_and_steps(tmp_path, cfg):
    """The Euler loop keeps the prompt frames at zero and, with zero velocity weights, leaves x0."""
    p = S.write_dit_model(str(tmp_path / "d.gguf"), seed=4, depth=1)
    W = O.load(p)
    W["dit.proj_out.weight"][:] = 0
    W["dit.proj_out.bias"][:] = 0
    rng = np.random.default_rng(5)
    T, P = 30, 7
    x0 = rng.standard_normal((100, T)).astype(np.float32)
    cond = rng.standard_normal((T, 1024)).astype(np.float32)
    out = O.sample(W, x0, cond, cond, P, 2, cfg)
    assert np.array_equal(out, x0[:, P:])


def test_seeded_noise_follows_gsv_rng():
    """x0 = randn01 * 0.875 from gsv_rng (src/gsv_sampler.h:33-40, src/gsv_dit.cpp:1403-1408): the first
    values from the xorshift64* formula written out here, and the distribution."""
    s = 99
    def nxt():
        nonlocal s
        s ^= s >> 12
        s ^= (s << 25) & (2 ** 64 - 1)
        s ^= s >> 27
        return (s * 0x2545F4914F6CDD1D) % 2 ** 64
    u1 = np.float32((nxt() >> 40) / 16777216.0)
    u2 = np.float32((nxt() >> 40) / 16777216.0)
    v = np.float32(math.sqrt(-2.0 * math.log(u1)) * math.cos(6.283185307179586 * u2) * 0.875)
    z = O.noise(99, 20000)
    assert abs(z[0] - v) < 1e-5
    assert abs(float(z.std()) - 0.875) < 0.02 and abs(float(z.mean())) < 0.02


def test_prepare_negative_drops_the_prompt(tmp_path):
    """The negative condition is the projection of [0 | text]: it does not depend on the prompt frames."""
    p = S.write_dit_model(str(tmp_path / "d.gguf"), seed=6, depth=1)
    W = O.load(p)
    rng = np.random.default_rng(7)
    T = 40
    mu = rng.standard_normal((512, T)).astype(np.float32)
    a = O.prepare(W, rng.standard_normal((100, T)).astype(np.float32), mu)
    b = O.prepare(W, np.zeros((100, T), np.float32), mu)
    assert np.array_equal(a[1], b[1]) and np.array_equal(b[0], b[1]) and not np.array_equal(a[0], b[0])


def test_synthesize_single_chunk_is_one_sample(tmp_path):
    """synthesize with one chunk (N <= block) is sample() on [reference features | target features] with the
    reference mel as prompt and the given seed; the reference frames are the last 500 of the common length."""
    p = S.write_dit_model(str(tmp_path / "d.gguf"), seed=8, depth=1)
    W = O.load(p)
    rng = np.random.default_rng(9)
    fea_ref = rng.standard_normal((512, 34)).astype(np.float32)
    fea_todo = rng.standard_normal((512, 20)).astype(np.float32)
    mel_ref = rng.standard_normal((100, 30)).astype(np.float32)
    out = O.synthesize(W, fea_ref, fea_todo, mel_ref, 2, 1.5, 5, block_override=64)
    mu = np.concatenate([fea_ref[:, :30], fea_todo], axis=1)
    ref = O.sample_full(W, mu, mel_ref, 30, 2, 1.5, 5)
    assert np.array_equal(out, ref)
