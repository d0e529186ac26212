"""The allocation-free decode attention entry point (gsvcu_op_decode_attention_noalloc).

It exists for callers of this library that may not allocate device memory where they run attention
(a framework's caching allocator owning the device, a real-time callback that must not block in the
driver's allocator, an embedder that forbids allocations after start-up). Its split-KV scratch is a
fixed array inside the library instead of memory obtained with cudaMalloc. This file is collected
last on purpose; it passes alone in a fresh process as well as after the other tests.

Checked: through the C ABI, on two calls in a row (the shared scratch keeps the first call's
contents), its outputs equal those of gsvcu_op_decode_attention on the same inputs, bit for bit --
the tolerance the decode-attention parity test holds that kernel to -- for F16 and F32 KV pools with
multi-chunk sequences; at exactly the scratch's capacity (16 sequences x 64 pages, some at the last
key) it is accepted and also equals the oracle bit for bit; sizes beyond the fixed scratch are rejected.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _inputs(rng, lens, kv_dtype, n_layer=2):
    PAGE = 64
    B = len(lens)
    maxp = max((l + PAGE - 1) // PAGE for l in lens) + 1
    npages = sum((l + PAGE - 1) // PAGE for l in lens) + 2
    dt = np.float16 if kv_dtype == 0 else np.float32
    pool = rng.standard_normal((npages, n_layer, 2, 16, PAGE, 32)).astype(dt)
    perm = rng.permutation(npages)
    bt = np.zeros((B, maxp), np.int32)
    at = 0
    for b, l in enumerate(lens):
        for p in range((l + PAGE - 1) // PAGE):
            bt[b, p] = perm[at]
            at += 1
    q = rng.standard_normal((B, 1536)).astype(np.float32)
    kvpos = np.array(lens, np.int32) - 1
    active = np.ones(B, np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(q=t(q), pool=t(pool), bt=t(bt), maxp=maxp, kvpos=t(kvpos), active=t(active), B=B, n_layer=n_layer)


def _outs(B):
    return (torch.full((B, 512), 55, dtype=torch.int8, device="cuda"),
            torch.zeros((B, 16), dtype=torch.int16, device="cuda"),
            torch.full((B, 512), -7.0, dtype=torch.float32, device="cuda"))


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_noalloc_matches_existing_entry_point_twice(kv_dtype):
    import gsvcu
    lib = gsvcu.load_library()
    ctx = gsvcu.Context(0)
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((100 + kv_dtype, 200 + kv_dtype)):   # two calls in a row
        rng = np.random.default_rng(seed)
        lens = [1, 70, 256, 257, 900, 1500] if call == 0 else [2049, 33, 512, 511, 1100]
        x = _inputs(rng, lens, kv_dtype)
        B = x["B"]
        ref_q, ref_d, ref_f = _outs(B)
        ctx.op_decode_attention(x["q"], 1536, x["pool"], kv_dtype, x["n_layer"], 1, x["bt"], x["maxp"], x["kvpos"],
                                x["active"], B, ref_q, ref_d, ref_f)
        ctx.sync()
        got_q, got_d, got_f = _outs(B)
        p = lambda a: C.c_void_p(a.data_ptr())
        rc = lib.gsvcu_op_decode_attention_noalloc(C.c_void_p(stream), p(x["q"]), 1536, p(x["pool"]), kv_dtype,
                                                   x["n_layer"], 1, p(x["bt"]), x["maxp"], p(x["kvpos"]),
                                                   p(x["active"]), B, p(got_q), p(got_d), p(got_f))
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(got_f.view(torch.int32), ref_f.view(torch.int32)), call
        assert torch.equal(got_q, ref_q) and torch.equal(got_d, ref_d), call
    ctx.close()


def test_noalloc_at_full_capacity_matches_oracle():
    """B x max_pages exactly at the limit (16 x 64 = GSVCU_NOALLOC_MAX_ITEMS), several sequences at the
    last key the block table holds: accepted, equal to gsvcu_op_decode_attention and to the oracle bit for
    bit (the kernels and the oracle share one fixed float order), twice in a row."""
    import gsvcu
    import oracle as O
    lib = gsvcu.load_library()
    ctx = gsvcu.Context(0)
    stream = torch.cuda.current_stream().cuda_stream
    B, maxp, n_layer, layer = 16, 64, 2, 1
    for call in range(2):
        rng = np.random.default_rng(300 + call)
        lens = [maxp * 64] * 4 + [int(l) for l in rng.integers(1, maxp * 64 + 1, B - 4)]
        npages = B * maxp
        pool = rng.standard_normal((npages, n_layer, 2, 16, 64, 32)).astype(np.float16)
        bt = rng.permutation(npages).astype(np.int32).reshape(B, maxp)
        q = rng.standard_normal((B, 512)).astype(np.float32)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        x = dict(q=t(q), pool=t(pool), bt=t(bt), kvpos=t(np.array(lens, np.int32) - 1), active=t(np.ones(B, np.int32)))
        ref_q, ref_d, ref_f = _outs(B)
        ctx.op_decode_attention(x["q"], 512, x["pool"], 0, n_layer, layer, x["bt"], maxp, x["kvpos"], x["active"], B,
                                ref_q, ref_d, ref_f)
        ctx.sync()
        got_q, got_d, got_f = _outs(B)
        p = lambda a: C.c_void_p(a.data_ptr())
        rc = lib.gsvcu_op_decode_attention_noalloc(C.c_void_p(stream), p(x["q"]), 512, p(x["pool"]), 0, n_layer, layer,
                                                   p(x["bt"]), maxp, p(x["kvpos"]), p(x["active"]), B, p(got_q),
                                                   p(got_d), p(got_f))
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(got_f.view(torch.int32), ref_f.view(torch.int32)), call
        assert torch.equal(got_q, ref_q) and torch.equal(got_d, ref_d), call
        Lmax = max(lens)
        kk = np.zeros((B, Lmax, 16, 32), np.float32)
        vv = np.zeros((B, Lmax, 16, 32), np.float32)
        for b, l in enumerate(lens):
            pages = pool[bt[b, :(l + 63) // 64], layer].astype(np.float32)     # [pages][K,V][16][64][32]
            kk[b, :l] = pages[:, 0].transpose(0, 2, 1, 3).reshape(-1, 16, 32)[:l]
            vv[b, :l] = pages[:, 1].transpose(0, 2, 1, 3).reshape(-1, 16, 32)[:l]
        want = O.decode_attention(q.reshape(B, 16, 32), kk, vv, np.array(lens, np.int32),
                                  1.0 / np.sqrt(np.float32(32))).reshape(B, 512)
        assert np.array_equal(got_f.cpu().numpy().view(np.uint32), want.view(np.uint32)), call
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import gsvcu
    lib = gsvcu.load_library()
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    # B x max_pages must stay within 1024 sequence-pages: 64 x 80 does not fit
    rc = lib.gsvcu_op_decode_attention_noalloc(None, p, 1536, p, 0, 1, 0, p, 80, p, p, 64, p, p, None)
    assert rc == -1
    # nor does 64 x 17 = 1088 (F32 pool)
    rc = lib.gsvcu_op_decode_attention_noalloc(None, p, 1536, p, 1, 1, 0, p, 17, p, p, 64, p, p, None)
    assert rc == -1
    # nor 1025 sequences of one page
    rc = lib.gsvcu_op_decode_attention_noalloc(None, p, 1536, p, 0, 1, 0, p, 1, p, p, 1025, p, p, None)
    assert rc == -1
