"""Failure paths of the library, with no GPU fault: host-side rejections, exhausted slots and device
memory, and a bounded device-side wait that runs out.

The reference exits the process when its KV cache cannot be allocated (src/gsv_ar.cpp:111) and reads
out of range on bad ids. The library instead returns a status code from every entry point and keeps
the context usable afterwards; each test checks that a valid call right after the failure still gives
the oracle's tokens.
"""
import numpy as np
import pytest

import gsv_synth as S
import oracle as O

pytestmark = pytest.mark.gpu

ERR_ARG, ERR_CUDA, ERR_OOM = -1, -2, -3


@pytest.fixture(scope="module")
def small(model_small):
    import gsvcu
    c = gsvcu.Context(0)
    c.load(model_small)
    yield c, O.OracleModel(model_small)
    c.close()


def _req(rng, T=20, P=8):
    return S.make_request(rng, T, P)


def _still_works(ctx, orc, kv=1):
    """A valid generate right after a failure equals the oracle."""
    ctx.release_cache()
    ctx.kv_reserve(8, 256, kv)
    rng = np.random.default_rng(5)
    reqs = [_req(rng), _req(rng, 30, 12)]
    got, glens = ctx.generate(reqs, seeds=[11, 12], max_steps=24)
    ref, rlens = orc.generate(reqs, seeds=[11, 12], max_steps=24, kv_f16=(kv == 0))
    assert glens == rlens
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)


def _code(excinfo):
    return excinfo.value.code


def test_out_of_range_ids_are_rejected(small):
    import gsvcu
    ctx, orc = small
    ctx.release_cache()
    ctx.kv_reserve(8, 256, 1)
    rng = np.random.default_rng(1)
    bad_phone = _req(rng)
    bad_phone.phones[3] = 732                      # phoneme vocabulary is 732
    bad_code = _req(rng)
    bad_code.prompt[2] = 1025                      # semantic vocabulary is 1025
    for r, what in ((bad_phone, "phone id"), (bad_code, "prompt code")):
        with pytest.raises(gsvcu.GsvcuError) as e:
            ctx.generate([r], max_steps=8)
        assert _code(e) == ERR_ARG and what in str(e.value)
        with pytest.raises(gsvcu.GsvcuError) as e:
            ctx.first_logits([r])
        assert _code(e) == ERR_ARG
    with pytest.raises(gsvcu.GsvcuError) as e:     # teacher-forced token outside the vocabulary
        ctx.generate([_req(rng)], max_steps=8, oracle_tokens=np.array([5, 2000, 7], np.int32))
    assert _code(e) == ERR_ARG and "forced token" in str(e.value)
    _still_works(ctx, orc)


def test_contexts_beyond_the_reserve_or_the_pe_table_are_rejected(small):
    import gsvcu
    ctx, orc = small
    ctx.release_cache()
    with pytest.raises(gsvcu.GsvcuError) as e:     # the positional table has 8192 rows
        ctx.kv_reserve(8, 8193, 1)
    assert _code(e) == ERR_ARG
    ctx.kv_reserve(8, 256, 1)
    rng = np.random.default_rng(2)
    with pytest.raises(gsvcu.GsvcuError) as e:     # generate grows the reserve, but not past the PE table
        ctx.generate([_req(rng, 60, 40)], max_steps=8100)
    assert _code(e) == ERR_ARG
    with pytest.raises(gsvcu.GsvcuError) as e:     # serving: 200 prefix + 100 steps > 256 reserved positions
        ctx.serve_admit([_req(rng, 150, 50)], [1], [0], max_steps=100)
    assert _code(e) == ERR_ARG and "reserved context" in str(e.value)
    assert ctx.serve_active() == 0
    _still_works(ctx, orc)


def test_slot_exhaustion_returns_oom(small):
    import gsvcu
    ctx, orc = small
    ctx.release_cache()
    ctx.kv_reserve(8, 256, 0)
    rng = np.random.default_rng(3)
    ctx.serve_admit([_req(rng) for _ in range(8)], list(range(8)), list(range(8)), max_steps=16)
    with pytest.raises(gsvcu.GsvcuError) as e:
        ctx.serve_admit([_req(rng)], [9], [9], max_steps=16)
    assert _code(e) == ERR_OOM and "slot" in str(e.value)
    assert ctx.serve_active() == 8                  # the admitted sequences are untouched
    done = []
    for _ in range(4):
        done += ctx.serve_step(8, tok_cap=10000)
    assert len(done) == 8
    _still_works(ctx, orc, kv=0)


def test_device_memory_exhaustion_returns_oom(small):
    import gsvcu
    ctx, orc = small
    ctx.release_cache()
    with pytest.raises(gsvcu.GsvcuError) as e:     # 4096 slots x 8192 positions of F32 K/V: ~3 TB
        ctx.kv_reserve(4096, 8192, 1)
    assert _code(e) == ERR_OOM
    _still_works(ctx, orc)


@pytest.mark.parametrize("fused", [1, 0])
def test_bounded_kv_wait_gives_up_and_the_context_recovers(small, fused):
    """Fault injection on the host's side of the launch: every decode-attention page wait expects 16 bytes
    more than is staged, with a 4096-poll limit. The waits run out (all copies complete; only the count
    is never reached), the kernels flag it and return, the call reports GSVCU_ERR_CUDA, and after the
    fault is switched off the same context decodes as the oracle again."""
    import gsvcu
    ctx, orc = small
    ctx.set_fused_decode(fused)
    try:
        ctx.release_cache()
        ctx.kv_reserve(8, 256, 1)
        rng = np.random.default_rng(4)
        reqs = [_req(rng, 70, 10)]                  # two K/V pages: partials and the merge run
        ctx.set_wait_fault(True)
        try:
            with pytest.raises(gsvcu.GsvcuError) as e:
                ctx.generate(reqs, seeds=[3], max_steps=20)
            assert _code(e) == ERR_CUDA and "never arrived" in str(e.value)
        finally:
            ctx.set_wait_fault(False)
        _still_works(ctx, orc)
    finally:
        ctx.set_fused_decode(1)


def test_op_entry_wait_timeout_is_reported_by_sync(small):
    import torch
    import gsvcu
    ctx, _ = small
    rng = np.random.default_rng(6)
    B, maxp = 2, 3
    pool = torch.from_numpy(rng.standard_normal((6, 1, 2, 16, 64, 32)).astype(np.float16)).cuda()
    bt = torch.tensor([[0, 1, 2], [3, 4, 5]], dtype=torch.int32, device="cuda")
    q = torch.randn((B, 512), device="cuda")
    kvpos = torch.tensor([150, 40], dtype=torch.int32, device="cuda")
    active = torch.ones(B, dtype=torch.int32, device="cuda")
    oq = torch.empty((B, 512), dtype=torch.int8, device="cuda")
    od = torch.empty((B, 16), dtype=torch.int16, device="cuda")
    ctx.set_wait_fault(True)
    try:
        ctx.op_decode_attention(q, 512, pool, 0, 1, 0, bt, maxp, kvpos, active, B, oq, od)
        with pytest.raises(gsvcu.GsvcuError) as e:
            ctx.sync()
        assert _code(e) == ERR_CUDA
    finally:
        ctx.set_wait_fault(False)
    ctx.op_decode_attention(q, 512, pool, 0, 1, 0, bt, maxp, kvpos, active, B, oq, od)
    ctx.sync()   # reported once, then clear
